/*
 * gen.c — seeded test generators, block formats and the scalar dequantizer.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h).
 */
#include <math.h>
#include <string.h>

#include "sg_oracle.h"

static uint32_t f32_bits(float v) { uint32_t b; memcpy(&b, &v, 4); return b; }
static float bits_f32(uint32_t b) { float v; memcpy(&v, &b, 4); return v; }

/* xorshift64 step of the tests' `Rng::next` (quant_q8k.rs:302-309). */
uint64_t or_rng_next(uint64_t *s)
{
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return x;
}

/* `Rng::f`: lo + (hi - lo) * (top 24 bits / 2^24), all in f32 (quant_q8k.rs:310-312). */
float or_rng_f(uint64_t *s, float lo, float hi)
{
    float unit = (float)(or_rng_next(s) >> 40) / 16777216.0f;
    float span = hi - lo;
    float scaled = span * unit;
    return lo + scaled;
}

void or_rng_fill_f32(uint64_t *s, float lo, float hi, float *out, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = or_rng_f(s, lo, hi);
}

/* Truncating f32 -> f16 of the tests (quant_q8k.rs:315-321): the exponent is
 * re-biased with 16-bit wrap-around and the mantissa truncated. */
uint16_t or_f16_trunc(float v)
{
    uint32_t b = f32_bits(v);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    uint16_t exp = (uint16_t)((int32_t)((b >> 23) & 0xffu) - 127 + 15);
    uint16_t mant = (uint16_t)((b >> 13) & 0x3ffu);
    return (uint16_t)(sign | (uint16_t)(exp << 10) | mant);
}

/* Variant of quant.rs:1680-1690: magnitudes below the smallest normal half
 * become a signed zero. */
uint16_t or_f16_trunc_flush(float v)
{
    uint32_t b = f32_bits(v);
    if (fabsf(v) < 6.1035156e-5f) return (uint16_t)((b >> 16) & 0x8000u);
    return or_f16_trunc(v);
}

/* IEEE half -> float, exact for every input (quant.rs:877-899 f16_to_f32_exact,
 * which equals the F16C conversion the kernels use). */
float or_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = 127 - 14;
            while (!(mant & 0x400u)) { mant <<= 1; e--; }
            bits = sign | ((uint32_t)e << 23) | ((mant & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    return bits_f32(bits);
}

static float rd16(const uint8_t *p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

static void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* Bytes per row (quant.rs:1527-1542): -1 for an unsupported type or width. */
int64_t or_row_bytes(int32_t dtype, uint64_t cols)
{
    uint64_t blk, bytes;
    switch (dtype) {
    case OR_F32: blk = 1; bytes = 4; break;
    case OR_F16: case OR_BF16: blk = 1; bytes = 2; break;
    case OR_Q4_0: blk = 32; bytes = 18; break;
    case OR_Q4_1: blk = 32; bytes = 20; break;
    case OR_Q5_0: blk = 32; bytes = 22; break;
    case OR_Q5_1: blk = 32; bytes = 24; break;
    case OR_Q8_0: blk = 32; bytes = 34; break;
    case OR_Q4_K: blk = 256; bytes = 144; break;
    case OR_Q5_K: blk = 256; bytes = 176; break;
    case OR_Q6_K: blk = 256; bytes = 210; break;
    default: return -1;
    }
    if (cols % blk) return -1;
    return (int64_t)(cols / blk * bytes);
}

/* Q4_K 12-byte scale block -> 8 six-bit scales and 8 six-bit mins
 * (q4k_gemv.rs:75-85). */
void or_unpack_q4k_scales(const uint8_t p[12], uint8_t sc[8], uint8_t mn[8])
{
    for (int j = 0; j < 4; j++) {
        sc[j] = p[j] & 63;
        mn[j] = p[j + 4] & 63;
        sc[j + 4] = (uint8_t)((p[j + 8] & 0x0f) | ((p[j] >> 6) << 4));
        mn[j + 4] = (uint8_t)((p[j + 8] >> 4) | ((p[j + 4] >> 6) << 4));
    }
}

/* random_matrix (quant_q8k.rs:323-336; Q8_0/F32 arms from quant_multi.rs:301-322):
 * random bytes, then every scale field set to a truncated f16 of U(0.001, 0.05). */
int or_random_matrix(int32_t dtype, size_t cols, size_t rows, uint64_t *rng, uint8_t *out)
{
    int64_t rb = or_row_bytes(dtype, cols);
    if (rb < 0) return -1;
    size_t total = (size_t)rb * rows;
    for (size_t i = 0; i < total; i++) out[i] = (uint8_t)or_rng_next(rng);
    size_t bb;
    size_t offs[2];
    int n_offs;
    switch (dtype) {
    case OR_Q8_0: bb = 34; offs[0] = 0; n_offs = 1; break;
    case OR_Q4_K: bb = 144; offs[0] = 0; offs[1] = 2; n_offs = 2; break;
    case OR_Q6_K: bb = 210; offs[0] = 208; n_offs = 1; break;
    case OR_F32:
        for (size_t i = 0; i + 4 <= total; i += 4) {
            float v = or_rng_f(rng, -1.0f, 1.0f);
            memcpy(out + i, &v, 4);
        }
        return 0;
    default: return -1;
    }
    for (size_t b = 0; b + bb <= total; b += bb)
        for (int k = 0; k < n_offs; k++)
            put16(out + b + offs[k], or_f16_trunc(or_rng_f(rng, 0.001f, 0.05f)));
    return 0;
}

/* random_row (quant.rs:1693-1723): random bytes with sane scale fields, for
 * every format of the float-kernel test. */
int or_random_row(int32_t dtype, size_t cols, uint64_t *rng, uint8_t *out)
{
    int64_t len = or_row_bytes(dtype, cols);
    if (len < 0) return -1;
    for (int64_t i = 0; i < len; i++) out[i] = (uint8_t)or_rng_next(rng);
    size_t bb;
    size_t offs[2];
    int n_offs;
    switch (dtype) {
    case OR_Q8_0: case OR_Q4_0: case OR_Q5_0:
        bb = (size_t)or_row_bytes(dtype, 32); offs[0] = 0; n_offs = 1; break;
    case OR_Q4_1: case OR_Q5_1:
        bb = (size_t)or_row_bytes(dtype, 32); offs[0] = 0; offs[1] = 2; n_offs = 2; break;
    case OR_Q4_K: case OR_Q5_K:
        bb = (size_t)or_row_bytes(dtype, 256); offs[0] = 0; offs[1] = 2; n_offs = 2; break;
    case OR_Q6_K: bb = 210; offs[0] = 208; n_offs = 1; break;
    case OR_F16: bb = 2; offs[0] = 0; n_offs = 1; break;
    case OR_BF16:
        for (int64_t i = 0; i + 2 <= len; i += 2)
            put16(out + i, (uint16_t)(f32_bits(or_rng_f(rng, -1.0f, 1.0f)) >> 16));
        return 0;
    case OR_F32:
        for (int64_t i = 0; i + 4 <= len; i += 4) {
            float v = or_rng_f(rng, -1.0f, 1.0f);
            memcpy(out + i, &v, 4);
        }
        return 0;
    default: return -1;
    }
    for (size_t b = 0; b + bb <= (size_t)len; b += bb)
        for (int k = 0; k < n_offs; k++) {
            float v = dtype == OR_F16 ? or_rng_f(rng, -1.0f, 1.0f) : or_rng_f(rng, 0.001f, 0.05f);
            put16(out + b + offs[k], or_f16_trunc_flush(v));
        }
    return 0;
}

/* Scalar dequantization of one row straight from the format definitions
 * (quant.rs:1551-1660).  Every product is rounded separately, left to right. */
int or_dequant_row(int32_t dtype, const uint8_t *row, size_t cols, float *y)
{
    if (or_row_bytes(dtype, cols) < 0) return -1;
    switch (dtype) {
    case OR_F32:
        memcpy(y, row, cols * 4);
        return 0;
    case OR_F16:
        for (size_t i = 0; i < cols; i++) y[i] = rd16(row + 2 * i);
        return 0;
    case OR_BF16:
        for (size_t i = 0; i < cols; i++)
            y[i] = bits_f32((uint32_t)(row[2 * i] | (row[2 * i + 1] << 8)) << 16);
        return 0;
    case OR_Q8_0:
        for (size_t b = 0; b < cols / 32; b++) {
            const uint8_t *blk = row + b * 34;
            float d = rd16(blk);
            for (int j = 0; j < 32; j++) y[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
        return 0;
    case OR_Q4_0: case OR_Q4_1: case OR_Q5_0: case OR_Q5_1: {
        int has_m = dtype == OR_Q4_1 || dtype == OR_Q5_1;
        int has_h = dtype == OR_Q5_0 || dtype == OR_Q5_1;
        size_t size = (size_t)or_row_bytes(dtype, 32);
        int center = has_m ? 0 : (has_h ? 16 : 8);
        for (size_t b = 0; b < cols / 32; b++) {
            const uint8_t *blk = row + b * size;
            float d = rd16(blk);
            float m = has_m ? rd16(blk + 2) : 0.0f;
            size_t p = has_m ? 4 : 2;
            uint32_t qh = 0;
            if (has_h) {
                qh = (uint32_t)blk[p] | ((uint32_t)blk[p + 1] << 8) | ((uint32_t)blk[p + 2] << 16) |
                     ((uint32_t)blk[p + 3] << 24);
                p += 4;
            }
            const uint8_t *qs = blk + p;
            for (int j = 0; j < 16; j++) {
                int lo = qs[j] & 0x0f, hi = qs[j] >> 4;
                if (has_h) {
                    lo |= (int)(((qh >> j) & 1u) << 4);
                    hi |= (int)(((qh >> (j + 16)) & 1u) << 4);
                }
                float a = (float)(lo - center) * d;
                float c = (float)(hi - center) * d;
                y[b * 32 + j] = a + m;
                y[b * 32 + j + 16] = c + m;
            }
        }
        return 0;
    }
    case OR_Q4_K: case OR_Q5_K: {
        size_t size = dtype == OR_Q4_K ? 144 : 176;
        for (size_t b = 0; b < cols / 256; b++) {
            const uint8_t *blk = row + b * size;
            float d = rd16(blk), dmin = rd16(blk + 2);
            uint8_t sc[8], mn[8];
            or_unpack_q4k_scales(blk + 4, sc, mn);
            const uint8_t *qh = blk + 16;
            const uint8_t *qs = size == 176 ? blk + 48 : blk + 16;
            float *out = y + b * 256;
            for (int c = 0; c < 4; c++)
                for (int l = 0; l < 32; l++) {
                    uint32_t q = qs[c * 32 + l];
                    uint32_t lo = q & 0x0f, hi = q >> 4;
                    if (size == 176) {
                        lo |= ((uint32_t)(qh[l] >> (2 * c)) & 1u) << 4;
                        hi |= ((uint32_t)(qh[l] >> (2 * c + 1)) & 1u) << 4;
                    }
                    float s0 = d * (float)sc[2 * c], o0 = dmin * (float)mn[2 * c];
                    float s1 = d * (float)sc[2 * c + 1], o1 = dmin * (float)mn[2 * c + 1];
                    float w0 = s0 * (float)lo, w1 = s1 * (float)hi;
                    out[c * 64 + l] = w0 - o0;
                    out[c * 64 + 32 + l] = w1 - o1;
                }
        }
        return 0;
    }
    case OR_Q6_K:
        for (size_t b = 0; b < cols / 256; b++) {
            const uint8_t *blk = row + b * 210;
            float d = rd16(blk + 208);
            for (int half = 0; half < 2; half++) {
                const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
                const int8_t *sc = (const int8_t *)(blk + 192 + half * 8);
                float *out = y + b * 256 + half * 128;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    int q1 = ((ql[l] & 0xf) | ((qh[l] & 3) << 4)) - 32;
                    int q2 = ((ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    out[l] = (d * (float)sc[is]) * (float)q1;
                    out[l + 32] = (d * (float)sc[is + 2]) * (float)q2;
                    out[l + 64] = (d * (float)sc[is + 4]) * (float)q3;
                    out[l + 96] = (d * (float)sc[is + 6]) * (float)q4;
                }
            }
        }
        return 0;
    default:
        return -1;
    }
}
