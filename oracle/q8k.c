/*
 * q8k.c — the integer K-quant path of spindle (quant_q8k.rs), restated.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h).  Compiled with
 * -mavx2 -mfma -mf16c -ffp-contract=off so that each float operation below is
 * the same single x86 instruction the reference executes.
 */
#include <immintrin.h>
#include <math.h>
#include <string.h>

#include "sg_oracle.h"

#define AVX __attribute__((target("avx2,fma,f16c")))
#define INL __attribute__((always_inline)) inline

AVX static INL float half_at(const uint8_t *p)
{
    return _cvtsh_ss((unsigned short)(p[0] | (p[1] << 8)));
}

/* Q8K::quantize / quantize_avx2 (quant_q8k.rs:73-121).
 * amax: 8 running lane maxima over x[j], x[j+8], ... (MAXPS keeps its second
 * operand on a NaN), folded hi->lo, 2->0, 1->0.  d = amax/127, and each value
 * becomes cvtps_epi32(x * (127/amax)) (round-to-nearest-even; NaN and
 * out-of-range give INT32_MIN) saturated to int8 by the two packs. */
AVX void or_q8k_quantize(const float *x, size_t n, float *d, int8_t *qs, int16_t *bsums)
{
    const __m256 abs_mask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7fffffff));
    for (size_t b = 0; b < n / 256; b++) {
        const float *xb = x + b * 256;
        __m256 lane_max = _mm256_setzero_ps();
        for (int j = 0; j < 256; j += 8)
            lane_max = _mm256_max_ps(lane_max, _mm256_and_ps(abs_mask, _mm256_loadu_ps(xb + j)));
        __m128 v = _mm_max_ps(_mm256_castps256_ps128(lane_max), _mm256_extractf128_ps(lane_max, 1));
        v = _mm_max_ps(v, _mm_movehl_ps(v, v));
        v = _mm_max_ss(v, _mm_shuffle_ps(v, v, 0x55));
        float amax = _mm_cvtss_f32(v);
        int8_t *q = qs + b * 256;
        int16_t *bs = bsums + b * 16;
        if (!(amax > 0.0f) || !isfinite(amax)) {
            d[b] = 0.0f;
            memset(q, 0, 256);
            memset(bs, 0, 32);
            continue;
        }
        const __m256 inv = _mm256_set1_ps(127.0f / amax);
        d[b] = amax / 127.0f;
        for (int j = 0; j < 256; j += 8) {
            int32_t t[8];
            _mm256_storeu_si256((__m256i *)t, _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(xb + j), inv)));
            for (int k = 0; k < 8; k++)
                q[j + k] = (int8_t)(t[k] > 127 ? 127 : (t[k] < -128 ? -128 : t[k]));
        }
        for (int g = 0; g < 16; g++) {
            int16_t s = 0;
            for (int k = 0; k < 16; k++) s = (int16_t)(s + q[g * 16 + k]);
            bs[g] = s;
        }
    }
}

/* hsum of quant_q8k.rs:153-158: (l0+l4, l1+l5, l2+l6, l3+l7) -> (a0+a2, a1+a3) -> sum. */
AVX static INL float hsum_q8k(__m256 v)
{
    __m128 x = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    x = _mm_add_ps(x, _mm_movehl_ps(x, x));
    x = _mm_add_ss(x, _mm_shuffle_ps(x, x, 0x55));
    return _mm_cvtss_f32(x);
}

/* Decoded super-block: 8 x 32 unsigned weight bytes (chunk k covers weights
 * 32k..32k+31), 8 int16 scale vectors and the float scales. */
typedef struct {
    __m256i w[8];
    __m256i sv[8];
    float d, dmin;
    uint8_t mn[8];
    const int8_t *sc6;
} blk_t;

/* Q4_K (q4k_gemv.rs:26-31): chunk 2c = low nibbles of qs[32c..32c+32], chunk
 * 2c+1 = high nibbles, scales from the 12-byte packed field. */
AVX static INL void decode_q4k(const uint8_t *blk, blk_t *o)
{
    const __m256i lo4 = _mm256_set1_epi8(0x0f);
    uint8_t sc[8];
    o->d = half_at(blk);
    o->dmin = half_at(blk + 2);
    or_unpack_q4k_scales(blk + 4, sc, o->mn);
    for (int c = 0; c < 4; c++) {
        __m256i v = _mm256_loadu_si256((const __m256i *)(blk + 16 + 32 * c));
        o->w[2 * c] = _mm256_and_si256(v, lo4);
        o->w[2 * c + 1] = _mm256_and_si256(_mm256_srli_epi16(v, 4), lo4);
        o->sv[2 * c] = _mm256_set1_epi16(sc[2 * c]);
        o->sv[2 * c + 1] = _mm256_set1_epi16(sc[2 * c + 1]);
    }
}

/* Q6_K (quant.rs:34-39): per half h, chunks 4h..4h+3 take low/high nibbles of
 * ql[64h..64h+32] and ql[64h+32..64h+64] plus 2-bit fields of qh[32h..]; the
 * first 16 bytes of chunk 4h+k use scale 8h+2k, the last 16 use 8h+2k+1. */
AVX static INL void decode_q6k(const uint8_t *blk, blk_t *o)
{
    const __m256i lo4 = _mm256_set1_epi8(0x0f), lo2 = _mm256_set1_epi8(3);
    const int8_t *sc = (const int8_t *)(blk + 192);
    o->d = half_at(blk + 208);
    o->sc6 = sc;
    for (int h = 0; h < 2; h++) {
        __m256i a = _mm256_loadu_si256((const __m256i *)(blk + 64 * h));
        __m256i b = _mm256_loadu_si256((const __m256i *)(blk + 64 * h + 32));
        __m256i hb = _mm256_loadu_si256((const __m256i *)(blk + 128 + 32 * h));
        __m256i h0 = _mm256_slli_epi16(_mm256_and_si256(hb, lo2), 4);
        __m256i h1 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 2), lo2), 4);
        __m256i h2 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 4), lo2), 4);
        __m256i h3 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 6), lo2), 4);
        o->w[4 * h + 0] = _mm256_or_si256(_mm256_and_si256(a, lo4), h0);
        o->w[4 * h + 1] = _mm256_or_si256(_mm256_and_si256(b, lo4), h1);
        o->w[4 * h + 2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(a, 4), lo4), h2);
        o->w[4 * h + 3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(b, 4), lo4), h3);
        for (int k = 0; k < 4; k++)
            o->sv[4 * h + k] = _mm256_setr_m128i(_mm_set1_epi16(sc[8 * h + 2 * k]),
                                                 _mm_set1_epi16(sc[8 * h + 2 * k + 1]));
    }
}

/* Lane sums: lane l = sum_k scale_k(l) * sum_{j=4l..4l+3} w[k][j] * y[32k+j]
 * via u8 x i8 -> i16 pairs (maddubs) and i16 x i16 -> i32 pairs (madd). */
AVX static INL __m256i lane_sums(const blk_t *o, const int8_t *y)
{
    __m256i s = _mm256_setzero_si256();
    for (int k = 0; k < 8; k++) {
        __m256i p = _mm256_maddubs_epi16(o->w[k], _mm256_loadu_si256((const __m256i *)(y + 32 * k)));
        s = _mm256_add_epi32(s, _mm256_madd_epi16(p, o->sv[k]));
    }
    return s;
}

/* rows<B,T> (quant_q8k.rs:166-250) for nv <= 8 vectors: per block, acc_b =
 * fma(d*xd, float(lane sums), acc_b); the min / -32 offset correction is a
 * scalar running sum; out = hsum(acc_b) - corr_b. */
AVX static INL void rows_nv(int q6, const uint8_t *tensor, size_t nb, size_t nv,
                            const float *const *xd, const int8_t *const *xs,
                            const int16_t *const *xb, float *const *outs, size_t r0, size_t r1)
{
    size_t bbytes = q6 ? 210 : 144;
    for (size_t r = r0; r < r1; r++) {
        const uint8_t *row = tensor + r * nb * bbytes;
        __m256 acc[8];
        float corr[8];
        for (size_t b = 0; b < nv; b++) { acc[b] = _mm256_setzero_ps(); corr[b] = 0.0f; }
        for (size_t i = 0; i < nb; i++) {
            blk_t o;
            if (q6) {
                decode_q6k(row + i * bbytes, &o);
                for (size_t b = 0; b < nv; b++) {
                    const int16_t *bs = xb[b] + i * 16;
                    int32_t s = 0;
                    for (int g = 0; g < 16; g++) s += (int32_t)o.sc6[g] * (int32_t)bs[g];
                    float t = o.d * xd[b][i];
                    corr[b] += t * (float)(32 * s);
                }
            } else {
                decode_q4k(row + i * bbytes, &o);
                for (size_t b = 0; b < nv; b++) {
                    const int16_t *bs = xb[b] + i * 16;
                    int32_t s = 0;
                    for (int j = 0; j < 8; j++) s += (int32_t)o.mn[j] * ((int32_t)bs[2 * j] + (int32_t)bs[2 * j + 1]);
                    float t = o.dmin * xd[b][i];
                    corr[b] += t * (float)s;
                }
            }
            for (size_t b = 0; b < nv; b++) {
                __m256i s = lane_sums(&o, xs[b] + i * 256);
                acc[b] = _mm256_fmadd_ps(_mm256_set1_ps(o.d * xd[b][i]), _mm256_cvtepi32_ps(s), acc[b]);
            }
        }
        for (size_t b = 0; b < nv; b++) outs[b][r] = hsum_q8k(acc[b]) - corr[b];
    }
}

/* One instantiation per vector count so the vector loops are unrolled the way
 * the reference's monomorphised rows::<B, T> are. */
#define ROWS_INST(NV)                                                                          \
    AVX static void rows_##NV(int q6, const uint8_t *t, size_t nb, const float *const *xd,     \
                              const int8_t *const *xs, const int16_t *const *xb,               \
                              float *const *o, size_t r0, size_t r1)                           \
    {                                                                                          \
        rows_nv(q6, t, nb, NV, xd, xs, xb, o, r0, r1);                                         \
    }
ROWS_INST(1) ROWS_INST(2) ROWS_INST(3) ROWS_INST(4)
ROWS_INST(5) ROWS_INST(6) ROWS_INST(7) ROWS_INST(8)

typedef void (*rows_fn)(int, const uint8_t *, size_t, const float *const *, const int8_t *const *,
                        const int16_t *const *, float *const *, size_t, size_t);
static const rows_fn ROWS[9] = {0, rows_1, rows_2, rows_3, rows_4, rows_5, rows_6, rows_7, rows_8};

/* matmul_rows (quant_q8k.rs:255-295): up to 8 vectors in one pass over the
 * rows; more vectors walk 16-row tiles and run every group of 8 on each tile. */
int or_matmul_rows(const uint8_t *base, const or_mat *m, size_t n_vec, const float *const *xd,
                   const int8_t *const *xs, const int16_t *const *xb, float *const *outs,
                   size_t r0, size_t r1)
{
    if (m->dtype != OR_Q4_K && m->dtype != OR_Q6_K) return -1;
    if (m->cols == 0 || m->cols % 256) return -1;
    if (r1 <= r0 || n_vec == 0) return 0;
    const uint8_t *tensor = base + m->offset;
    size_t nb = m->cols / 256;
    int q6 = m->dtype == OR_Q6_K;
    for (size_t t0 = r0; t0 < r1;) {
        size_t t1 = n_vec > 8 ? (t0 + 16 < r1 ? t0 + 16 : r1) : r1;
        for (size_t g = 0; g < n_vec; g += 8) {
            size_t e = g + 8 < n_vec ? g + 8 : n_vec;
            ROWS[e - g](q6, tensor, nb, xd + g, xs + g, xb + g, outs + g, t0, t1);
        }
        t0 = t1;
    }
    return 0;
}

/* The per-block int32 lane sums that rows<B,T> converts to float, exported for
 * the bit-exact block-sum check. */
AVX int or_block_sums(const uint8_t *base, const or_mat *m, const int8_t *xs, size_t r0, size_t r1,
                      int32_t *out)
{
    if (m->dtype != OR_Q4_K && m->dtype != OR_Q6_K) return -1;
    if (m->cols == 0 || m->cols % 256) return -1;
    const uint8_t *tensor = base + m->offset;
    size_t nb = m->cols / 256;
    int q6 = m->dtype == OR_Q6_K;
    size_t bbytes = q6 ? 210 : 144;
    for (size_t r = r0; r < r1; r++)
        for (size_t i = 0; i < nb; i++) {
            blk_t o;
            const uint8_t *blk = tensor + (r * nb + i) * bbytes;
            if (q6) decode_q6k(blk, &o); else decode_q4k(blk, &o);
            _mm256_storeu_si256((__m256i *)(out + ((r - r0) * nb + i) * 8), lane_sums(&o, xs + i * 256));
        }
    return 0;
}

int or_cpu_has_avx2(void)
{
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
}
