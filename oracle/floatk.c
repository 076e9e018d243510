/*
 * floatk.c — spindle's float matvec kernels (quant.rs:939-1094 single vector,
 * quant_multi.rs:126-273 multi vector), restated for F32, F16, BF16, Q8_0,
 * Q4_K and Q6_K.  TEST INFRASTRUCTURE ONLY (see sg_oracle.h).
 *
 * The reference's 1-, 2- and 4-row variants do the same arithmetic per row
 * (they only share activation loads), so one row at a time is bit-identical.
 */
#include <immintrin.h>
#include <string.h>

#include "sg_oracle.h"

#define AVX __attribute__((target("avx2,fma,f16c")))
#define INL __attribute__((always_inline)) inline

AVX static INL float half_at(const uint8_t *p)
{
    return _cvtsh_ss((unsigned short)(p[0] | (p[1] << 8)));
}

/* hsum_avx2 (quant.rs:903-908): lo+hi, then two horizontal adds:
 * ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)). */
AVX static INL float hsum_hadd(__m256 v)
{
    __m128 x = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    x = _mm_hadd_ps(x, x);
    x = _mm_hadd_ps(x, x);
    return _mm_cvtss_f32(x);
}

/* hsum of quant_multi.rs:35-40 (same as quant_q8k.rs:153-158). */
AVX static INL float hsum_shuf(__m256 v)
{
    __m128 x = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    x = _mm_add_ps(x, _mm_movehl_ps(x, x));
    x = _mm_add_ss(x, _mm_shuffle_ps(x, x, 0x55));
    return _mm_cvtss_f32(x);
}

/* dot_f32_avx2 (quant.rs:863-874): 8-lane FMA chain, scalar tail with separate
 * multiply and add, result hsum + tail. */
AVX static float dot_f32(const float *a, const float *x, size_t n)
{
    __m256 acc = _mm256_setzero_ps();
    size_t main = n & ~(size_t)7;
    for (size_t i = 0; i < main; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(x + i), acc);
    float tail = 0.0f;
    for (size_t i = main; i < n; i++) { float p = a[i] * x[i]; tail += p; }
    return hsum_hadd(acc) + tail;
}

/* dot_f16_row_avx2 (quant.rs:1412-1425). */
AVX static float dot_f16(const uint8_t *row, const float *x, size_t n)
{
    __m256 acc = _mm256_setzero_ps();
    size_t main = n & ~(size_t)7;
    for (size_t i = 0; i < main; i += 8)
        acc = _mm256_fmadd_ps(_mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(row + 2 * i))), _mm256_loadu_ps(x + i), acc);
    float tail = 0.0f;
    for (size_t i = main; i < n; i++) { float p = half_at(row + 2 * i) * x[i]; tail += p; }
    return hsum_hadd(acc) + tail;
}

/* dot_bf16_row_avx2 (quant.rs:1486-1503). */
AVX static float dot_bf16(const uint8_t *row, const float *x, size_t n)
{
    __m256 acc = _mm256_setzero_ps();
    size_t main = n & ~(size_t)7;
    for (size_t i = 0; i < main; i += 8) {
        __m256i wide = _mm256_cvtepu16_epi32(_mm_loadu_si128((const __m128i *)(row + 2 * i)));
        acc = _mm256_fmadd_ps(_mm256_castsi256_ps(_mm256_slli_epi32(wide, 16)), _mm256_loadu_ps(x + i), acc);
    }
    float tail = 0.0f;
    for (size_t i = main; i < n; i++) {
        uint32_t b = (uint32_t)(row[2 * i] | (row[2 * i + 1] << 8)) << 16;
        float w;
        memcpy(&w, &b, 4);
        float p = w * x[i];
        tail += p;
    }
    return hsum_hadd(acc) + tail;
}

/* dot_q8_0_row_avx2 (quant.rs:51-71): per 32-block an 8-lane FMA chain of
 * q*x over four 8-value steps, then acc = fma(d, s, acc). */
AVX static float dot_q8_0(const uint8_t *row, const float *x, size_t n)
{
    __m256 acc = _mm256_setzero_ps();
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = row + b * 34;
        __m256 s = _mm256_setzero_ps();
        for (int k = 0; k < 32; k += 8) {
            __m256 q = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(blk + 2 + k))));
            s = _mm256_fmadd_ps(q, _mm256_loadu_ps(x + b * 32 + k), s);
        }
        acc = _mm256_fmadd_ps(_mm256_set1_ps(half_at(blk)), s, acc);
    }
    return hsum_hadd(acc);
}

/* compute_subblock_sums_32 (quant.rs:167-178): per 32 values
 * hsum_avx2((v0+v1)+(v2+v3)). */
AVX static void sub_sums_32(const float *x, size_t n, float *out)
{
    for (size_t sb = 0; sb < n / 32; sb++) {
        const float *p = x + sb * 32;
        __m256 a = _mm256_add_ps(_mm256_loadu_ps(p), _mm256_loadu_ps(p + 8));
        __m256 c = _mm256_add_ps(_mm256_loadu_ps(p + 16), _mm256_loadu_ps(p + 24));
        out[sb] = hsum_hadd(_mm256_add_ps(a, c));
    }
}

/* 16 nibble bytes times x[0..16] into one 8-lane FMA chain (quant.rs:183-190). */
AVX static INL __m256 fma_nib16(__m128i v, const float *x, __m256 s)
{
    __m256 a = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(v));
    __m256 b = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(v, 8)));
    return _mm256_fmadd_ps(b, _mm256_loadu_ps(x + 8), _mm256_fmadd_ps(a, _mm256_loadu_ps(x), s));
}

/* dot_q4_k_row_avx2_presum (quant.rs:250-290): per block the min term
 * sum_k mn_k * subsum_k (separately rounded) scaled by dmin into a running
 * total; per chunk and nibble half an FMA chain scaled by d*sc into acc. */
AVX static float dot_q4k(const uint8_t *row, const float *x, const float *sums, size_t n)
{
    const __m128i lo4 = _mm_set1_epi8(0x0f);
    __m256 acc = _mm256_setzero_ps();
    float total_min = 0.0f;
    for (size_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = row + b * 144;
        float d = half_at(blk), dmin = half_at(blk + 2);
        uint8_t sc[8], mn[8];
        or_unpack_q4k_scales(blk + 4, sc, mn);
        const float *xb = x + b * 256;
        float mt = 0.0f;
        for (int k = 0; k < 8; k++) { float p = (float)mn[k] * sums[b * 8 + k]; mt += p; }
        float tm = mt * dmin;
        total_min += tm;
        for (int c = 0; c < 4; c++) {
            __m128i q0 = _mm_loadu_si128((const __m128i *)(blk + 16 + 32 * c));
            __m128i q1 = _mm_loadu_si128((const __m128i *)(blk + 16 + 32 * c + 16));
            const float *a1 = xb + c * 64, *a2 = xb + c * 64 + 32;
            __m256 s = fma_nib16(_mm_and_si128(q0, lo4), a1, _mm256_setzero_ps());
            s = fma_nib16(_mm_and_si128(q1, lo4), a1 + 16, s);
            acc = _mm256_fmadd_ps(_mm256_set1_ps(d * (float)sc[2 * c]), s, acc);
            s = fma_nib16(_mm_and_si128(_mm_srli_epi16(q0, 4), lo4), a2, _mm256_setzero_ps());
            s = fma_nib16(_mm_and_si128(_mm_srli_epi16(q1, 4), lo4), a2 + 16, s);
            acc = _mm256_fmadd_ps(_mm256_set1_ps(d * (float)sc[2 * c + 1]), s, acc);
        }
    }
    return hsum_hadd(acc) - total_min;
}

/* Q6_K signed weights q - 32 of 8 consecutive positions l..l+7 of one half
 * (quant.rs:574-607): out[0..4] are the four 32-apart groups. */
AVX static INL void q6_groups(const uint8_t *ql, const uint8_t *qh, int l, __m256i out[4])
{
    const __m256i m4 = _mm256_set1_epi32(0x0f), m3 = _mm256_set1_epi32(3), off = _mm256_set1_epi32(32);
    __m256i a = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(ql + l)));
    __m256i b = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(ql + l + 32)));
    __m256i h = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(qh + l)));
    out[0] = _mm256_sub_epi32(_mm256_or_si256(_mm256_and_si256(a, m4), _mm256_slli_epi32(_mm256_and_si256(h, m3), 4)), off);
    out[1] = _mm256_sub_epi32(_mm256_or_si256(_mm256_and_si256(b, m4),
                                              _mm256_slli_epi32(_mm256_and_si256(_mm256_srli_epi32(h, 2), m3), 4)), off);
    out[2] = _mm256_sub_epi32(_mm256_or_si256(_mm256_srli_epi32(a, 4),
                                              _mm256_slli_epi32(_mm256_and_si256(_mm256_srli_epi32(h, 4), m3), 4)), off);
    out[3] = _mm256_sub_epi32(_mm256_or_si256(_mm256_srli_epi32(b, 4),
                                              _mm256_slli_epi32(_mm256_and_si256(_mm256_srli_epi32(h, 6), m3), 4)), off);
}

/* dot_q6_k_row_avx2 (quant.rs:552-616): per block a chain of
 * fma(q * sc, x, acc) over halves, 8-position steps and the four groups;
 * then total = fma(d, acc, total). */
AVX static float dot_q6k(const uint8_t *row, const float *x, size_t n)
{
    __m256 total = _mm256_setzero_ps();
    for (size_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = row + b * 210;
        __m256 acc = _mm256_setzero_ps();
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
            const float *y = x + b * 256 + 128 * h;
            for (int l = 0; l < 32; l += 8) {
                int is = l / 16;
                __m256i q[4];
                q6_groups(ql, qh, l, q);
                for (int g = 0; g < 4; g++) {
                    __m256 w = _mm256_mul_ps(_mm256_cvtepi32_ps(q[g]), _mm256_set1_ps((float)sc[is + 2 * g]));
                    acc = _mm256_fmadd_ps(w, _mm256_loadu_ps(y + l + 32 * g), acc);
                }
            }
        }
        total = _mm256_fmadd_ps(_mm256_set1_ps(half_at(blk + 208)), acc, total);
    }
    return hsum_hadd(total);
}

/* matvec_rows_avx2 (quant.rs:939-1094) for the formats on this path. */
AVX int or_matvec_rows(const uint8_t *base, const or_mat *m, const float *x, float *out, size_t r0, size_t n_rows)
{
    int64_t rb = or_row_bytes(m->dtype, m->cols);
    if (rb < 0) return -1;
    const uint8_t *t = base + m->offset;
    size_t n = m->cols;
    float sums_stack[512];
    float *sums = sums_stack;
    float *heap = NULL;
    if (m->dtype == OR_Q4_K) {
        if (n / 32 > 512) {
            heap = (float *)_mm_malloc(n / 32 * sizeof(float), 32);
            if (!heap) return -2;
            sums = heap;
        }
        sub_sums_32(x, n, sums);
    }
    int rc = 0;
    for (size_t i = 0; i < n_rows; i++) {
        const uint8_t *row = t + (r0 + i) * (size_t)rb;
        switch (m->dtype) {
        case OR_F32: out[i] = dot_f32((const float *)row, x, n); break;
        case OR_F16: out[i] = dot_f16(row, x, n); break;
        case OR_BF16: out[i] = dot_bf16(row, x, n); break;
        case OR_Q8_0: out[i] = dot_q8_0(row, x, n); break;
        case OR_Q4_K: out[i] = dot_q4k(row, x, sums, n); break;
        case OR_Q6_K: out[i] = dot_q6k(row, x, n); break;
        default: rc = -1; i = n_rows; break;
        }
    }
    if (heap) _mm_free(heap);
    return rc;
}

/* ---- multi-vector float path (quant_multi.rs:126-273) ---- */

/* deq_q4k (quant_multi.rs:55-72): w = fma(d*sc, q, -(dmin*mn)), one rounding. */
AVX static void deq_q4k(const uint8_t *blk, float *w)
{
    float d = half_at(blk), dmin = half_at(blk + 2);
    uint8_t sc[8], mn[8];
    or_unpack_q4k_scales(blk + 4, sc, mn);
    const __m128i lo4 = _mm_set1_epi8(0x0f);
    for (int c = 0; c < 4; c++) {
        __m128i q[2] = {_mm_loadu_si128((const __m128i *)(blk + 16 + 32 * c)),
                        _mm_loadu_si128((const __m128i *)(blk + 16 + 32 * c + 16))};
        for (int half = 0; half < 2; half++) {
            __m256 s = _mm256_set1_ps(d * (float)sc[2 * c + half]);
            __m256 o = _mm256_set1_ps(dmin * (float)mn[2 * c + half]);
            for (int p = 0; p < 2; p++) {
                __m128i v = half ? _mm_and_si128(_mm_srli_epi16(q[p], 4), lo4) : _mm_and_si128(q[p], lo4);
                float *dst = w + c * 64 + half * 32 + p * 16;
                _mm256_storeu_ps(dst, _mm256_fmsub_ps(s, _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(v)), o));
                _mm256_storeu_ps(dst + 8, _mm256_fmsub_ps(s, _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(v, 8))), o));
            }
        }
    }
}

/* deq_q6k (quant_multi.rs:77-110): w = (d*sc) * q. */
AVX static void deq_q6k(const uint8_t *blk, float *w)
{
    float d = half_at(blk + 208);
    for (int h = 0; h < 2; h++) {
        const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
        const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
        for (int l = 0; l < 32; l += 8) {
            int is = l / 16;
            __m256i q[4];
            q6_groups(ql, qh, l, q);
            for (int g = 0; g < 4; g++) {
                __m256 s = _mm256_set1_ps(d * (float)sc[is + 2 * g]);
                _mm256_storeu_ps(w + 128 * h + 32 * g + l, _mm256_mul_ps(s, _mm256_cvtepi32_ps(q[g])));
            }
        }
    }
}

/* rows_multi<B,T> (quant_multi.rs:126-217) for nv <= 8 vectors: two
 * accumulator sets (even / odd 8-wide chunk), result hsum(acc0 + acc1). */
AVX static INL void rows_multi_nv(int32_t dtype, const uint8_t *tensor, size_t n, size_t nv,
                                  const float *const *xs, float *const *outs, size_t r0, size_t r1)
{
    size_t bs = dtype == OR_Q8_0 ? 32 : (dtype == OR_F32 ? 8 : 256);
    size_t bb = dtype == OR_Q4_K ? 144 : dtype == OR_Q6_K ? 210 : dtype == OR_Q8_0 ? 34 : 32;
    size_t rb = n / bs * bb;
    float wbuf[256] __attribute__((aligned(32)));
    for (size_t r = r0; r < r1; r++) {
        const uint8_t *row = tensor + r * rb;
        __m256 a0[8], a1[8];
        for (size_t b = 0; b < nv; b++) { a0[b] = _mm256_setzero_ps(); a1[b] = _mm256_setzero_ps(); }
        if (dtype == OR_F32) {
            const float *wp = (const float *)row;
            size_t j = 0;
            for (; j + 16 <= n; j += 16) {
                __m256 w0 = _mm256_loadu_ps(wp + j), w1 = _mm256_loadu_ps(wp + j + 8);
                for (size_t b = 0; b < nv; b++) {
                    a0[b] = _mm256_fmadd_ps(w0, _mm256_loadu_ps(xs[b] + j), a0[b]);
                    a1[b] = _mm256_fmadd_ps(w1, _mm256_loadu_ps(xs[b] + j + 8), a1[b]);
                }
            }
            for (; j < n; j += 8) {
                __m256 w0 = _mm256_loadu_ps(wp + j);
                for (size_t b = 0; b < nv; b++) a0[b] = _mm256_fmadd_ps(w0, _mm256_loadu_ps(xs[b] + j), a0[b]);
            }
        } else if (dtype == OR_Q8_0) {
            for (size_t k = 0; k < n / 32; k++) {
                const uint8_t *bp = row + k * 34;
                __m256 d = _mm256_set1_ps(half_at(bp));
                __m256 s[8];
                for (size_t b = 0; b < nv; b++) s[b] = _mm256_setzero_ps();
                for (int i = 0; i < 4; i++) {
                    __m256 w = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(bp + 2 + 8 * i))));
                    for (size_t b = 0; b < nv; b++) s[b] = _mm256_fmadd_ps(w, _mm256_loadu_ps(xs[b] + k * 32 + 8 * i), s[b]);
                }
                for (size_t b = 0; b < nv; b++) {
                    if (k & 1) a1[b] = _mm256_fmadd_ps(d, s[b], a1[b]);
                    else a0[b] = _mm256_fmadd_ps(d, s[b], a0[b]);
                }
            }
        } else {
            for (size_t k = 0; k < n / 256; k++) {
                if (dtype == OR_Q4_K) deq_q4k(row + k * 144, wbuf);
                else deq_q6k(row + k * 210, wbuf);
                for (size_t j = 0; j < 256; j += 16) {
                    __m256 w0 = _mm256_load_ps(wbuf + j), w1 = _mm256_load_ps(wbuf + j + 8);
                    for (size_t b = 0; b < nv; b++) {
                        a0[b] = _mm256_fmadd_ps(w0, _mm256_loadu_ps(xs[b] + k * 256 + j), a0[b]);
                        a1[b] = _mm256_fmadd_ps(w1, _mm256_loadu_ps(xs[b] + k * 256 + j + 8), a1[b]);
                    }
                }
            }
        }
        for (size_t b = 0; b < nv; b++) outs[b][r] = hsum_shuf(_mm256_add_ps(a0[b], a1[b]));
    }
}

#define MULTI_INST(NV)                                                                           \
    AVX static void multi_##NV(int32_t dt, const uint8_t *t, size_t n, const float *const *xs,   \
                               float *const *o, size_t r0, size_t r1)                            \
    {                                                                                            \
        rows_multi_nv(dt, t, n, NV, xs, o, r0, r1);                                              \
    }
MULTI_INST(1) MULTI_INST(2) MULTI_INST(3) MULTI_INST(4)
MULTI_INST(5) MULTI_INST(6) MULTI_INST(7) MULTI_INST(8)

typedef void (*multi_fn)(int32_t, const uint8_t *, size_t, const float *const *, float *const *, size_t, size_t);
static const multi_fn MULTI[9] = {0, multi_1, multi_2, multi_3, multi_4, multi_5, multi_6, multi_7, multi_8};

/* has_multi_kernel (quant_multi.rs:220-227). */
static int has_multi(int32_t dtype, uint64_t n)
{
    switch (dtype) {
    case OR_Q4_K: case OR_Q6_K: return n % 256 == 0;
    case OR_Q8_0: return n % 32 == 0;
    case OR_F32: return n % 8 == 0;
    default: return 0;
    }
}

/* matmul_rows_avx2 (quant_multi.rs:232-273): one vector, or a format without a
 * shared-decode kernel, goes through matvec_rows per vector; otherwise groups
 * of 8 vectors per pass over the rows. */
int or_matmul_rows_multi(const uint8_t *base, const or_mat *m, size_t n_vec, const float *const *xs,
                         float *const *outs, size_t r0, size_t r1)
{
    if (or_row_bytes(m->dtype, m->cols) < 0) return -1;
    if (r1 <= r0 || n_vec == 0) return 0;
    if (!has_multi(m->dtype, m->cols) || n_vec == 1) {
        for (size_t b = 0; b < n_vec; b++) {
            int rc = or_matvec_rows(base, m, xs[b], outs[b] + r0, r0, r1 - r0);
            if (rc) return rc;
        }
        return 0;
    }
    const uint8_t *t = base + m->offset;
    for (size_t g = 0; g < n_vec; g += 8) {
        size_t e = g + 8 < n_vec ? g + 8 : n_vec;
        MULTI[e - g](m->dtype, t, m->cols, xs + g, outs + g, r0, r1);
    }
    return 0;
}

/* dot_f16_row_avx2 (quant.rs:1412-1425) for the attention scores: f16 K row
 * times the fp32 query, as the forward pass calls it (smollm_chat.rs:3475). */
float or_dot_f16_row(const uint8_t *row, const float *x, size_t n) { return dot_f16(row, x, n); }
