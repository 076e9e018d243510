/*
 * synth.c — the reference's synthetic benchmark kernels, restated.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h): the checker for the GPU kernels
 * of spindle_b200/csrc/synth.cu.
 *
 * These are the prototypes of the reference's early benchmark (main.rs), not
 * used by its chat engine: fixed 4096-wide rows, outputs wrapped modulo 4096,
 * a non-IEEE f16 conversion that clamps exponents.
 *
 * or_synth_f16          f16_to_f32             q4k_gemv.rs:37-68
 * or_q4k_block_dot      q4k_block_dot_avx2     q4k_gemv.rs:91-176
 * or_q4k_gemv_4row      q4k_gemv_4row_avx2     q4k_gemv.rs:183-226
 * or_q4k_gemm_spec4     q4k_gemm_spec4_slice   q4k_gemv.rs:361-403 (the per-vector
 *                       dot of q4k_block_dot_spec4_avx2, :232-354, is the single
 *                       dot's operation sequence for each vector)
 * or_route_moe_top2     route_moe_top2         moe_engine.rs:124-164
 * or_kvcache_init       QuantizedKvCache::new  transformer.rs:428-447
 * or_flash_gqa_spec4    flash_decoding_gqa_spec4_avx2, transformer.rs:455-600
 *
 * Compiled with -ffp-contract=off: every product and sum is the one the
 * reference's intrinsics (or Rust's unfused arithmetic) perform.
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "sg_oracle.h"

#define AVX __attribute__((target("avx2,fma")))

enum { SY_HIDDEN = 4096, SY_QK = 256, SY_BLOCKS = 16, SY_ROW_BYTES = 2304, SY_NE = 8, SY_HEADS = 32, SY_KV_HEADS = 8,
       SY_HD = 128, SY_GQA = 4, SY_KV_DIM = 1024, SY_MAX_SEQ = 512, SY_LAYERS = 32, SY_SPEC = 4 };

float or_synth_f16(uint16_t h)
{
    uint32_t sign = ((uint32_t)(h & 0x8000)) << 16, e = (h >> 10) & 0x1f, mant = h & 0x03ff, bits;
    if (e == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            uint32_t m = mant;
            int32_t ex = 127 - 14;
            while ((m & 0x0400) == 0) {
                m <<= 1;
                ex -= 1;
            }
            bits = sign | ((uint32_t)ex << 23) | ((m & 0x03ff) << 13);
        }
    } else if (e == 31) {
        bits = sign | (119u << 23) | (mant << 13);
    } else {
        int32_t se = (int32_t)e - 15;
        se = se < -10 ? -10 : (se > 4 ? 4 : se);
        bits = sign | ((uint32_t)(se + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static void unpack_scales(const uint8_t *sc, uint8_t *s, uint8_t *m)
{
    for (int j = 0; j < 4; j++) {
        s[j] = sc[j] & 63;
        m[j] = sc[j + 4] & 63;
        s[j + 4] = (sc[j + 8] & 0x0F) | ((sc[j] >> 6) << 4);
        m[j + 4] = (sc[j + 8] >> 4) | ((sc[j + 4] >> 6) << 4);
    }
}

AVX static __m256 fma32(__m256i bytes32, __m256 scale, __m256 neg_min, const float *act, __m256 acc)
{
    __m128i lo = _mm256_castsi256_si128(bytes32), hi = _mm256_extracti128_si256(bytes32, 1);
    __m256 dq;
    dq = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(lo)), scale, neg_min);
    acc = _mm256_fmadd_ps(dq, _mm256_loadu_ps(act), acc);
    dq = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(lo, 8))), scale, neg_min);
    acc = _mm256_fmadd_ps(dq, _mm256_loadu_ps(act + 8), acc);
    dq = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(hi)), scale, neg_min);
    acc = _mm256_fmadd_ps(dq, _mm256_loadu_ps(act + 16), acc);
    dq = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(hi, 8))), scale, neg_min);
    acc = _mm256_fmadd_ps(dq, _mm256_loadu_ps(act + 24), acc);
    return acc;
}

AVX static float hsum256(__m256 v)
{
    __m128 x = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    x = _mm_hadd_ps(x, x);
    x = _mm_hadd_ps(x, x);
    return _mm_cvtss_f32(x);
}

AVX float or_q4k_block_dot(const uint8_t *blk, const float *act)
{
    const float d = or_synth_f16((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = or_synth_f16((uint16_t)(blk[2] | (blk[3] << 8)));
    uint8_t sc[8], mn[8];
    unpack_scales(blk + 4, sc, mn);
    const __m256i low = _mm256_set1_epi8(0x0F);
    __m256 acc = _mm256_setzero_ps();
    for (int c = 0; c < 4; c++) {
        __m256i q = _mm256_loadu_si256((const __m256i *)(blk + 16 + 32 * c));
        __m256i ql = _mm256_and_si256(q, low), qh = _mm256_and_si256(_mm256_srli_epi16(q, 4), low);
        __m256 sl = _mm256_set1_ps(d * (float)sc[2 * c]), ml = _mm256_set1_ps(-dmin * (float)mn[2 * c]);
        __m256 sh = _mm256_set1_ps(d * (float)sc[2 * c + 1]), mh = _mm256_set1_ps(-dmin * (float)mn[2 * c + 1]);
        acc = fma32(ql, sl, ml, act + 64 * c, acc);
        acc = fma32(qh, sh, mh, act + 64 * c + 32, acc);
    }
    return hsum256(acc);
}

/* Rows of 16 blocks in groups of 4 (a remainder of fewer than 4 rows is not
 * processed); y[(row_offset + r) & 4095] += the row's sum; returns the rows done. */
uint64_t or_q4k_gemv_4row(const uint8_t *chunk, uint64_t chunk_len, const float *x, float *y, uint64_t row_offset)
{
    const uint64_t groups = chunk_len / SY_ROW_BYTES / 4;
    for (uint64_t g = 0; g < groups; g++) {
        float sums[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int b = 0; b < SY_BLOCKS; b++)
            for (int i = 0; i < 4; i++)
                sums[i] += or_q4k_block_dot(chunk + (4 * g + i) * SY_ROW_BYTES + 144 * b, x + SY_QK * b);
        const uint64_t dst = (row_offset + 4 * g) & (SY_HIDDEN - 1);
        for (int i = 0; i < 4; i++) y[(dst + i) & (SY_HIDDEN - 1)] += sums[i];
    }
    return groups * 4;
}

/* Rows [r0, r1) for four activation vectors x4[k] (4096 floats each), into
 * y4[k][(base + r) & 4095]. */
void or_q4k_gemm_spec4(const uint8_t *chunk, uint64_t r0, uint64_t r1, const float *x4, float *y4, uint64_t base)
{
    for (uint64_t r = r0; r < r1; r++) {
        float sums[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int b = 0; b < SY_BLOCKS; b++)
            for (int k = 0; k < 4; k++)
                sums[k] += or_q4k_block_dot(chunk + r * SY_ROW_BYTES + 144 * b, x4 + (uint64_t)k * SY_HIDDEN + SY_QK * b);
        const uint64_t dst = (base + r) & (SY_HIDDEN - 1);
        for (int k = 0; k < 4; k++) y4[(uint64_t)k * SY_HIDDEN + dst] += sums[k];
    }
}

void or_route_moe_top2(const float *x, const float *gates, uint64_t layer, int32_t *experts, float *weights)
{
    float s[SY_NE];
    for (int e = 0; e < SY_NE; e++) {
        float acc = 0.0f;
        for (int i = 0; i < SY_HIDDEN; i += 16) acc += x[i] * gates[(size_t)e * SY_HIDDEN + i];
        acc += (float)((layer + (uint64_t)e) % SY_NE) * 0.05f;
        s[e] = acc;
    }
    int b0 = 0, b1 = 1;
    if (s[b1] > s[b0]) {
        b0 = 1;
        b1 = 0;
    }
    for (int e = 2; e < SY_NE; e++) {
        if (s[e] > s[b0]) {
            b1 = b0;
            b0 = e;
        } else if (s[e] > s[b1]) {
            b1 = e;
        }
    }
    const float mx = s[b0];
    const float w0 = or_expf(s[b0] - mx), w1 = or_expf(s[b1] - mx);
    const float inv = 1.0f / (w0 + w1);
    experts[0] = b0;
    experts[1] = b1;
    weights[0] = w0 * inv;
    weights[1] = w1 * inv;
}

/* QuantizedKvCache::new: k, v int8 [layers][max_seq][kv_dim]; scales f32
 * [layers][max_seq][kv_heads], all 1/127; the first init_ctx positions filled. */
void or_kvcache_init(int8_t *k, int8_t *v, float *ks, float *vs, uint64_t init_ctx)
{
    const uint64_t ctx = init_ctx < SY_MAX_SEQ - SY_SPEC ? init_ctx : SY_MAX_SEQ - SY_SPEC;
    memset(k, 0, (size_t)SY_LAYERS * SY_MAX_SEQ * SY_KV_DIM);
    memset(v, 0, (size_t)SY_LAYERS * SY_MAX_SEQ * SY_KV_DIM);
    for (size_t i = 0; i < (size_t)SY_LAYERS * SY_MAX_SEQ * SY_KV_HEADS; i++) ks[i] = vs[i] = 1.0f / 127.0f;
    for (uint64_t l = 0; l < SY_LAYERS; l++)
        for (uint64_t t = 0; t < ctx; t++)
            for (uint64_t i = 0; i < SY_KV_DIM; i++) {
                const size_t o = ((size_t)l * SY_MAX_SEQ + t) * SY_KV_DIM + i;
                k[o] = (int8_t)((int8_t)((l * 17 + t * 31 + i) % 127) - 63);
                v[o] = (int8_t)((int8_t)((l * 13 + t * 29 + i) % 127) - 63);
            }
}

/* quantize_kv_step_avx2 (transformer.rs:455-479) */
static void quantize_kv(const float *src, int8_t *q, float *scales)
{
    for (int h = 0; h < SY_KV_HEADS; h++) {
        const float *s = src + h * SY_HD;
        float mx = 1e-6f;
        for (int d = 0; d < SY_HD; d++) {
            const float a = fabsf(s[d]);
            if (a > mx) mx = a;
        }
        const float inv = 127.0f / mx;
        scales[h] = mx / 127.0f;
        for (int d = 0; d < SY_HD; d++) {
            float r = roundf(s[d] * inv);  /* f32::round: half away from zero */
            if (isnan(r)) {
                q[h * SY_HD + d] = 0;
                continue;
            }
            r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
            q[h * SY_HD + d] = (int8_t)r;
        }
    }
}

AVX static float dot_q_k(const float *q, const int8_t *k, float ks)
{
    __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
    for (int d = 0; d < SY_HD; d += 16) {
        __m256 k0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(k + d))));
        __m256 k1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(k + d + 8))));
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(q + d), k0, a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(q + d + 8), k1, a1);
    }
    return hsum256(_mm256_add_ps(a0, a1)) * ks;
}

AVX static void fmadd_v(float *out, float rescale, const int8_t *v, float w)
{
    const __m256 r = _mm256_set1_ps(rescale), wv = _mm256_set1_ps(w);
    for (int d = 0; d < SY_HD; d += 16) {
        __m256 v0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(v + d))));
        __m256 v1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(v + d + 8))));
        __m256 o0 = _mm256_mul_ps(_mm256_loadu_ps(out + d), r), o1 = _mm256_mul_ps(_mm256_loadu_ps(out + d + 8), r);
        _mm256_storeu_ps(out + d, _mm256_fmadd_ps(v0, wv, o0));
        _mm256_storeu_ps(out + d + 8, _mm256_fmadd_ps(v1, wv, o1));
    }
}

static float fmaxr(float a, float b) { return isnan(a) ? b : (isnan(b) ? a : (a > b ? a : b)); } /* f32::max */

/* q_spec [4][4096] in place; the cache as or_kvcache_init lays it out; seq_len
 * is the cache's filled length. */
AVX void or_flash_gqa_spec4(float *q_spec, int8_t *kq, int8_t *vq, float *ks, float *vs, uint64_t seq_len,
                            uint64_t layer)
{
    const uint64_t l = layer % SY_LAYERS, base = seq_len < SY_MAX_SEQ - SY_SPEC ? seq_len : SY_MAX_SEQ - SY_SPEC;
    const float inv_sqrt_d = 1.0f / sqrtf((float)SY_HD);
    for (int k = 0; k < SY_SPEC; k++) {
        const size_t o = ((size_t)l * SY_MAX_SEQ + base + k);
        quantize_kv(q_spec + (size_t)k * SY_HIDDEN, kq + o * SY_KV_DIM, ks + o * SY_KV_HEADS);
        quantize_kv(q_spec + (size_t)k * SY_HIDDEN, vq + o * SY_KV_DIM, vs + o * SY_KV_HEADS);
    }
    float out[SY_HD];
    for (int k = 0; k < SY_SPEC; k++) {
        const uint64_t end = base + k + 1;
        for (int qh = 0; qh < SY_HEADS; qh++) {
            const int kvh = qh / SY_GQA;
            const float *q = q_spec + (size_t)k * SY_HIDDEN + qh * SY_HD;
            memset(out, 0, sizeof out);
            float m_prev = -INFINITY, l_prev = 0.0f;
            for (uint64_t pos = 0; pos < end; pos++) {
                const size_t o = (size_t)l * SY_MAX_SEQ + pos;
                float score = dot_q_k(q, kq + o * SY_KV_DIM + kvh * SY_HD, ks[o * SY_KV_HEADS + kvh]) * inv_sqrt_d;
                score = score < -20.0f ? -20.0f : (score > 20.0f ? 20.0f : score);
                const float m_new = fmaxr(m_prev, score);
                const float alpha = or_expf(m_prev - m_new), p = or_expf(score - m_new);
                l_prev = l_prev * alpha + p;
                m_prev = m_new;
                fmadd_v(out, alpha, vq + o * SY_KV_DIM + kvh * SY_HD, p * vs[o * SY_KV_HEADS + kvh]);
            }
            const float inv_l = 1.0f / fmaxr(l_prev, 1e-8f);
            float *dst = q_spec + (size_t)k * SY_HIDDEN + qh * SY_HD;
            for (int d = 0; d < SY_HD; d++) dst[d] = out[d] * inv_l;
        }
    }
}
