/*
 * forward.c — spindle's decoder forward pass, restated.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h): the checker for the GPU forward.
 *
 * or_rmsnorm     rmsnorm              smollm_chat.rs:569-575
 * (heads)        rmsnorm_heads        smollm_chat.rs:578-584
 * or_rope_freqs  Rope::new            smollm_chat.rs:1403-1406
 * or_rope_rotate Rope::rotate         smollm_chat.rs:1408-1419
 * or_kv_shift    shift_kv             smollm_chat.rs:2942-2972
 * (matvec)       matvec               smollm_chat.rs:309-349 (integer path when supported)
 * or_forward     forward_slice        smollm_chat.rs:3371-3552 (one token; no bias tensors,
 *                                     no layer streaming or expert cache)
 * or_argmax      sample_from_logits   smollm_chat.rs:3661-3671 at temperature 0
 *
 * Scalar float code keeps the Rust expression order with one rounding per
 * operation (-ffp-contract=off); powf/sqrtf are glibc's and sin/cos/exp
 * glibc's sinf/cosf/expf, as Rust's f32 methods call them on Linux (or the
 * correctly rounded values, see libm.c).
 */
#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "sg_oracle.h"

#define AVX __attribute__((target("avx2,fma,f16c")))

/* Rust f32::max: the other operand when one is NaN. */
static float rmax(float a, float b)
{
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

void or_rmsnorm(const float *x, const float *w, float *out, size_t n, float eps)
{
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++) { float p = x[i] * x[i]; ss += p; }
    float mean = ss / (float)n;
    float inv = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < n; i++) { float t = x[i] * inv; out[i] = t * w[i]; }
}

void or_rope_freqs(float theta, uint32_t head_dim, float *inv_freq)
{
    for (uint32_t i = 0; i < head_dim / 2; i++) {
        float e = (2.0f * (float)i) / (float)head_dim;
        inv_freq[i] = 1.0f / powf(theta, e);
    }
}

void or_rope_rotate(float *v, size_t len, uint32_t head_dim, const float *inv_freq, int neox, float pos)
{
    uint32_t half = head_dim / 2;
    for (size_t h0 = 0; h0 < len; h0 += head_dim) {
        float *head = v + h0;
        for (uint32_t i = 0; i < half; i++) {
            float ang = pos * inv_freq[i];
            float s = or_sinf(ang), c = or_cosf(ang);
            uint32_t a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            float x0 = head[a], x1 = head[b];
            float t0 = x0 * c, t1 = x1 * s;
            head[a] = t0 - t1;
            float t2 = x0 * s, t3 = x1 * c;
            head[b] = t2 + t3;
        }
    }
}

static int int_supported(const or_mat *m, int int_on)
{
    return int_on && (m->dtype == OR_Q4_K || m->dtype == OR_Q6_K) && m->cols && m->cols % 256 == 0;
}

/* matvec (smollm_chat.rs:309-349): Q8_K of x then the integer kernel when the
 * matrix supports it, else the float kernel. */
static int matvec(const uint8_t *base, const or_mat *m, const float *x, float *out, int int_on)
{
    if (!int_supported(m, int_on)) return or_matvec_rows(base, m, x, out, 0, m->rows);
    size_t nb = m->cols / 256;
    float *d = malloc(nb * sizeof(float));
    int8_t *qs = malloc(m->cols);
    int16_t *bs = malloc(nb * 16 * sizeof(int16_t));
    int rc = -2;
    if (d && qs && bs) {
        or_q8k_quantize(x, m->cols, d, qs, bs);
        const float *dp = d;
        const int8_t *qp = qs;
        const int16_t *bp = bs;
        rc = or_matmul_rows(base, m, 1, &dp, &qp, &bp, &out, 0, m->rows);
    }
    free(d); free(qs); free(bs);
    return rc;
}

/* f32_to_f16_slice (quant.rs:1506-1512): _mm256_cvtps_ph, round to nearest even. */
AVX static void to_f16(const float *src, uint16_t *dst, size_t n)
{
    for (size_t i = 0; i < n; i += 8)
        _mm_storeu_si128((__m128i *)(dst + i), _mm256_cvtps_ph(_mm256_loadu_ps(src + i), _MM_FROUND_TO_NEAREST_INT));
}

/* compute_head_fn (smollm_chat.rs:3463-3495): online softmax over 0..=pos. */
AVX static void attn_head(const uint16_t *kc, const uint16_t *vc, size_t stride, const float *q, uint32_t head_dim,
                          uint32_t pos, float scale, float *out)
{
    __m256 acc[64];
    uint32_t nv = head_dim / 8;
    for (uint32_t d = 0; d < nv; d++) acc[d] = _mm256_setzero_ps();
    float m_prev = -INFINITY, l_prev = 0.0f;
    for (uint32_t t = 0; t <= pos; t++) {
        const uint16_t *k = kc + (size_t)t * stride, *v = vc + (size_t)t * stride;
        float dot = or_dot_f16_row((const uint8_t *)k, q, head_dim);
        float score = dot * scale;
        float m_new = rmax(m_prev, score);
        float alpha = or_expf(m_prev - m_new);
        float p = or_expf(score - m_new);
        float la = l_prev * alpha;
        l_prev = la + p;
        m_prev = m_new;
        __m256 va = _mm256_set1_ps(alpha), vp = _mm256_set1_ps(p);
        for (uint32_t d = 0; d < nv; d++) {
            __m256 ov = _mm256_mul_ps(acc[d], va);
            __m256 vv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(v + 8 * d)));
            acc[d] = _mm256_fmadd_ps(vp, vv, ov);
        }
    }
    __m256 inv = _mm256_set1_ps(1.0f / rmax(l_prev, 1e-9f));
    for (uint32_t d = 0; d < nv; d++) _mm256_storeu_ps(out + 8 * d, _mm256_mul_ps(acc[d], inv));
}

int or_forward(const uint8_t *base, const or_model *m, uint16_t *kcache, uint16_t *vcache, int64_t token,
               const float *in_hidden, uint32_t pos, int int_on, float *hidden_out, float *logits_out)
{
    size_t dim = m->dim, hd = m->head_dim, q_dim = (size_t)m->n_heads * hd, kv_dim = (size_t)m->n_kv_heads * hd;
    if (!m->n_heads || !m->n_kv_heads || m->n_heads % m->n_kv_heads || hd % 8 || hd > 512 || pos >= m->max_seq)
        return -1;
    int rc = 0;
    float *x = malloc(dim * 4), *xn = malloc(dim * 4), *q = malloc(q_dim * 4), *k = malloc(kv_dim * 4);
    float *v = malloc(kv_dim * 4), *att = malloc(q_dim * 4), *proj = malloc(dim * 4), *tmp = malloc(hd * 4);
    float *freqs = malloc(hd / 2 * 4);
    if (!x || !xn || !q || !k || !v || !att || !proj || !tmp || !freqs) { rc = -2; goto done; }
    or_rope_freqs(m->rope_theta, m->head_dim, freqs);
    if (token >= 0) {
        if ((uint64_t)token >= m->embed.rows) { rc = -1; goto done; }
        int64_t rb = or_row_bytes(m->embed.dtype, dim);
        if (rb < 0 || (rc = or_dequant_row(m->embed.dtype, base + m->embed.offset + (uint64_t)token * rb, dim, x)))
            { rc = -1; goto done; }
        if (m->embedding_scale != 1.0f)
            for (size_t i = 0; i < dim; i++) x[i] *= m->embedding_scale;
    } else if (in_hidden) {
        memcpy(x, in_hidden, dim * 4);
    } else {
        rc = -1;
        goto done;
    }
    float scale = m->attn_scale != 0.0f ? m->attn_scale : 1.0f / sqrtf((float)hd);
    uint32_t heads_per_kv = m->n_heads / m->n_kv_heads;
    for (uint32_t l = 0; l < m->n_layers; l++) {
        const or_layer *ly = &m->layers[l];
        or_rmsnorm(x, (const float *)(base + ly->attn_norm), xn, dim, m->rms_eps);
        if ((rc = matvec(base, &ly->wq, xn, q, int_on)) || (rc = matvec(base, &ly->wk, xn, k, int_on)) ||
            (rc = matvec(base, &ly->wv, xn, v, int_on)))
            goto done;
        if (ly->q_norm != UINT64_MAX)
            for (size_t h = 0; h < q_dim; h += hd) {
                or_rmsnorm(q + h, (const float *)(base + ly->q_norm), tmp, hd, m->rms_eps);
                memcpy(q + h, tmp, hd * 4);
            }
        if (ly->k_norm != UINT64_MAX)
            for (size_t h = 0; h < kv_dim; h += hd) {
                or_rmsnorm(k + h, (const float *)(base + ly->k_norm), tmp, hd, m->rms_eps);
                memcpy(k + h, tmp, hd * 4);
            }
        or_rope_rotate(q, q_dim, m->head_dim, freqs, m->rope_neox, (float)pos);
        or_rope_rotate(k, kv_dim, m->head_dim, freqs, m->rope_neox, (float)pos);
        size_t kv_off = ((size_t)l * m->max_seq + pos) * kv_dim;
        to_f16(k, kcache + kv_off, kv_dim);
        to_f16(v, vcache + kv_off, kv_dim);
        for (uint32_t h = 0; h < m->n_heads; h++) {
            size_t kvh = h / heads_per_kv, lo = (size_t)l * m->max_seq * kv_dim + kvh * hd;
            attn_head(kcache + lo, vcache + lo, kv_dim, q + h * hd, m->head_dim, pos, scale, att + h * hd);
        }
        if ((rc = matvec(base, &ly->wo, att, proj, int_on))) goto done;
        for (size_t i = 0; i < dim; i++) { float t = m->residual_scale * proj[i]; x[i] += t; }
        or_rmsnorm(x, (const float *)(base + ly->ffn_norm), xn, dim, m->rms_eps);
        if (ly->is_moe) {
            rc = or_moe_forward(base, &ly->moe, xn, proj, int_on, NULL, NULL, NULL);
        } else {
            /* ffn_forward with the fused FFN (smollm_chat.rs:591-595) */
            float one = 1.0f;
            memset(proj, 0, dim * 4);
            rc = or_ffns_fused(base, &ly->gate, &ly->up, &ly->down, &one, 1, xn, proj, int_on);
        }
        if (rc) goto done;
        for (size_t i = 0; i < dim; i++) { float t = m->residual_scale * proj[i]; x[i] += t; }
    }
    or_rmsnorm(x, (const float *)(base + m->output_norm), xn, dim, m->rms_eps);
    if (hidden_out) memcpy(hidden_out, xn, dim * 4);
    if (logits_out) rc = matvec(base, &m->lm_head, xn, logits_out, int_on);
done:
    free(x); free(xn); free(q); free(k); free(v); free(att); free(proj); free(tmp); free(freqs);
    return rc;
}

/* f32::total_cmp order as a signed integer */
static int32_t total_key(float f)
{
    int32_t i;
    memcpy(&i, &f, 4);
    return i ^ (int32_t)((uint32_t)(i >> 31) >> 1);
}

int64_t or_argmax(const float *logits, size_t n)
{
    if (!n) return 0;
    size_t best = 0;
    int32_t bk = total_key(logits[0]);
    for (size_t i = 1; i < n; i++) {
        int32_t ki = total_key(logits[i]);
        if (ki >= bk) { bk = ki; best = i; }  /* max_by keeps the last maximum */
    }
    return (int64_t)best;
}

/* f16_to_f32_slice (quant.rs:1516-1522): _mm256_cvtph_ps, exact. */
AVX static void from_f16(const uint16_t *src, float *dst, size_t n)
{
    for (size_t i = 0; i < n; i += 8)
        _mm256_storeu_ps(dst + i, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(src + i))));
}

/* shift_kv (smollm_chat.rs:2942-2972): drop n_discard positions after the
 * n_keep pinned ones (clamped to cur_pos - n_keep); each kept K row slides down
 * by n_discard, widened to f32, re-rotated by -n_discard and rounded back to
 * f16; V rows are copied; layers [l0, l1), in increasing position order as the
 * reference does.  Returns the new position. */
uint32_t or_kv_shift(const or_model *m, uint16_t *kcache, uint16_t *vcache, uint32_t l0, uint32_t l1, uint32_t n_keep,
                     uint32_t n_discard, uint32_t cur_pos)
{
    const uint32_t kv_dim = m->n_kv_heads * m->head_dim;
    const uint32_t n_ctx = cur_pos > n_keep ? cur_pos - n_keep : 0;
    if (n_discard > n_ctx) n_discard = n_ctx;
    if (n_discard == 0) return cur_pos;
    const uint32_t n_move = n_ctx - n_discard;
    float freqs[512], *tmp = malloc(sizeof(float) * kv_dim);
    or_rope_freqs(m->rope_theta, m->head_dim, freqs);
    for (uint32_t l = l0; l < l1; l++) {
        const size_t layer = (size_t)l * m->max_seq;
        for (uint32_t i = 0; i < n_move; i++) {
            const size_t src = (layer + n_keep + n_discard + i) * kv_dim, dst = (layer + n_keep + i) * kv_dim;
            from_f16(kcache + src, tmp, kv_dim);
            or_rope_rotate(tmp, kv_dim, m->head_dim, freqs, m->rope_neox, -(float)n_discard);
            to_f16(tmp, kcache + dst, kv_dim);
            memmove(vcache + dst, vcache + src, sizeof(uint16_t) * kv_dim);
        }
    }
    free(tmp);
    return cur_pos - n_discard;
}
