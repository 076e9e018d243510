/*
 * moe.c — spindle's fused FFN and MoE layer (smollm_chat.rs), restated.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h).
 *
 * or_ffns_fused   ffns_fused        smollm_chat.rs:382-442
 * or_moe_forward  moe_forward       smollm_chat.rs:1178-1240 (router, softmax,
 *                                   top-k, prune), :1333-1351 (fused experts),
 *                                   :1367-1382 (shared expert)
 * Scalar float code follows the Rust expressions left to right with separate
 * roundings (-ffp-contract=off); exp is glibc expf, as Rust's f32::exp on Linux
 * (or the correctly rounded value, see libm.c).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "sg_oracle.h"

/* silu, smollm_chat.rs:586-588: x / (1 + exp(-x)). */
static float silu(float x)
{
    float e = or_expf(-x);
    float den = 1.0f + e;
    return x / den;
}

static int int_supported(const or_mat *m, int int_on)
{
    return int_on && (m->dtype == OR_Q4_K || m->dtype == OR_Q6_K) && m->cols && m->cols % 256 == 0;
}

/* rows_into (smollm_chat.rs:341-349): the integer kernel when the matrix
 * supports it and x was quantized, else the float kernel on x. */
static int rows_into(const uint8_t *base, const or_mat *m, const float *x, const float *xd, const int8_t *xs,
                     const int16_t *xb, int have_q, int int_on, float *out, size_t r0, size_t r1)
{
    if (r1 <= r0) return 0;
    if (have_q && int_supported(m, int_on)) return or_matmul_rows(base, m, 1, &xd, &xs, &xb, &out, r0, r1);
    return or_matvec_rows(base, m, x, out + r0, r0, r1 - r0);
}

typedef struct {
    float *d;
    int8_t *qs;
    int16_t *bs;
} q8k_buf;

static int q8k_alloc(q8k_buf *q, size_t n)
{
    q->d = malloc((n / 256 + 1) * sizeof(float));
    q->qs = malloc(n + 1);
    q->bs = malloc((n / 16 + 1) * sizeof(int16_t));
    return q->d && q->qs && q->bs ? 0 : -2;
}

static void q8k_free(q8k_buf *q) { free(q->d); free(q->qs); free(q->bs); }

/* ffns_fused: out[r] = out[r] + w_0*y_0[r] + w_1*y_1[r] + ... (in order) for the
 * k SwiGLU FFNs (gate[e], up[e], down[e]) on input x. */
int or_ffns_fused(const uint8_t *base, const or_mat *gate, const or_mat *up, const or_mat *down,
                  const float *weights, size_t k, const float *x, float *out, int int_on)
{
    if (k == 0) return 0;
    size_t n_ff = gate[0].rows, dim = down[0].rows, cols = gate[0].cols;
    int any_int = 0, any_int_down = 0;
    for (size_t e = 0; e < k; e++) {
        any_int |= int_supported(&gate[e], int_on) || int_supported(&up[e], int_on);
        any_int_down |= int_supported(&down[e], int_on);
    }
    int rc = 0;
    float *h = malloc(k * n_ff * sizeof(float)), *u = malloc(k * n_ff * sizeof(float));
    float *y = malloc(k * dim * sizeof(float));
    q8k_buf xq = {0}, *hq = calloc(k, sizeof(q8k_buf));
    if (!h || !u || !y || !hq) { rc = -2; goto done; }
    if (any_int) {
        if ((rc = q8k_alloc(&xq, cols))) goto done;
        or_q8k_quantize(x, cols, xq.d, xq.qs, xq.bs);
    }
    for (size_t e = 0; e < k; e++) {
        float *he = h + e * n_ff, *ue = u + e * n_ff;
        if ((rc = rows_into(base, &gate[e], x, xq.d, xq.qs, xq.bs, any_int, int_on, he, 0, n_ff))) goto done;
        if ((rc = rows_into(base, &up[e], x, xq.d, xq.qs, xq.bs, any_int, int_on, ue, 0, n_ff))) goto done;
        for (size_t r = 0; r < n_ff; r++) {
            float s = silu(he[r]);
            he[r] = s * ue[r];
        }
    }
    for (size_t e = 0; e < k; e++) {
        if (any_int_down) {
            if ((rc = q8k_alloc(&hq[e], n_ff))) goto done;
            or_q8k_quantize(h + e * n_ff, n_ff, hq[e].d, hq[e].qs, hq[e].bs);
        }
        if ((rc = rows_into(base, &down[e], h + e * n_ff, hq[e].d, hq[e].qs, hq[e].bs, any_int_down, int_on,
                            y + e * dim, 0, dim)))
            goto done;
    }
    for (size_t r = 0; r < dim; r++) {
        float acc = out[r];
        for (size_t e = 0; e < k; e++) {
            float t = weights[e] * y[e * dim + r];
            acc += t;
        }
        out[r] = acc;
    }
done:
    if (hq) for (size_t e = 0; e < k; e++) q8k_free(&hq[e]);
    free(hq);
    q8k_free(&xq);
    free(h); free(u); free(y);
    return rc;
}

static or_mat expert_view(const or_mat *m, size_t e)
{
    or_mat v = *m;
    v.offset = m->offset + e * m->rows * (uint64_t)or_row_bytes(m->dtype, m->cols);
    return v;
}

/* Rust f32::max: the other operand when one is NaN. */
static float rmax(float a, float b)
{
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* Ordering of f32::total_cmp on the bit patterns. */
static int32_t total_key(float f)
{
    int32_t i;
    memcpy(&i, &f, 4);
    return i ^ (int32_t)((uint32_t)(i >> 31) >> 1);
}

int or_moe_route(const uint8_t *base, const or_moe *m, const float *x, float *probs, int32_t *chosen,
                 float *weights, uint32_t *n_chosen)
{
    size_t ne = m->n_expert, k = m->n_used;
    if (k == 0 || k > ne || ne > 4096) return -1;
    /* router logits: matvec -> float path (F32 router) */
    int rc = or_matvec_rows(base, &m->router, x, probs, 0, ne);
    if (rc) return rc;
    float mx = -INFINITY;
    for (size_t e = 0; e < ne; e++) mx = rmax(mx, probs[e]);
    for (size_t e = 0; e < ne; e++) { float d = probs[e] - mx; probs[e] = or_expf(d); }
    float sum = 0.0f;
    for (size_t e = 0; e < ne; e++) sum += probs[e];
    for (size_t e = 0; e < ne; e++) probs[e] /= sum;
    /* top-k, descending (total order); ties keep the lower expert index first */
    int32_t *idx = malloc(ne * sizeof(int32_t));
    if (!idx) return -2;
    for (size_t e = 0; e < ne; e++) idx[e] = (int32_t)e;
    for (size_t i = 0; i < k; i++) {
        size_t best = i;
        for (size_t j = i + 1; j < ne; j++) {
            int32_t kj = total_key(probs[idx[j]]), kb = total_key(probs[idx[best]]);
            if (kj > kb || (kj == kb && idx[j] < idx[best])) best = j;
        }
        int32_t t = idx[i]; idx[i] = idx[best]; idx[best] = t;
    }
    size_t keep = k;
    if (m->moe_prune > 0.0f && k > 2) {
        size_t min_keep = k / 2 > 2 ? k / 2 : 2;
        if (m->moe_prune >= 1.0f) {
            size_t p = (size_t)m->moe_prune;
            keep = p < min_keep ? min_keep : (p > k ? k : p);
        } else {
            float top_sum = 0.0f;
            for (size_t i = 0; i < k; i++) top_sum += probs[idx[i]];
            float target = top_sum * (1.0f - m->moe_prune);
            float cum = 0.0f;
            size_t i = 0;
            while (i < k && (i < min_keep || cum < target)) { cum += probs[idx[i]]; i++; }
            keep = i;
        }
    }
    float wsum = 0.0f;
    for (size_t i = 0; i < keep; i++) wsum += probs[idx[i]];
    for (size_t i = 0; i < keep; i++) {
        chosen[i] = idx[i];
        weights[i] = m->norm ? probs[idx[i]] / wsum : probs[idx[i]];
    }
    *n_chosen = (uint32_t)keep;
    free(idx);
    return 0;
}

int or_moe_forward(const uint8_t *base, const or_moe *m, const float *x, float *out, int int_on,
                   int32_t *chosen_out, float *weights_out, uint32_t *n_chosen_out)
{
    size_t ne = m->n_expert, dim = m->down.rows;
    float *probs = malloc(ne * sizeof(float));
    int32_t chosen[256];
    float ws[256];
    uint32_t nk = 0;
    int rc;
    if (!probs) return -2;
    if (m->n_used > 256) { free(probs); return -1; }
    if ((rc = or_moe_route(base, m, x, probs, chosen, ws, &nk))) { free(probs); return rc; }
    or_mat g[256], u[256], d[256];
    for (uint32_t i = 0; i < nk; i++) {
        g[i] = expert_view(&m->gate, (size_t)chosen[i]);
        u[i] = expert_view(&m->up, (size_t)chosen[i]);
        d[i] = expert_view(&m->down, (size_t)chosen[i]);
    }
    for (size_t r = 0; r < dim; r++) out[r] = 0.0f;
    rc = or_ffns_fused(base, g, u, d, ws, nk, x, out, int_on);
    if (!rc && m->has_shared) {
        float *tmp = calloc(dim, sizeof(float));
        float one = 1.0f;
        if (!tmp) { free(probs); return -2; }
        rc = or_ffns_fused(base, &m->sh_gate, &m->sh_up, &m->sh_down, &one, 1, x, tmp, int_on);
        float gsc = 1.0f;
        if (m->has_shared_gate) {
            const float *w = (const float *)(base + m->shared_gate_offset);
            float z = 0.0f;
            for (size_t c = 0; c < m->gate.cols; c++) { float p = w[c] * x[c]; z += p; }
            float e = or_expf(-z);
            float den = 1.0f + e;
            gsc = 1.0f / den;
        }
        for (size_t r = 0; r < dim; r++) { float t = gsc * tmp[r]; out[r] += t; }
        free(tmp);
    }
    if (chosen_out) memcpy(chosen_out, chosen, nk * sizeof(int32_t));
    if (weights_out) memcpy(weights_out, ws, nk * sizeof(float));
    if (n_chosen_out) *n_chosen_out = nk;
    free(probs);
    return rc;
}
