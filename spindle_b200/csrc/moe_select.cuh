// moe_select.cuh — the expert choice of moe_forward (smollm_chat.rs:1199-1240)
// by one CTA, from the router's logits: softmax, top-k (probability
// descending, equal probabilities by lower index), prune, mixing weights.
#pragma once

#include "tiled_block.cuh"

namespace sg {

namespace moe {

// Rust's f32::max: the other operand when one is NaN.
__device__ __forceinline__ float rmax(float a, float b) { return isnan(a) ? b : isnan(b) ? a : (a > b ? a : b); }

// f32::total_cmp's order as a signed integer key.
__device__ __forceinline__ int32_t total_key(float f) {
    const int32_t i = __float_as_int(f);
    return i ^ (int32_t)((uint32_t)(i >> 31) >> 1);
}

struct Choice {
    uint32_t n;
    int32_t id[MOE_MAXK];
    float w[MOE_MAXK];
};

// The prune rule and the weights over the top-k probabilities pv[0..k) (the
// same registers in every lane of the calling warp); lane i < k writes
// expert i of the choice.  The sums run in order, as the reference's.
__device__ __forceinline__ void choose(const float (&pv)[MOE_MAXK], const int32_t (&top)[MOE_MAXK], uint32_t k,
                                       int32_t norm, float prune, Choice *out, uint32_t lane) {
    uint32_t keep = k;
    if (prune > 0.0f && k > 2) {
        const uint32_t min_keep = k / 2 > 2 ? k / 2 : 2;
        if (prune >= 1.0f) {
            // `prune as usize` (saturating), clamped to [min_keep, k]
            const uint32_t p = prune >= 4294967040.0f ? 0xFFFFFFFFu : (uint32_t)prune;
            keep = p < min_keep ? min_keep : (p > k ? k : p);
        } else {
            float top_sum = 0.0f;
#pragma unroll
            for (uint32_t i = 0; i < MOE_MAXK; i++)
                if (i < k) top_sum = __fadd_rn(top_sum, pv[i]);
            const float target = __fmul_rn(top_sum, __fsub_rn(1.0f, prune));
            float cum = 0.0f;
            uint32_t n = 0;
#pragma unroll
            for (uint32_t i = 0; i < MOE_MAXK; i++) {
                if (n == i && i < k && (i < min_keep || cum < target)) {
                    cum = __fadd_rn(cum, pv[i]);
                    n = i + 1;
                }
            }
            keep = n;
        }
    }
    float wsum = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < MOE_MAXK; i++)
        if (i < keep) wsum = __fadd_rn(wsum, pv[i]);
    float mine = 0.0f;
    int32_t mid = 0;
#pragma unroll
    for (uint32_t i = 0; i < MOE_MAXK; i++)
        if (i == lane) {
            mine = pv[i];
            mid = top[i];
        }
    if (lane < MOE_MAXK) {
        const bool on = lane < keep;
        out->id[lane] = on ? mid : 0;
        out->w[lane] = on ? (norm ? __fdiv_rn(mine, wsum) : mine) : 0.0f;
    }
    if (lane == 0) out->n = keep;
}

// The whole choice by one warp, with up to 32 * R experts in registers
// (expert lane + 32 i in slot i): no block barrier.  S: 32 * R floats of
// shared memory (16-byte aligned) for the in-order sum.
template <int R>
__device__ __forceinline__ void select_warp(const float *logits, uint32_t ne, uint32_t k, int32_t norm, float prune,
                                            Choice *out, float *probs, float *S, uint32_t lane) {
    float p[R];
    bool valid[R];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < R; i++) {
        const uint32_t e = lane + 32u * i;
        valid[i] = e < ne;
        p[i] = valid[i] ? __ldcg(logits + e) : 0.0f;
        if (valid[i]) m = rmax(m, p[i]);
    }
    // max folded with f32::max (NaN ignored): any order gives the same value
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = rmax(m, __shfl_xor_sync(0xffffffffu, m, o));
#pragma unroll
    for (int i = 0; i < R; i++)
        if (valid[i]) p[i] = tiled::expf_ref(__fsub_rn(p[i], m));
    // the sum in expert order (Iterator::sum), replayed identically by every
    // lane from shared memory; each group of loads is issued before its adds
#pragma unroll
    for (int i = 0; i < R; i++) S[lane + 32u * i] = p[i];
    __syncwarp();
    float s = 0.0f;
    const float4 *S4 = reinterpret_cast<const float4 *>(S);
    uint32_t e = 0;
    for (; e + 32 <= ne; e += 32) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = S4[e / 4 + i];
#pragma unroll
        for (int i = 0; i < 8; i++) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[i].x), v[i].y), v[i].z), v[i].w);
    }
    for (; e < ne; e++) s = __fadd_rn(s, S[e]);
    uint32_t key[R];  // f32::total_cmp order as unsigned
#pragma unroll
    for (int i = 0; i < R; i++) {
        if (valid[i]) {
            p[i] = __fdiv_rn(p[i], s);
            if (probs) probs[lane + 32u * i] = p[i];
        }
        key[i] = (uint32_t)total_key(p[i]) ^ 0x80000000u;
    }
    // top-k: k rounds of (largest key, then lowest expert index among equals)
    float pv[MOE_MAXK];
    int32_t top[MOE_MAXK];
    uint32_t taken = 0;
#pragma unroll
    for (uint32_t r = 0; r < MOE_MAXK; r++) {
        pv[r] = 0.0f;
        top[r] = 0;
        if (r < k) {
            uint32_t bk = 0, be = 0xFFFFFFFFu;
            float bp = 0.0f;
            int bi = -1;
#pragma unroll
            for (int i = 0; i < R; i++)
                if (valid[i] && !(taken >> i & 1u) && (bi < 0 || key[i] > bk)) {
                    bk = key[i];
                    bi = i;
                    bp = p[i];
                    be = lane + 32u * i;
                }
            const uint32_t mk = __reduce_max_sync(0xffffffffu, bi >= 0 ? bk : 0u);
            const uint32_t win = __reduce_min_sync(0xffffffffu, bi >= 0 && bk == mk ? be : 0xFFFFFFFFu);
            if (be == win) taken |= 1u << bi;
            top[r] = (int32_t)win;
            pv[r] = __shfl_sync(0xffffffffu, bp, win & 31u);
        }
    }
    choose(pv, top, k, norm, prune, out, lane);
}

// All threads of the CTA call it.  P (16-byte aligned) and K: n_expert floats
// and keys; red: 64 floats of scratch; out: the choice (shared memory).
// Writes probs[e] when probs is not null.
static __device__ void select(const float *logits, uint32_t ne, uint32_t k, int32_t norm, float prune, float *P,
                       int32_t *K, float *red, Choice *out, float *probs) {
    const uint32_t tid = threadIdx.x, nt = blockDim.x, lane = tid & 31u, warp = tid >> 5;
    // max folded with f32::max (NaN ignored): any order gives the same value
    float m = -INFINITY;
    for (uint32_t e = tid; e < ne; e += nt) {
        P[e] = __ldcg(logits + e);
        m = rmax(m, P[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = rmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float mx = red[0];
    for (uint32_t w = 1; w < nt / 32; w++) mx = rmax(mx, red[w]);
    for (uint32_t e = tid; e < ne; e += nt) P[e] = tiled::expf_ref(__fsub_rn(P[e], mx));
    __syncthreads();
    if (tid == 0) {
        // the sum, in order (Iterator::sum); each group of loads is issued
        // before its adds so that the add chain does not wait on them
        float s = 0.0f;
        const float4 *P4 = reinterpret_cast<const float4 *>(P);
        uint32_t e = 0;
        for (; e + 32 <= ne; e += 32) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = P4[e / 4 + i];
#pragma unroll
            for (int i = 0; i < 8; i++) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[i].x), v[i].y), v[i].z), v[i].w);
        }
        for (; e < ne; e++) s = __fadd_rn(s, P[e]);
        red[32] = s;
    }
    __syncthreads();
    const float sum = red[32];
    for (uint32_t e = tid; e < ne; e += nt) {
        const float p = __fdiv_rn(P[e], sum);
        P[e] = p;
        K[e] = total_key(p);
        if (probs) probs[e] = p;
    }
    __syncthreads();
    // rank of e = experts before it in (probability descending, index
    // ascending) order; ranks 0..k-1 are the top-k in order.  Warp w ranks
    // experts w, w + nwarps, ...: its lanes hold 32 keys at a time and a
    // ballot counts those before e.
    int32_t *top = reinterpret_cast<int32_t *>(red + 40);
    const uint32_t nwarps = nt / 32, nchunks = (ne + 31) / 32;
    constexpr uint32_t KREG = 8;  // keys kept in registers (ne <= 256)
    int32_t kr[KREG];
#pragma unroll
    for (uint32_t c = 0; c < KREG; c++) kr[c] = c * 32 + lane < ne ? K[c * 32 + lane] : INT32_MIN;
    for (uint32_t e = warp; e < ne; e += nwarps) {
        const int32_t key = K[e];
        uint32_t cnt = 0;
#pragma unroll
        for (uint32_t c = 0; c < KREG; c++) {
            if (c < nchunks) {
                const uint32_t j = c * 32 + lane;
                cnt += __popc(__ballot_sync(0xffffffffu, j < ne && (kr[c] > key || (kr[c] == key && j < e))));
            }
        }
        for (uint32_t c = KREG; c < nchunks; c++) {
            const uint32_t j = c * 32 + lane;
            const int32_t kj = j < ne ? K[j] : INT32_MIN;
            cnt += __popc(__ballot_sync(0xffffffffu, j < ne && (kj > key || (kj == key && j < e))));
        }
        if (lane == 0 && cnt < k) top[cnt] = (int32_t)e;
    }
    __syncthreads();
    if (warp == 0) {
        // the top-k probabilities, one per lane; every lane replays the short
        // sequential sums of the prune rule and the weight normalization
        const float pv = lane < k ? P[top[lane]] : 0.0f;
        uint32_t keep = k;
        if (prune > 0.0f && k > 2) {
            const uint32_t min_keep = k / 2 > 2 ? k / 2 : 2;
            if (prune >= 1.0f) {
                // `prune as usize` (saturating), clamped to [min_keep, k]
                const uint32_t p = prune >= 4294967040.0f ? 0xFFFFFFFFu : (uint32_t)prune;
                keep = p < min_keep ? min_keep : (p > k ? k : p);
            } else {
                float top_sum = 0.0f;
                for (uint32_t i = 0; i < k; i++) top_sum = __fadd_rn(top_sum, __shfl_sync(0xffffffffu, pv, i));
                const float target = __fmul_rn(top_sum, __fsub_rn(1.0f, prune));
                float cum = 0.0f;
                uint32_t i = 0;
                while (i < k && (i < min_keep || cum < target)) {
                    cum = __fadd_rn(cum, __shfl_sync(0xffffffffu, pv, i));
                    i++;
                }
                keep = i;
            }
        }
        float wsum = 0.0f;
        for (uint32_t i = 0; i < keep; i++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, pv, i));
        if (lane < MOE_MAXK) {
            const bool on = lane < keep;
            out->id[lane] = on ? top[lane] : 0;
            out->w[lane] = on ? (norm ? __fdiv_rn(pv, wsum) : pv) : 0.0f;
        }
        if (lane == 0) out->n = keep;
    }
    __syncthreads();
}

}  // namespace moe

}  // namespace sg
