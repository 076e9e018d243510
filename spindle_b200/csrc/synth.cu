// synth.cu — the reference's synthetic benchmark kernels on the GPU: the
// float Q4_K GEMV of q4k_gemv.rs (one vector and the four-vector speculative
// form), the toy top-2-of-8 router of moe_engine.rs and the int8-KV flash
// decoding of transformer.rs.  The reference's early benchmark (main.rs)
// drives them; its chat engine does not.  Each reproduces the AVX2 kernel's
// operations in its order (the 8-lane FMA chains, the hsum256 tree, the
// sequential sums), so results are bit for bit the reference's.
#include "common.cuh"
#include "glibc_math.h"

namespace sg {
namespace {

constexpr uint32_t SY_HIDDEN = 4096, SY_ROW_BYTES = 2304, SY_NE = 8, SY_HEADS = 32, SY_KV_HEADS = 8, SY_HD = 128,
                   SY_GQA = 4, SY_KV_DIM = 1024, SY_MAX_SEQ = 512, SY_LAYERS = 32, SY_SPEC = 4;

// q4k_gemv.rs:37-68: IEEE for normal values, but exponents clamped to
// [-10, 4] and the Inf/NaN codes mapped to finite values
__device__ float synth_f16(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, mant = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            uint32_t m = mant;
            int32_t ex = 127 - 14;
            while ((m & 0x400u) == 0) {
                m <<= 1;
                ex -= 1;
            }
            bits = sign | ((uint32_t)ex << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        bits = sign | (119u << 23) | (mant << 13);
    } else {
        int32_t se = (int32_t)e - 15;
        se = se < -10 ? -10 : (se > 4 ? 4 : se);
        bits = sign | ((uint32_t)(se + 127) << 23) | (mant << 13);
    }
    return __uint_as_float(bits);
}

// q4k_block_dot_avx2 (q4k_gemv.rs:91-176) for each of nv vectors, by a pair
// of lanes: lane h of the pair keeps AVX lanes 4h..4h+3 of the 8-lane
// accumulator; returns the dot (hsum256 tree) in both lanes of the pair.
template <int NV>
__device__ void block_dot_pair(const uint8_t *blk, const float *const *act, uint32_t h, float (&dot)[NV]) {
    const float d = synth_f16(blk[0] | (blk[1] << 8)), dmin = synth_f16(blk[2] | (blk[3] << 8));
    const uint8_t *sc = blk + 4;
    float acc[NV][4];
#pragma unroll
    for (int v = 0; v < NV; v++)
#pragma unroll
        for (int m = 0; m < 4; m++) acc[v][m] = 0.0f;
    for (int c = 0; c < 4; c++) {
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int sb = 2 * c + half;
            uint32_t s, mn;
            if (sb < 4) {
                s = sc[sb] & 63u;
                mn = sc[sb + 4] & 63u;
            } else {
                s = (sc[sb + 4] & 0x0Fu) | ((sc[sb - 4] >> 6) << 4);
                mn = (sc[sb + 4] >> 4) | ((sc[sb] >> 6) << 4);
            }
            const float scale = __fmul_rn(d, (float)s), neg_min = __fmul_rn(-dmin, (float)mn);
#pragma unroll
            for (int g = 0; g < 4; g++) {
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    const uint32_t L = 4 * h + m;
                    const uint32_t byte = blk[16 + 32 * c + 8 * g + L];
                    const float dq = __fmaf_rn((float)(half ? byte >> 4 : byte & 15u), scale, neg_min);
#pragma unroll
                    for (int v = 0; v < NV; v++)
                        acc[v][m] = __fmaf_rn(dq, act[v][64 * c + 32 * half + 8 * g + L], acc[v][m]);
                }
            }
        }
    }
#pragma unroll
    for (int v = 0; v < NV; v++) {
        float x[4];
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const float other = __shfl_xor_sync(0xffffffffu, acc[v][m], 1);
            x[m] = h == 0 ? __fadd_rn(acc[v][m], other) : __fadd_rn(other, acc[v][m]);  // low half + high half
        }
        dot[v] = __fadd_rn(__fadd_rn(x[0], x[1]), __fadd_rn(x[2], x[3]));
    }
}

// One warp per output index j (of 4096): the rows that land on j, in
// increasing row order, each as the reference computes it (16 block dots
// summed in order), added to y.  Rows r with (base + r) & 4095 == j and
// r0 <= r < r1; x holds NV vectors 4096 apart, y likewise.
template <int NV>
__global__ void synth_gemv_kernel(const uint8_t *chunk, uint64_t r0, uint64_t r1, const float *x, float *y,
                                  uint64_t base) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= SY_HIDDEN) return;
    const uint64_t first = (uint64_t)((j - (uint32_t)(base & (SY_HIDDEN - 1))) & (SY_HIDDEN - 1));
    uint64_t r = first;
    if (r < r0) r += (r0 - r + SY_HIDDEN - 1) / SY_HIDDEN * SY_HIDDEN;
    const uint32_t b = lane >> 1, h = lane & 1u;
    const float *act[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) act[v] = x + (uint64_t)v * SY_HIDDEN + 256u * b;
    for (; r < r1; r += SY_HIDDEN) {
        float dot[NV];
        block_dot_pair<NV>(chunk + r * SY_ROW_BYTES + 144u * b, act, h, dot);
        float sum[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) sum[v] = 0.0f;
        for (uint32_t bb = 0; bb < 16; bb++)
#pragma unroll
            for (int v = 0; v < NV; v++) sum[v] = __fadd_rn(sum[v], __shfl_sync(0xffffffffu, dot[v], 2 * bb));
        if (lane == 0)
#pragma unroll
            for (int v = 0; v < NV; v++) y[(uint64_t)v * SY_HIDDEN + j] = __fadd_rn(y[(uint64_t)v * SY_HIDDEN + j], sum[v]);
    }
}

// route_moe_top2 (moe_engine.rs:124-164): one block of 8 warps; warp e's lane
// 0 runs expert e's strided dot in order.
__global__ void synth_route_kernel(const float *x, const float *gates, uint64_t layer, int32_t *experts,
                                   float *weights) {
    __shared__ float s[SY_NE];
    const uint32_t e = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (e < SY_NE && lane == 0) {
        float acc = 0.0f;
        for (uint32_t i = 0; i < SY_HIDDEN; i += 16) acc = __fadd_rn(acc, __fmul_rn(x[i], gates[e * SY_HIDDEN + i]));
        acc = __fadd_rn(acc, __fmul_rn((float)((layer + e) % SY_NE), 0.05f));
        s[e] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int b0 = 0, b1 = 1;
        if (s[b1] > s[b0]) {
            b0 = 1;
            b1 = 0;
        }
        for (int k = 2; k < (int)SY_NE; k++) {
            if (s[k] > s[b0]) {
                b1 = b0;
                b0 = k;
            } else if (s[k] > s[b1]) {
                b1 = k;
            }
        }
        const float mx = s[b0];
        const float w0 = gm_expf(__fsub_rn(s[b0], mx)), w1 = gm_expf(__fsub_rn(s[b1], mx));
        const float inv = __fdiv_rn(1.0f, __fadd_rn(w0, w1));
        experts[0] = b0;
        experts[1] = b1;
        weights[0] = __fmul_rn(w0, inv);
        weights[1] = __fmul_rn(w1, inv);
    }
}

__device__ __forceinline__ float fmax_rust(float a, float b) {  // f32::max: a NaN yields the other
    return isnan(a) ? b : (isnan(b) ? a : (a > b ? a : b));
}

// quantize_kv_step_avx2 (transformer.rs:455-479) of token k's vector into K
// (blockIdx.y 0) or V (1) at position base + k: one warp per KV head.
__global__ void synth_kv_quant_kernel(const float *q_spec, int8_t *kq, int8_t *vq, float *ks, float *vs,
                                      uint64_t l, uint64_t base) {
    const uint32_t k = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const float *src = q_spec + (uint64_t)k * SY_HIDDEN + h * SY_HD;
    float mx = 1e-6f;
    for (uint32_t d = lane; d < SY_HD; d += 32) {
        const float a = fabsf(src[d]);
        if (a > mx) mx = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float inv = __fdiv_rn(127.0f, mx);
    const uint64_t row = l * SY_MAX_SEQ + base + k;
    int8_t *q = (blockIdx.y ? vq : kq) + row * SY_KV_DIM + h * SY_HD;
    if (lane == 0) (blockIdx.y ? vs : ks)[row * SY_KV_HEADS + h] = __fdiv_rn(mx, 127.0f);
    for (uint32_t d = lane; d < SY_HD; d += 32) {
        float r = roundf(__fmul_rn(src[d], inv));  // f32::round: half away from zero
        q[d] = isnan(r) ? (int8_t)0 : (int8_t)(r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r));
    }
}

// flash_decoding_gqa_spec4_avx2's attention (transformer.rs:541-600): one CTA
// of 128 threads per (query head, draft token).  Scores of all positions in
// parallel (each the reference's dot: two 8-lane FMA accumulators, their sum,
// the hsum256 tree, times the scale, the clamp), the m / alpha / p / l
// recurrences by one thread in position order, then thread d runs its output
// element's recurrence out = fma(v, p * vscale, out * alpha) in order.
__global__ void synth_flash_kernel(float *q_spec, const int8_t *kq, const int8_t *vq, const float *ks,
                                   const float *vs, uint64_t l, uint64_t base) {
    __shared__ float sc[SY_MAX_SEQ], al[SY_MAX_SEQ], qv[SY_HD];
    __shared__ float inv_l;
    const uint32_t qh = blockIdx.x, k = blockIdx.y, kvh = qh / SY_GQA, t = threadIdx.x;
    const uint64_t end = base + k + 1;
    float *q = q_spec + (uint64_t)k * SY_HIDDEN + qh * SY_HD;
    qv[t] = q[t];
    __syncthreads();
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)SY_HD));
    for (uint64_t p = t; p < end; p += blockDim.x) {
        const uint64_t row = l * SY_MAX_SEQ + p;
        const int8_t *kr = kq + row * SY_KV_DIM + kvh * SY_HD;
        float a0[8], a1[8];
#pragma unroll
        for (int i = 0; i < 8; i++) a0[i] = a1[i] = 0.0f;
        for (int d = 0; d < (int)SY_HD; d += 16)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                a0[i] = __fmaf_rn(qv[d + i], (float)kr[d + i], a0[i]);
                a1[i] = __fmaf_rn(qv[d + 8 + i], (float)kr[d + 8 + i], a1[i]);
            }
        float sm[8];
#pragma unroll
        for (int i = 0; i < 8; i++) sm[i] = __fadd_rn(a0[i], a1[i]);
        const float x0 = __fadd_rn(sm[0], sm[4]), x1 = __fadd_rn(sm[1], sm[5]), x2 = __fadd_rn(sm[2], sm[6]),
                    x3 = __fadd_rn(sm[3], sm[7]);
        const float dot = __fmul_rn(__fadd_rn(__fadd_rn(x0, x1), __fadd_rn(x2, x3)), ks[row * SY_KV_HEADS + kvh]);
        float s = __fmul_rn(dot, inv_sqrt_d);
        s = s < -20.0f ? -20.0f : (s > 20.0f ? 20.0f : s);
        sc[p] = s;
    }
    __syncthreads();
    if (t == 0) {
        float m_prev = -INFINITY, l_prev = 0.0f;
        for (uint64_t p = 0; p < end; p++) {
            const float m_new = fmax_rust(m_prev, sc[p]);
            const float alpha = gm_expf(__fsub_rn(m_prev, m_new)), pp = gm_expf(__fsub_rn(sc[p], m_new));
            l_prev = __fadd_rn(__fmul_rn(l_prev, alpha), pp);
            m_prev = m_new;
            al[p] = alpha;
            sc[p] = __fmul_rn(pp, vs[(l * SY_MAX_SEQ + p) * SY_KV_HEADS + kvh]);  // p * v_scale
        }
        inv_l = __fdiv_rn(1.0f, fmax_rust(l_prev, 1e-8f));
    }
    __syncthreads();
    float out = 0.0f;
    for (uint64_t p = 0; p < end; p++)
        out = __fmaf_rn((float)vq[(l * SY_MAX_SEQ + p) * SY_KV_DIM + kvh * SY_HD + t], sc[p], __fmul_rn(out, al[p]));
    q[t] = __fmul_rn(out, inv_l);
}

}  // namespace
}  // namespace sg

using namespace sg;

extern "C" {

sg_status sg_q4k_gemv_4row(const uint8_t *d_chunk, uint64_t chunk_len, const float *d_x, float *d_y,
                           uint64_t row_offset, uint64_t *rows_done, void *stream) {
    if ((chunk_len && !d_chunk) || !d_x || !d_y) return SG_ERR_INVALID;
    const uint64_t rows = chunk_len / SY_ROW_BYTES / 4 * 4;  // whole groups of four rows only
    if (rows_done) *rows_done = rows;
    if (!rows) return SG_OK;
    synth_gemv_kernel<1><<<SY_HIDDEN / 8, 256, 0, (cudaStream_t)stream>>>(d_chunk, 0, rows, d_x, d_y, row_offset);
    return cudaGetLastError() == cudaSuccess ? SG_OK : SG_ERR_CUDA;
}

sg_status sg_q4k_gemm_spec4(const uint8_t *d_chunk, uint64_t r0, uint64_t r1, const float *d_x4, float *d_y4,
                            uint64_t base, void *stream) {
    if (!d_chunk || !d_x4 || !d_y4 || r0 > r1) return SG_ERR_INVALID;
    if (r0 == r1) return SG_OK;
    synth_gemv_kernel<4><<<SY_HIDDEN / 8, 256, 0, (cudaStream_t)stream>>>(d_chunk, r0, r1, d_x4, d_y4, base);
    return cudaGetLastError() == cudaSuccess ? SG_OK : SG_ERR_CUDA;
}

sg_status sg_route_moe_top2(const float *d_x, const float *d_gates, uint64_t layer, int32_t *d_experts,
                            float *d_weights, void *stream) {
    if (!d_x || !d_gates || !d_experts || !d_weights) return SG_ERR_INVALID;
    synth_route_kernel<<<1, 32 * SY_NE, 0, (cudaStream_t)stream>>>(d_x, d_gates, layer, d_experts, d_weights);
    return cudaGetLastError() == cudaSuccess ? SG_OK : SG_ERR_CUDA;
}

sg_status sg_flash_gqa_spec4(float *d_q_spec, int8_t *d_kq, int8_t *d_vq, float *d_ks, float *d_vs,
                             uint64_t seq_len, uint64_t layer, void *stream) {
    if (!d_q_spec || !d_kq || !d_vq || !d_ks || !d_vs) return SG_ERR_INVALID;
    const uint64_t l = layer % SY_LAYERS, base = seq_len < SY_MAX_SEQ - SY_SPEC ? seq_len : SY_MAX_SEQ - SY_SPEC;
    cudaStream_t s = (cudaStream_t)stream;
    synth_kv_quant_kernel<<<dim3(SY_SPEC, 2), 32 * SY_KV_HEADS, 0, s>>>(d_q_spec, d_kq, d_vq, d_ks, d_vs, l, base);
    synth_flash_kernel<<<dim3(SY_HEADS, SY_SPEC), SY_HD, 0, s>>>(d_q_spec, d_kq, d_vq, d_ks, d_vs, l, base);
    return cudaGetLastError() == cudaSuccess ? SG_OK : SG_ERR_CUDA;
}

}  // extern "C"
