// decode.cu — embedding, RMSNorm, RoPE + KV write, attention and argmax of one
// decoder step (see decode.cuh).
#include "decode.cuh"
#include "gemv_tiled.cuh"
#include "q8k_block.cuh"
#include "tiled_block.cuh"

namespace sg {
using namespace tiled;

namespace {

__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

}  // namespace

// One thread per output value, the arithmetic of dequant_row.
__global__ void embed_kernel(const __grid_constant__ EmbedArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.dim) return;
    const int32_t tok = a.state[0];
    if (tok < 0 || (uint32_t)tok >= a.vocab) {
        if (i == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        a.x[i] = __int_as_float(0x7fc00000);
        return;
    }
    float y;
    if (a.dtype == SG_F32) {
        y = reinterpret_cast<const float *>(a.embed)[(uint64_t)tok * a.dim + i];
    } else if (a.dtype == SG_F16) {
        y = f16_at(a.embed + ((uint64_t)tok * a.dim + i) * 2);
    } else if (a.dtype == SG_Q4_K) {
        const uint8_t *blk = a.embed + (uint64_t)tok * (a.dim / 256) * 144 + (i / 256) * 144;
        const uint32_t o = i % 256, c = o / 64, j = o % 64, sub = 2 * c + (j >= 32);
        const float d = f16_at(blk), dmin = f16_at(blk + 2);
        const uint8_t *s = blk + 4;
        // get_scale_min_k4 (the 6-bit packing of Q4_K scales and mins)
        const uint32_t sc = sub < 4 ? (s[sub] & 63u) : ((s[sub + 4] & 0xFu) | ((s[sub - 4] >> 6) << 4));
        const uint32_t mn = sub < 4 ? (s[sub + 4] & 63u) : ((s[sub + 4] >> 4) | ((s[sub] >> 6) << 4));
        const uint32_t qb = blk[16 + c * 32 + (j & 31u)], q = j < 32 ? (qb & 0xFu) : (qb >> 4);
        const float sv = __fmul_rn(d, (float)sc), ov = __fmul_rn(dmin, (float)mn);
        y = __fsub_rn(__fmul_rn(sv, (float)q), ov);
    } else {  // SG_Q6_K
        const uint8_t *blk = a.embed + (uint64_t)tok * (a.dim / 256) * 210 + (i / 256) * 210;
        const uint32_t o = i % 256, half = o / 128, quad = (o % 128) / 32, l = o % 32;
        const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + half * 8);
        const uint32_t lo = (quad & 1u) ? ql[l + 32] : ql[l];
        const uint32_t nib = (quad & 2u) ? (lo >> 4) : (lo & 0xFu);
        const int q = (int)(nib | (((qh[l] >> (2 * quad)) & 3u) << 4)) - 32;
        const float d = f16_at(blk + 208);
        y = __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * quad]), (float)q);
    }
    if (a.scale != 1.0f) y = __fmul_rn(y, a.scale);
    a.x[i] = y;
}

// The sum of squares of n values in shared memory, one element after the other
// (Iterator::sum over v * v, as rmsnorm does): one thread, loads issued in
// groups ahead of the dependent adds.  n a multiple of 4, xs 16-byte aligned.
__device__ float seq_sum_squares(const float *xs, uint32_t n) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    float s = 0.0f;
    uint32_t i = 0;
    for (; i + 32 <= n; i += 32) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = x4[i / 4 + j];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            s = __fadd_rn(s, __fmul_rn(v[j].x, v[j].x));
            s = __fadd_rn(s, __fmul_rn(v[j].y, v[j].y));
            s = __fadd_rn(s, __fmul_rn(v[j].z, v[j].z));
            s = __fadd_rn(s, __fmul_rn(v[j].w, v[j].w));
        }
    }
    for (; i < n; i++) s = __fadd_rn(s, __fmul_rn(xs[i], xs[i]));
    return s;
}

// One CTA.  Each thread keeps up to 8 of the n values in registers; the sum of
// squares is the reference's sequential one, so xn (and its Q8_K image) are
// the reference's bits.
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const __grid_constant__ NormArgs a) {
    __shared__ float inv_s;
    extern __shared__ __align__(16) float xs[];  // x, then the normed vector for the Q8_K image
    grid_dependency_wait();
    grid_launch_dependents();
    constexpr int PER = 8;
    if (a.n > PER * blockDim.x || a.n % 4 || a.n * 4 > dynamic_smem_size() || (a.qx && a.n % 256)) {
        if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    float v[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const uint32_t i = threadIdx.x + j * blockDim.x;
        v[j] = 0.0f;
        if (i < a.n) {
            float x = a.x[i];
            if (a.add) {
                x = __fadd_rn(x, __fmul_rn(a.rs, a.add[i]));
                a.x[i] = x;
            }
            v[j] = x;
            xs[i] = x;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float ss = seq_sum_squares(xs, a.n);
        inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.n), a.eps)));
    }
    __syncthreads();
    const float inv = inv_s;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const uint32_t i = threadIdx.x + j * blockDim.x;
        if (i < a.n) {
            const float y = __fmul_rn(__fmul_rn(v[j], inv), a.w[i]);
            a.xn[i] = y;
            if (a.qx) xs[i] = y;
        }
    }
    if (a.qx) {
        __syncthreads();
        const uint32_t nb = a.n / 256, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
        for (uint32_t b = warp; b < nb; b += blockDim.x / 32)
            q8k_block(xs + 256u * b, reinterpret_cast<int8_t *>(a.qx + 256u * b),
                      reinterpret_cast<int16_t *>(a.qx + 256u * nb + 32u * b),
                      reinterpret_cast<float *>(a.qx + 288u * nb + 4u * b), lane);
    }
}

// One warp per head: q heads first, then k heads (each also writes its v head).
__global__ void rope_kv_kernel(const __grid_constant__ RopeArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t h = blockIdx.x, lane = threadIdx.x, hd = a.head_dim, half = hd / 2;
    const bool is_q = h < a.n_heads;
    const uint32_t kh = is_q ? 0u : h - a.n_heads;
    const uint32_t pos = (uint32_t)a.state[1];
    if (hd > 256 || (hd & 63u) || pos >= a.max_seq || blockDim.x != 32) {
        if (lane == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    const float *src = is_q ? a.q + h * hd : a.k + kh * hd;
    const float *nw = is_q ? a.qn_w : a.kn_w;
    // lane holds the pairs (i, i + half), i = lane + 32 j
    constexpr int MAXP = 4;
    const uint32_t np = half / 32;
    float x0[MAXP], x1[MAXP];
    __shared__ __align__(16) float hs[256];
#pragma unroll
    for (int j = 0; j < MAXP; j++)
        if ((uint32_t)j < np) {
            const uint32_t i = lane + 32u * j;
            const uint32_t ia = a.neox ? i : 2 * i, ib = a.neox ? i + half : 2 * i + 1;
            x0[j] = src[ia];
            x1[j] = src[ib];
            hs[ia] = x0[j];
            hs[ib] = x1[j];
        }
    if (nw) {
        // rmsnorm_heads: the head's sum of squares in element order, by lane 0
        __syncwarp();
        float inv = 0.0f;
        if (lane == 0) inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(seq_sum_squares(hs, hd), (float)hd), a.eps)));
        inv = __shfl_sync(0xffffffffu, inv, 0);
#pragma unroll
        for (int j = 0; j < MAXP; j++)
            if ((uint32_t)j < np) {
                const uint32_t i = lane + 32u * j;
                const uint32_t ia = a.neox ? i : 2 * i, ib = a.neox ? i + half : 2 * i + 1;
                x0[j] = __fmul_rn(__fmul_rn(x0[j], inv), nw[ia]);
                x1[j] = __fmul_rn(__fmul_rn(x1[j], inv), nw[ib]);
            }
    }
    const float fpos = (float)pos;
    const uint32_t kv_dim = a.n_kv * hd;
#pragma unroll
    for (int j = 0; j < MAXP; j++)
        if ((uint32_t)j < np) {
            const uint32_t i = lane + 32u * j;
            const uint32_t ia = a.neox ? i : 2 * i, ib = a.neox ? i + half : 2 * i + 1;
            const float ang = __fmul_rn(fpos, a.inv_freq[i]);
            const float s = (float)sin((double)ang), c = (float)cos((double)ang);
            const float y0 = __fsub_rn(__fmul_rn(x0[j], c), __fmul_rn(x1[j], s));
            const float y1 = __fadd_rn(__fmul_rn(x0[j], s), __fmul_rn(x1[j], c));
            if (is_q) {
                a.q[h * hd + ia] = y0;
                a.q[h * hd + ib] = y1;
            } else {
                uint16_t *kr = a.kc + (uint64_t)pos * kv_dim + kh * hd;
                kr[ia] = __half_as_ushort(__float2half_rn(y0));
                kr[ib] = __half_as_ushort(__float2half_rn(y1));
            }
        }
    if (!is_q) {
        uint16_t *vr = a.vc + (uint64_t)pos * kv_dim + kh * hd;
        for (uint32_t i = lane; i < hd; i += 32) vr[i] = __half_as_ushort(__float2half_rn(a.v[kh * hd + i]));
    }
}

// One CTA per query head: compute_head_fn (smollm_chat.rs:3463-3495) with the
// reference's bits.  Its online softmax is a recurrence over positions, but
// most of it does not depend on the recurrence: the scores (dot_f16_row_avx2,
// quant.rs:1412-1425, times scale), the running maxima m_t (a prefix maximum
// under f32::max), alpha_t = exp(m_{t-1} - m_t) and p_t = exp(s_t - m_t) are
// computed for all positions in parallel; only l_t = l_{t-1} * alpha_t + p_t
// (one thread) and acc_t[d] = fma(p_t, v_t[d], acc_{t-1}[d] * alpha_t) (one
// thread per d) run position by position.
__global__ void __launch_bounds__(ATTN_THREADS) attention_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t h = blockIdx.x, hd = a.head_dim, tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t nwarps = blockDim.x / 32, pos = (uint32_t)a.state[1], T = pos + 1;
    if (hd > 256 || (hd & 63u) || pos >= a.max_seq || attn_smem_bytes(hd, a.max_seq) > dynamic_smem_size() ||
        blockDim.x != ATTN_THREADS) {
        if (tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    // q | s (scores, then p) | al (alpha) | l
    float *qs = sm, *sc = sm + hd, *al = sc + a.max_seq, *lsh = al + a.max_seq;
    const uint32_t kvh = h / (a.n_heads / a.n_kv), kv_dim = a.n_kv * hd;
    for (uint32_t d = tid; d < hd; d += blockDim.x) qs[d] = a.q[h * hd + d];
    __syncthreads();
    // scores: 8 lanes per position (the 8 AVX lanes), 4 positions per warp
    const uint32_t grp = lane >> 3, l8 = lane & 7u, nsteps = hd / 8;
    for (uint32_t t0 = warp * 4; t0 < T; t0 += nwarps * 4) {
        const uint32_t t = t0 + grp;
        float acc = 0.0f;
        if (t < T) {
            const uint16_t *kr = a.kc + (uint64_t)t * kv_dim + kvh * hd;
            for (uint32_t i = 0; i < nsteps; i++)
                acc = __fmaf_rn(__half2float(__ushort_as_half(kr[8 * i + l8])), qs[8 * i + l8], acc);
        }
        // hsum_avx2: ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)), + the empty tail (0.0)
        const float x4 = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
        const float x1 = __fadd_rn(x4, __shfl_down_sync(0xffffffffu, x4, 1));
        const float x2 = __fadd_rn(x1, __shfl_down_sync(0xffffffffu, x1, 2));
        if (t < T && l8 == 0) sc[t] = __fmul_rn(__fadd_rn(x2, 0.0f), a.scale);
    }
    __syncthreads();
    // running maxima (f32::max ignores NaN: any grouping gives the same), by warp 0
    if (warp == 0) {
        float carry = -INFINITY;
        for (uint32_t t0 = 0; t0 < T; t0 += 32) {
            const uint32_t t = t0 + lane;
            float m = t < T ? sc[t] : -INFINITY;
            if (isnan(m)) m = -INFINITY;  // f32::max(prev, NaN) = prev
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float u = __shfl_up_sync(0xffffffffu, m, o);
                if (lane >= (uint32_t)o) m = fmaxf(m, u);
            }
            m = fmaxf(m, carry);
            const float prev = __shfl_up_sync(0xffffffffu, m, 1);
            const float mprev = lane == 0 ? carry : prev;
            if (t < T) {
                // alpha_t = exp(m_{t-1} - m_t), p_t = exp(s_t - m_t)
                al[t] = expf_cr(__fsub_rn(mprev, m));
                sc[t] = expf_cr(__fsub_rn(sc[t], m));
            }
            carry = __shfl_sync(0xffffffffu, m, 31);
        }
    }
    __syncthreads();
    if (tid == 0) {
        float l = 0.0f;
        for (uint32_t t = 0; t < T; t++) l = __fadd_rn(__fmul_rn(l, al[t]), sc[t]);
        *lsh = __fdiv_rn(1.0f, l > 1e-9f ? l : 1e-9f);  // 1 / l.max(1e-9): a NaN l gives 1e-9
    }
    // acc[d] over positions, one thread per d (V loads run ahead of the chain)
    float acc = 0.0f;
    if (tid < hd) {
        const uint16_t *vr = a.vc + kvh * hd + tid;
#pragma unroll 8
        for (uint32_t t = 0; t < T; t++)
            acc = __fmaf_rn(sc[t], __half2float(__ushort_as_half(vr[(uint64_t)t * kv_dim])), __fmul_rn(acc, al[t]));
    }
    __syncthreads();
    if (tid < hd) a.out[h * hd + tid] = __fmul_rn(acc, *lsh);
}

// One CTA: (total_cmp key, index) maximum with the larger index on ties.
__global__ void __launch_bounds__(ARGMAX_THREADS) argmax_kernel(const __grid_constant__ ArgmaxArgs a) {
    __shared__ unsigned long long red[32];
    grid_dependency_wait();
    grid_launch_dependents();
    unsigned long long best = 0;
    for (uint32_t i = threadIdx.x; i < a.n; i += blockDim.x) {
        const int32_t b = __float_as_int(a.logits[i]);
        const uint32_t key = (uint32_t)(b ^ (int32_t)((uint32_t)(b >> 31) >> 1)) ^ 0x80000000u;
        const unsigned long long v = ((unsigned long long)key << 32) | i;
        best = v > best ? v : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long u = __shfl_xor_sync(0xffffffffu, best, o);
        best = u > best ? u : best;
    }
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t w = 1; w < blockDim.x / 32; w++) best = red[w] > best ? red[w] : best;
        const int32_t tok = (int32_t)(best & 0xFFFFFFFFull);
        a.state[0] = tok;
        a.state[1] = a.state[1] + 1;
        if (a.out) *a.out = tok;
    }
}

}  // namespace sg
