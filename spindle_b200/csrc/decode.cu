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
    if (a.n_out && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *a.n_out = gridDim.y;
    if (i >= a.dim) return;
    const int32_t tok = a.tokens ? a.tokens[blockIdx.y] : a.state[0];
    float *const xo = a.x + (uint64_t)blockIdx.y * a.dim;
    if (tok < 0 || (uint32_t)tok >= a.vocab) {
        if (i == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        xo[i] = __int_as_float(0x7fc00000);
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
    xo[i] = y;
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

// One CTA per token; warp w holds 256-block w of the n values (lane l: values
// 8l..8l+7), so that the block's Q8_K image is made from registers.  The norm
// weights do not depend on the kernel before and are loaded before waiting for
// it.  The sum of squares is the reference's sequential one (thread 0), so xn
// and its Q8_K image are the reference's bits.
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const __grid_constant__ NormArgs a) {
    __shared__ float inv_s;
    __shared__ float cw[MOE_MAXK];
    __shared__ uint32_t cn_s;
    extern __shared__ __align__(16) float xs[];  // x in element order, for the sequential sum
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nb = a.n / 256;
    const bool bad = a.n % 256 || nb * 32 > blockDim.x || a.n * 4 > dynamic_smem_size() || (a.csel && gridDim.x != 1);
    const bool mine = !bad && warp < nb;
    const uint32_t i0 = 256u * warp + 8u * lane;
    float wv[8];
    if (mine) {
        const float4 w0 = reinterpret_cast<const float4 *>(a.w + i0)[0], w1 = reinterpret_cast<const float4 *>(a.w + i0)[1];
        wv[0] = w0.x, wv[1] = w0.y, wv[2] = w0.z, wv[3] = w0.w, wv[4] = w1.x, wv[5] = w1.y, wv[6] = w1.z, wv[7] = w1.w;
    }
    grid_dependency_wait();
    grid_launch_dependents();
    if (bad) {
        if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    // CTA t: token t of a batch (one token: t = 0)
    const uint64_t to = (uint64_t)blockIdx.x * a.n;
    float *const X = a.x + to, *const XN = a.xn + to;
    const float *const ADD = a.add ? a.add + to : nullptr;
    uint8_t *const QX = a.qx ? a.qx + (uint64_t)blockIdx.x * act_bytes(nb) : nullptr;
    if (a.csel) {
        if (threadIdx.x < MOE_MAXK) cw[threadIdx.x] = a.csel->weight[threadIdx.x];
        if (threadIdx.x == 0) cn_s = min(a.csel->n, a.cmax_slots);
        __syncthreads();
    }
    float v[8];
    if (mine) {
        const float4 p0 = reinterpret_cast<const float4 *>(X + i0)[0], p1 = reinterpret_cast<const float4 *>(X + i0)[1];
        v[0] = p0.x, v[1] = p0.y, v[2] = p0.z, v[3] = p0.w, v[4] = p1.x, v[5] = p1.y, v[6] = p1.z, v[7] = p1.w;
        if (ADD || a.csel) {
            float ad[8];
            if (ADD) {
                const float4 q0 = reinterpret_cast<const float4 *>(ADD + i0)[0], q1 = reinterpret_cast<const float4 *>(ADD + i0)[1];
                ad[0] = q0.x, ad[1] = q0.y, ad[2] = q0.z, ad[3] = q0.w, ad[4] = q1.x, ad[5] = q1.y, ad[6] = q1.z, ad[7] = q1.w;
            } else {
                // ffns_fused on a zeroed output: 0 + w_0*y_0 + w_1*y_1 + ... (smollm_chat.rs:431-438),
                // then the shared expert's g * (0 + 1 * ysh) (:1370-1382)
#pragma unroll
                for (int j = 0; j < 8; j++) ad[j] = 0.0f;
                for (uint32_t q = 0; q < cn_s; q++) {
                    const float4 y0 = reinterpret_cast<const float4 *>(a.cy + (uint64_t)q * a.n + i0)[0];
                    const float4 y1 = reinterpret_cast<const float4 *>(a.cy + (uint64_t)q * a.n + i0)[1];
                    const float yv[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
#pragma unroll
                    for (int j = 0; j < 8; j++) ad[j] = __fadd_rn(ad[j], __fmul_rn(cw[q], yv[j]));
                }
                if (a.cysh) {
                    const float g = *a.cscale;
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        ad[j] = __fadd_rn(ad[j], __fmul_rn(g, __fadd_rn(0.0f, __fmul_rn(1.0f, a.cysh[i0 + j]))));
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = __fadd_rn(v[j], __fmul_rn(a.rs, ad[j]));
            reinterpret_cast<float4 *>(X + i0)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4 *>(X + i0)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        reinterpret_cast<float4 *>(xs + i0)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(xs + i0)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float ss = seq_sum_squares(xs, a.n);
        inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.n), a.eps)));
    }
    __syncthreads();
    if (mine) {
        const float inv = inv_s;
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; j++) y[j] = __fmul_rn(__fmul_rn(v[j], inv), wv[j]);
        reinterpret_cast<float4 *>(XN + i0)[0] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4 *>(XN + i0)[1] = make_float4(y[4], y[5], y[6], y[7]);
        if (QX)
            q8k_block_regs(y, reinterpret_cast<int8_t *>(QX + 256u * warp),
                           reinterpret_cast<int16_t *>(QX + 256u * nb + 32u * warp),
                           reinterpret_cast<float *>(QX + 288u * nb + 4u * warp), lane);
    }
}

// One CTA per query head: this position's QK-norm, RoPE and f16 K/V (as
// rmsnorm_heads, Rope::rotate and the cache write of forward_slice,
// smollm_chat.rs:578-584, :1408-1419, :3431-3445), then compute_head_fn
// (:3463-3495) with the reference's bits.  Its online softmax is a recurrence
// over positions, but most of it does not depend on the recurrence: the scores
// (dot_f16_row_avx2, quant.rs:1412-1425, times scale), the running maxima m_t (a
// prefix maximum under f32::max), alpha_t = exp(m_{t-1} - m_t) and
// p_t = exp(s_t - m_t) are computed for all positions in parallel; only
// l_t = l_{t-1} * alpha_t + p_t (one thread) and
// acc_t[d] = fma(p_t, v_t[d], acc_{t-1}[d] * alpha_t) (one thread per d) run
// position by position.  The K and V rows of earlier positions were written by
// earlier steps, so their copies into shared memory are issued before the
// kernel waits for its predecessor; positions go through in chunks of
// a.chunk rows (64 or 128).
template <int HD, int CHK>
__global__ void __launch_bounds__(HD < 256 ? 256 : 288) attention_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) uint8_t sm8[];
    constexpr uint32_t RS = 2 * HD + ATTN_ROW_PAD, HALF = HD / 2;
    const uint32_t h = blockIdx.x, tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const bool prep = a.prepared != 0;
    const uint32_t nwarps = blockDim.x / 32, pos = prep ? (uint32_t)a.state[0] + blockIdx.y : (uint32_t)a.state[1];
    const uint32_t T = pos + 1;
    const uint32_t msq = attn_seq4(a.max_seq);
    const uint32_t NB = a.nbuf;
    if (a.head_dim != HD || pos >= a.max_seq || NB < 2 || NB > ATTN_MAX_BUF || a.chunk != (uint32_t)CHK ||
        attn_smem_bytes(HD, a.max_seq, NB, CHK) > dynamic_smem_size() ||
        blockDim.x != attn_threads(HD) || a.n_heads % a.n_kv) {
        grid_dependency_wait();
        if (tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    float *lsh = reinterpret_cast<float *>(sm8 + 32);          // 1/l, then inv_q, inv_k
    float *qs = reinterpret_cast<float *>(sm8 + 64);
    float *hs = qs + HD;                                       // q, then k, before RoPE
    float *sc = hs + 2 * HD, *al = sc + msq;
    uint8_t *bufs = reinterpret_cast<uint8_t *>(al + msq);
    uint16_t *kcur = reinterpret_cast<uint16_t *>(bufs + NB * CHK * RS), *vcur = kcur + HD;
    const uint32_t kvh = h / (a.n_heads / a.n_kv), kv_dim = a.n_kv * HD;
    const uint16_t *kg = a.kc + kvh * HD, *vg = a.vc + kvh * HD;

    // Rows of the earlier positions move in items: K chunks 0..nc-1, then V
    // chunks 0..nc-1 (CHK positions each).  Item i goes to buffer
    // i % NB; items i + 1 .. i + NB - 1 are in flight while item i is used.
    // Every thread copies 16-byte pieces of the rows (cp.async, one commit
    // group per item, empty for items whose rows all come from registers);
    // waiting for item i = waiting until no more than the groups committed
    // after it are pending, then a barrier.
    const uint32_t cached = prep ? T : pos;  // rows copied from the caches: [0, cached)
    const uint32_t nc = (T + CHK - 1) / CHK, nitems = 2 * nc;
    constexpr uint32_t SEGS = 2 * HD / 16;   // 16-byte pieces per row
    uint32_t committed = 0;
    auto issue = [&](uint32_t it) {
        if (it >= nitems) return;
        const uint32_t c0 = (it < nc ? it : it - nc) * CHK;
        const uint32_t cend = c0 + CHK < cached ? c0 + CHK : cached;
        const uint16_t *src = it < nc ? kg : vg;
        uint8_t *dst = bufs + (it % NB) * CHK * RS;
        const uint32_t n = cend > c0 ? (cend - c0) * SEGS : 0u;
        for (uint32_t u = tid; u < n; u += blockDim.x) {
            const uint32_t row = u / SEGS, sg = u - row * SEGS;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + row * RS + 16 * sg)),
                         "l"(src + (uint64_t)(c0 + row) * kv_dim + 8 * sg)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        committed++;
    };
    auto wait_item = [&](uint32_t it) {
        const uint32_t after = committed - (it + 1);  // groups committed after item it's
        if (after == 0)
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        else if (after == 1)
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        else if (after == 2)
            asm volatile("cp.async.wait_group 2;" ::: "memory");
        else
            asm volatile("cp.async.wait_group 3;" ::: "memory");
    };
    if (!prep)  // earlier steps wrote these rows: copy them before waiting
        for (uint32_t it = 0; it < NB; it++) issue(it);

    grid_dependency_wait();
    // one token: the next kernel (a GEMV) may launch now and prefetch its
    // weights; the batch form runs many waves of CTAs, whose slots the next
    // kernel's waiting CTAs would take, so it lets it launch at its end
    if (!prep) grid_launch_dependents();
    if (prep) {  // the kernel before this one wrote the batch's rows
        for (uint32_t it = 0; it < NB; it++) issue(it);
        for (uint32_t d = tid; d < HD; d += blockDim.x) qs[d] = a.q[(uint64_t)blockIdx.y * a.q_stride + h * HD + d];
    }
    if (!prep) {

    // ---- this position: head norms, RoPE, f16 K and V ----
    for (uint32_t d = tid; d < 2 * HD; d += blockDim.x) hs[d] = d < HD ? a.q[h * HD + d] : a.k[kvh * HD + d - HD];
    for (uint32_t d = tid; d < HD; d += blockDim.x) vcur[d] = __half_as_ushort(__float2half_rn(a.v[kvh * HD + d]));
    __syncthreads();
    if ((tid == 0 && a.qn_w) || (tid == 32 && a.kn_w)) {
        // rmsnorm_heads: the head's sum of squares in element order, one thread each for q and k
        const float ss = seq_sum_squares(hs + (tid ? HD : 0), HD);
        lsh[tid ? 2 : 1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), a.eps)));
    }
    __syncthreads();
    const float fpos = (float)pos;
    for (uint32_t j = tid; j < HD; j += blockDim.x) {  // j < HALF: q pair j; else k pair j - HALF
        const bool is_k = j >= HALF;
        const uint32_t i = is_k ? j - HALF : j;
        const uint32_t ia = a.neox ? i : 2 * i, ib = a.neox ? i + HALF : 2 * i + 1;
        const float *src = hs + (is_k ? HD : 0);
        float x0 = src[ia], x1 = src[ib];
        const float *nw = is_k ? a.kn_w : a.qn_w;
        if (nw) {
            const float inv = lsh[is_k ? 2 : 1];
            x0 = __fmul_rn(__fmul_rn(x0, inv), nw[ia]);
            x1 = __fmul_rn(__fmul_rn(x1, inv), nw[ib]);
        }
        const float ang = __fmul_rn(fpos, a.inv_freq[i]);
        const float s = gm_sinf(ang), c = gm_cosf(ang);
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        if (!is_k) {
            qs[ia] = y0;
            qs[ib] = y1;
        } else {
            kcur[ia] = __half_as_ushort(__float2half_rn(y0));
            kcur[ib] = __half_as_ushort(__float2half_rn(y1));
        }
    }
    __syncthreads();
    if (h % (a.n_heads / a.n_kv) == 0) {  // the group's first head stores this position's rows
        for (uint32_t d = tid; d < HD; d += blockDim.x) {
            a.kc[(uint64_t)pos * kv_dim + kvh * HD + d] = kcur[d];
            a.vc[(uint64_t)pos * kv_dim + kvh * HD + d] = vcur[d];
        }
    }
    }  // !prep
    __syncthreads();

    // ---- scores, chunk by chunk: 8 lanes per position (the 8 AVX lanes) ----
    const uint32_t grp = lane >> 3, l8 = lane & 7u;
    for (uint32_t c = 0; c < nc; c++) {
        const uint32_t c0 = c * CHK, cn = T - c0 < CHK ? T - c0 : CHK;
        uint8_t *buf = bufs + (c % NB) * CHK * RS;
        if (c > 0) {
            __syncthreads();  // item c - 1 is read: its buffer takes item c + NB - 1
            issue(c + NB - 1);
        }
        wait_item(c);
        if (!prep && pos < c0 + cn) {
            for (uint32_t d = tid; d < HD; d += blockDim.x)
                reinterpret_cast<uint16_t *>(buf + (pos - c0) * RS)[d] = kcur[d];
        }
        __syncthreads();
        for (uint32_t t0 = warp * 4; t0 < cn; t0 += nwarps * 4) {
            const uint32_t t = t0 + grp;
            float acc = 0.0f;
            if (t < cn) {
                const uint16_t *kr = reinterpret_cast<const uint16_t *>(buf + t * RS);
#pragma unroll
                for (uint32_t i = 0; i < HD / 8; i++)
                    acc = __fmaf_rn(__half2float(__ushort_as_half(kr[8 * i + l8])), qs[8 * i + l8], acc);
            }
            // hsum_avx2: ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)), + the empty tail (0.0)
            const float x4 = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
            const float x1 = __fadd_rn(x4, __shfl_down_sync(0xffffffffu, x4, 1));
            const float x2 = __fadd_rn(x1, __shfl_down_sync(0xffffffffu, x1, 2));
            if (t < cn && l8 == 0) sc[c0 + t] = __fmul_rn(__fadd_rn(x2, 0.0f), a.scale);
        }
    }
    __syncthreads();
    // ---- running maxima (f32::max ignores NaN: any grouping gives the same),
    // over all warps: warp w takes positions [w*seg, (w+1)*seg); its carry-in
    // is the maximum of the segments before it ----
    {
        float *segmax = hs;  // free after RoPE
        const uint32_t seg = ((T + nwarps - 1) / nwarps + 31) & ~31u;
        const uint32_t s0 = warp * seg, s1 = s0 + seg < T ? s0 + seg : T;
        float mw = -INFINITY;
        for (uint32_t t = s0 + lane; t < s1; t += 32) {
            const float v = sc[t];
            if (!isnan(v)) mw = fmaxf(mw, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, o));
        if (lane == 0) segmax[warp] = mw;
        __syncthreads();
        float carry = -INFINITY;
        for (uint32_t w = 0; w < warp; w++) carry = fmaxf(carry, segmax[w]);
        for (uint32_t t0 = s0; t0 < s1; t0 += 32) {
            const uint32_t t = t0 + lane;
            float m = t < s1 ? sc[t] : -INFINITY;
            if (isnan(m)) m = -INFINITY;  // f32::max(prev, NaN) = prev
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float u = __shfl_up_sync(0xffffffffu, m, o);
                if (lane >= (uint32_t)o) m = fmaxf(m, u);
            }
            m = fmaxf(m, carry);
            const float prev = __shfl_up_sync(0xffffffffu, m, 1);
            const float mprev = lane == 0 ? carry : prev;
            if (t < s1) {
                // alpha_t = exp(m_{t-1} - m_t), p_t = exp(s_t - m_t)
                al[t] = expf_ref(__fsub_rn(mprev, m));
                sc[t] = expf_ref(__fsub_rn(sc[t], m));
            }
            carry = __shfl_sync(0xffffffffu, m, 31);
        }
    }
    // ---- the two recurrences, chunk by chunk over V ----
    float acc = 0.0f, l = 0.0f;
    for (uint32_t c = 0; c < nc; c++) {
        const uint32_t it = nc + c, c0 = c * CHK, cn = T - c0 < CHK ? T - c0 : CHK;
        uint8_t *buf = bufs + (it % NB) * CHK * RS;
        __syncthreads();  // maxima done; item it - 1 is read: its buffer takes item it + NB - 1
        issue(it + NB - 1);
        wait_item(it);
        if (!prep && pos < c0 + cn) {
            for (uint32_t d = tid; d < HD; d += blockDim.x)
                reinterpret_cast<uint16_t *>(buf + (pos - c0) * RS)[d] = vcur[d];
        }
        __syncthreads();
        if (tid < HD) {
            const uint16_t *vr = reinterpret_cast<const uint16_t *>(buf) + tid;
#pragma unroll 8
            for (uint32_t t = 0; t < cn; t++)
                acc = __fmaf_rn(sc[c0 + t], __half2float(__ushort_as_half(vr[t * (RS / 2)])), __fmul_rn(acc, al[c0 + t]));
        } else if (tid == HD) {
            for (uint32_t t = 0; t < cn; t++) l = __fadd_rn(__fmul_rn(l, al[c0 + t]), sc[c0 + t]);
        }
    }
    if (tid == HD) lsh[0] = __fdiv_rn(1.0f, l > 1e-9f ? l : 1e-9f);  // 1 / l.max(1e-9): a NaN l gives 1e-9
    if (prep) grid_launch_dependents();
    __syncthreads();
    if (tid < HD)
        a.out[(uint64_t)blockIdx.y * a.n_heads * HD + h * HD + tid] = __fmul_rn(acc, lsh[0]);
}

template __global__ void attention_kernel<64, 64>(const __grid_constant__ AttnArgs);
template __global__ void attention_kernel<128, 64>(const __grid_constant__ AttnArgs);
template __global__ void attention_kernel<256, 64>(const __grid_constant__ AttnArgs);
template __global__ void attention_kernel<64, 128>(const __grid_constant__ AttnArgs);
template __global__ void attention_kernel<128, 128>(const __grid_constant__ AttnArgs);
template __global__ void attention_kernel<256, 128>(const __grid_constant__ AttnArgs);

// compute_head_fn (smollm_chat.rs:3463-3495) for a batch of positions in the
// prepared form (q normed and rotated, the batch's K/V rows in the caches),
// with the rows shared: CTA (g, b) takes KV head g's group of H = n_heads /
// n_kv query heads for the TB = ATTN_PAIRS / H tokens b * TB .. of the batch,
// pair p = (head g * H + p / TB, token b * TB + p % TB), and walks the
// positions in chunks of CH = ATTN_BCH whose K and V rows are copied into
// shared memory once for all pairs (the next chunk in flight meanwhile).  Per
// chunk, every pair's result is attention_kernel's, operation for operation:
//   scores: thread (pair, 2 positions): the 8 AVX lanes of dot_f16_row
//     (lane l: fma over dims l, l + 8, ... in order), the lane tree
//     ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)), + 0.0, * scale;
//   running maxima (f32::max, NaN ignored) by a warp scan per pair, carried
//     across chunks; alpha_t = exp(m_{t-1} - m_t), p_t = exp(s_t - m_t);
//   l_t = l_{t-1} * alpha_t + p_t (one thread per pair) and
//     acc_t[d] = fma(p_t, v_t[d], acc_{t-1}[d] * alpha_t) (thread: 4 pairs x
//     2 dims), position by position;
// then out = acc * (1 / max(l, 1e-9)).  A pair stops at its token's position.
template <int HD>
__global__ void __launch_bounds__(2 * HD, HD < 256 ? 2 : 1) attention_batch_kernel(const __grid_constant__ AttnArgs a) {
    constexpr uint32_t P = ATTN_PAIRS, CH = ATTN_BCH, ND = HD / 2, QS = HD + 4, SEG = HD * 2 / 16;
    static_assert(P * CH / 2 == 2 * HD || HD != 128, "one score task per thread at head_dim 128");
    extern __shared__ __align__(16) uint8_t sm8[];
    float *qf = reinterpret_cast<float *>(sm8);                      // [P][QS]
    uint16_t *kh = reinterpret_cast<uint16_t *>(qf + P * QS);        // [2][CH][HD]
    uint16_t *vh = kh + 2 * CH * HD;                                 // [2][CH][HD]
    float *kf = reinterpret_cast<float *>(vh + 2 * CH * HD);         // [CH][HD]
    float *vf = kf + CH * HD;                                        // [CH][HD]
    float *sc = vf + CH * HD;                                        // [P][CH]
    float2 *pa = reinterpret_cast<float2 *>(sc + P * CH);            // [P][CH]: (p_t, alpha_t)
    float *lsum = reinterpret_cast<float *>(pa + P * CH), *mrun = lsum + P;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const uint32_t H = a.n_kv ? a.n_heads / a.n_kv : 0u, TB = H ? P / H : 0u, g = blockIdx.x;
    if (a.head_dim != HD || blockDim.x != 2 * HD || H == 0 || a.n_heads % a.n_kv || P % H ||
        gridDim.x != a.n_kv || gridDim.y * TB < a.ntok || attn_batch_smem(HD) > dynamic_smem_size()) {
        grid_dependency_wait();
        if (tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    grid_dependency_wait();  // q and the batch's K/V rows come from the kernel before
    const uint32_t pos0 = (uint32_t)a.state[0], t0 = blockIdx.y * TB;
    const uint32_t tend = t0 + TB < a.ntok ? t0 + TB : a.ntok;
    const uint32_t T = pos0 + tend;  // positions [0, T): the block's last token is at T - 1
    if (t0 >= a.ntok || T > a.max_seq) {
        if (t0 < a.ntok && tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        grid_launch_dependents();
        return;
    }
    for (uint32_t i = tid; i < P * HD; i += blockDim.x) {
        const uint32_t p = i / HD, d = i - p * HD, t = t0 + p % TB;
        qf[p * QS + d] = t < tend ? a.q[(uint64_t)t * a.q_stride + (g * H + p / TB) * HD + d] : 0.0f;
    }
    for (uint32_t p = tid; p < P; p += blockDim.x) {
        lsum[p] = 0.0f;
        mrun[p] = -INFINITY;
    }
    const uint32_t kv_dim = a.n_kv * HD, nc = (T + CH - 1) / CH;
    const uint16_t *kg = a.kc + g * HD, *vg = a.vc + g * HD;
    auto issue = [&](uint32_t c) {  // chunk c's K and V rows into buffer c & 1 (one commit group, maybe empty)
        if (c < nc) {
            const uint32_t c0 = c * CH, n = T - c0 < CH ? T - c0 : CH, b = c & 1u;
            for (uint32_t u = tid; u < 2 * n * SEG; u += blockDim.x) {
                const uint32_t w = u / (n * SEG), rs = u - w * n * SEG, r = rs / SEG, sg = rs - r * SEG;
                const uint16_t *src = (w ? vg : kg) + (uint64_t)(c0 + r) * kv_dim + 8 * sg;
                uint16_t *dst = (w ? vh : kh) + (b * CH + r) * HD + 8 * sg;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // the positions pair p uses in chunk c0 .. c0 + n - 1: up to its token's position
    auto valid = [&](uint32_t p, uint32_t c0, uint32_t n) -> uint32_t {
        const uint32_t t = t0 + p % TB;
        if (t >= tend || pos0 + t < c0) return 0u;
        const uint32_t v = pos0 + t - c0 + 1;
        return v < n ? v : n;
    };
    const uint32_t d2 = tid % ND, pq = tid / ND;  // recurrence: dims 2 d2, 2 d2 + 1, pairs 4 pq ..
    float acc[4][2];
#pragma unroll
    for (int k = 0; k < 4; k++) acc[k][0] = acc[k][1] = 0.0f;
    issue(0);
    for (uint32_t c = 0; c < nc; c++) {
        issue(c + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();  // chunk c's rows are in, and everyone is done with chunk c - 1
        const uint32_t c0 = c * CH, n = T - c0 < CH ? T - c0 : CH, b = c & 1u;
        for (uint32_t i = tid; i < n * HD; i += blockDim.x) {
            kf[i] = __half2float(__ushort_as_half(kh[b * CH * HD + i]));
            vf[i] = __half2float(__ushort_as_half(vh[b * CH * HD + i]));
        }
        __syncthreads();
        // scores: thread (pair p, positions 2 pg, 2 pg + 1): pairs fastest, so
        // a warp reads the same K rows (broadcast) and padded q rows
        for (uint32_t task = tid; task < P * (CH / 2); task += blockDim.x) {
            const uint32_t p = task % P, pg = task / P;
            if (2 * pg >= valid(p, c0, n)) continue;
            float al[2][8];
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int l = 0; l < 8; l++) al[j][l] = 0.0f;
            const float *qp = qf + p * QS;
#pragma unroll 4
            for (uint32_t i = 0; i < HD / 8; i++) {
                const float4 q0 = *reinterpret_cast<const float4 *>(qp + 8 * i);
                const float4 q1 = *reinterpret_cast<const float4 *>(qp + 8 * i + 4);
                const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const float *kr = kf + (2 * pg + j) * HD + 8 * i;
                    const float4 k0 = *reinterpret_cast<const float4 *>(kr);
                    const float4 k1 = *reinterpret_cast<const float4 *>(kr + 4);
                    const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
                    for (int l = 0; l < 8; l++) al[j][l] = __fmaf_rn(kv[l], qv[l], al[j][l]);
                }
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float x = __fadd_rn(__fadd_rn(__fadd_rn(al[j][0], al[j][4]), __fadd_rn(al[j][1], al[j][5])),
                                          __fadd_rn(__fadd_rn(al[j][2], al[j][6]), __fadd_rn(al[j][3], al[j][7])));
                sc[p * CH + 2 * pg + j] = __fmul_rn(__fadd_rn(x, 0.0f), a.scale);
            }
        }
        __syncthreads();
        // running maxima, alpha and p: one warp per pair, lane = position
        for (uint32_t p = warp; p < P; p += nwarps) {
            const uint32_t vp = valid(p, c0, n);
            if (vp == 0) continue;
            const float s = lane < vp ? sc[p * CH + lane] : -INFINITY;
            float m = isnan(s) ? -INFINITY : s;  // f32::max(prev, NaN) = prev
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float u = __shfl_up_sync(0xffffffffu, m, o);
                if (lane >= (uint32_t)o) m = fmaxf(m, u);
            }
            const float carry = mrun[p];
            m = fmaxf(m, carry);
            const float prev = __shfl_up_sync(0xffffffffu, m, 1);
            const float mprev = lane == 0 ? carry : prev;
            // alpha = exp(0) = 1 exactly where the maximum did not move (a finite one:
            // an infinite maximum takes the exp, whose NaN the reference carries)
            if (lane < vp)
                pa[p * CH + lane] = make_float2(expf_ref(__fsub_rn(s, m)),
                                                mprev == m && isfinite(m) ? 1.0f : expf_ref(__fsub_rn(mprev, m)));
            const float mlast = __shfl_sync(0xffffffffu, m, 31);
            __syncwarp();
            if (lane == 0) mrun[p] = mlast;  // used only when all CH positions were the pair's
        }
        __syncthreads();
        // the recurrences: l (thread p < P), acc (thread: 4 pairs x 4 dims)
        if (tid < P) {
            const uint32_t vp = valid(tid, c0, n);
            float l = lsum[tid];
            for (uint32_t t = 0; t < vp; t++) {
                const float2 w = pa[tid * CH + t];
                l = __fadd_rn(__fmul_rn(l, w.y), w.x);
            }
            lsum[tid] = l;
        }
        uint32_t vk[4];
#pragma unroll
        for (int k = 0; k < 4; k++) vk[k] = valid(4 * pq + k, c0, n);
        const uint32_t vmax = max(max(vk[0], vk[1]), max(vk[2], vk[3]));
        const uint32_t vmin = min(min(vk[0], vk[1]), min(vk[2], vk[3])) & ~1u;
        const float4 *pa4 = reinterpret_cast<const float4 *>(pa);  // (p, alpha) of positions t, t + 1
        // positions every pair of the thread uses, two at a time, no predicates
        for (uint32_t t = 0; t < vmin; t += 2) {
            const float2 va = *reinterpret_cast<const float2 *>(vf + t * HD + 2 * d2);
            const float2 vb = *reinterpret_cast<const float2 *>(vf + (t + 1) * HD + 2 * d2);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float4 w = pa4[((4 * pq + k) * CH + t) / 2];
                acc[k][0] = __fmaf_rn(w.x, va.x, __fmul_rn(acc[k][0], w.y));
                acc[k][1] = __fmaf_rn(w.x, va.y, __fmul_rn(acc[k][1], w.y));
                acc[k][0] = __fmaf_rn(w.z, vb.x, __fmul_rn(acc[k][0], w.w));
                acc[k][1] = __fmaf_rn(w.z, vb.y, __fmul_rn(acc[k][1], w.w));
            }
        }
        for (uint32_t t = vmin; t < vmax; t++) {
            const float2 va = *reinterpret_cast<const float2 *>(vf + t * HD + 2 * d2);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (t < vk[k]) {
                    const float2 w = pa[(4 * pq + k) * CH + t];
                    acc[k][0] = __fmaf_rn(w.x, va.x, __fmul_rn(acc[k][0], w.y));
                    acc[k][1] = __fmaf_rn(w.x, va.y, __fmul_rn(acc[k][1], w.y));
                }
            }
        }
    }
    __syncthreads();
    grid_launch_dependents();
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t p = 4 * pq + k, t = t0 + p % TB;
        if (t >= tend) continue;
        const float l = lsum[p];
        const float inv = __fdiv_rn(1.0f, l > 1e-9f ? l : 1e-9f);  // 1 / l.max(1e-9): a NaN l gives 1e-9
        float *o = a.out + (uint64_t)t * a.n_heads * HD + (g * H + p / TB) * HD + 2 * d2;
        o[0] = __fmul_rn(acc[k][0], inv);
        o[1] = __fmul_rn(acc[k][1], inv);
    }
}

template __global__ void attention_batch_kernel<64>(const __grid_constant__ AttnArgs);
template __global__ void attention_batch_kernel<128>(const __grid_constant__ AttnArgs);
template __global__ void attention_batch_kernel<256>(const __grid_constant__ AttnArgs);

// ARGMAX_CTAS blocks: (total_cmp key, index) maxima with the larger index on
// ties, then the last block to finish reduces them.
__global__ void __launch_bounds__(ARGMAX_THREADS) argmax_kernel(const __grid_constant__ ArgmaxArgs a) {
    __shared__ unsigned long long red[ARGMAX_THREADS / 32];
    __shared__ bool last;
    grid_dependency_wait();
    grid_launch_dependents();
    auto block_max = [&](unsigned long long best) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long u = __shfl_xor_sync(0xffffffffu, best, o);
            best = u > best ? u : best;
        }
        if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = best;
        __syncthreads();
        best = red[0];
        for (uint32_t w = 1; w < blockDim.x / 32; w++) best = red[w] > best ? red[w] : best;
        return best;
    };
    // batch: token blockIdx.y (its logits, partial maxima and ticket)
    const uint32_t tb = blockIdx.y;
    const float *const lg = a.logits + (uint64_t)tb * a.ldl;
    unsigned long long *const part = a.partial + (uint64_t)tb * gridDim.x;
    unsigned *const cnt = a.count + tb;
    unsigned long long best = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
        const int32_t b = __float_as_int(lg[i]);
        const uint32_t key = (uint32_t)(b ^ (int32_t)((uint32_t)(b >> 31) >> 1)) ^ 0x80000000u;
        const unsigned long long v = ((unsigned long long)key << 32) | i;
        best = v > best ? v : best;
    }
    best = block_max(best);
    if (threadIdx.x == 0) {
        part[blockIdx.x] = best;
        __threadfence();
        last = atomicAdd(cnt, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    best = 0;
    for (uint32_t b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
        const unsigned long long v = __ldcg(part + b);
        best = v > best ? v : best;
    }
    __syncthreads();  // red[] is reused
    best = block_max(best);
    if (threadIdx.x == 0) {
        const int32_t tok = (int32_t)(best & 0xFFFFFFFFull);
        if (a.batch) {
            if (a.out) a.out[tb] = tok;
        } else {
            a.state[0] = tok;
            a.state[1] = a.state[1] + 1;
            if (a.out) *a.out = tok;
        }
        *cnt = 0;
    }
}

// Batch: token blockIdx.y at position *pos + blockIdx.y.  Warp h < n_heads:
// q head h (normed, rotated in place); else kv head h - n_heads: k normed and
// rotated, K and V rows rounded to f16 into the caches.  The arithmetic of the
// one-token attention kernel's first part.
__global__ void rope_kv_batch_kernel(const __grid_constant__ RopeBatchArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t h = blockIdx.x, lane = threadIdx.x, hd = a.head_dim, half = hd / 2, t = blockIdx.y;
    const bool is_q = h < a.n_heads;
    const uint32_t kh = is_q ? 0u : h - a.n_heads;
    const uint32_t pos = (uint32_t)*a.pos + t;
    if (hd > 256 || (hd & 63u) || pos >= a.max_seq || blockDim.x != 32) {
        if (lane == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    float *const q = a.q + (uint64_t)t * a.qkv_stride;
    const float *const k = a.k + (uint64_t)t * a.qkv_stride, *const v = a.v + (uint64_t)t * a.qkv_stride;
    const float *src = is_q ? q + h * hd : k + kh * hd;
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
            const float sn = gm_sinf(ang), cs = gm_cosf(ang);
            const float y0 = __fsub_rn(__fmul_rn(x0[j], cs), __fmul_rn(x1[j], sn));
            const float y1 = __fadd_rn(__fmul_rn(x0[j], sn), __fmul_rn(x1[j], cs));
            if (is_q) {
                q[h * hd + ia] = y0;
                q[h * hd + ib] = y1;
            } else {
                uint16_t *kr = a.kc + (uint64_t)pos * kv_dim + kh * hd;
                kr[ia] = __half_as_ushort(__float2half_rn(y0));
                kr[ib] = __half_as_ushort(__float2half_rn(y1));
            }
        }
    if (!is_q) {
        uint16_t *vr = a.vc + (uint64_t)pos * kv_dim + kh * hd;
        for (uint32_t i = lane; i < hd; i += 32) vr[i] = __half_as_ushort(__float2half_rn(v[kh * hd + i]));
    }
}

// The sender: every CTA first waits (bounded) until the receiver has
// acknowledged epoch e - 2, so that half e & 1 of its buffer is read; then the
// pairs go out.  The last CTA to finish (ticket) advances the epoch.
__global__ void pipe_send_kernel(const __grid_constant__ PipeArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const unsigned e = *a.epoch + 1u;
    __shared__ bool ok;
    if (threadIdx.x == 0) {
        ok = true;
        if (e > 2) {
            const uint64_t t0 = globaltimer_ns();
            for (;;) {
                unsigned v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.ack) : "memory");
                if (v + 2u >= e) break;
                if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
                    atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_PEER);
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
        }
    }
    __syncthreads();
    unsigned long long *half = a.recv + (uint64_t)(e & 1u) * a.half;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (uint64_t)gridDim.x * blockDim.x) {
        const unsigned long long pr = ((unsigned long long)e << 32) | __float_as_uint(ok ? a.src[i] : __int_as_float(0x7fc00000));
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(half + i), "l"(pr) : "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.ticket, 1u) == gridDim.x - 1) {
        *a.ticket = 0;
        *a.epoch = e;
    }
}

// The receiver: each value as soon as its pair carries epoch e; the last CTA
// to finish acknowledges e to the sender (release) and advances the epoch.
__global__ void pipe_recv_kernel(const __grid_constant__ PipeArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const unsigned e = *a.epoch + 1u;
    const unsigned long long *half = a.recv + (uint64_t)(e & 1u) * a.half;
    uint64_t t0 = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (uint64_t)gridDim.x * blockDim.x) {
        unsigned long long p;
        for (;;) {
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(p) : "l"(half + i) : "memory");
            if ((uint32_t)(p >> 32) == e) break;
            const uint64_t t = globaltimer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > WAIT_LIMIT_NS) {
                atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_PEER);
                p = 0x7fc00000ull;
                break;
            }
            __nanosleep(32);
        }
        a.dst[i] = __uint_as_float((uint32_t)p);
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.ticket, 1u) == gridDim.x - 1) {
        *a.ticket = 0;
        *a.epoch = e;
        // every block has read its values from half e & 1: the sender may reuse it
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.ack), "r"(e) : "memory");
    }
}

__global__ void residual_kernel(const float *x, const float *add, float rs, float *out, uint64_t n) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fadd_rn(x[i], __fmul_rn(rs, add[i]));
}

// One thread per (layer, row, pair of a head): K re-rotated, V copied.
__global__ void kv_shift_kernel(const __grid_constant__ KvShiftArgs a) {
    const uint32_t half = a.head_dim / 2, pairs = a.kv_dim / 2;
    const uint64_t rows = (uint64_t)(a.l1 - a.l0) * (a.i1 - a.i0);
    const float pos = -(float)a.n_discard;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < rows * pairs;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = t / pairs;
        const uint32_t p = (uint32_t)(t - row * pairs);
        const uint32_t l = a.l0 + (uint32_t)(row / (a.i1 - a.i0)), i = a.i0 + (uint32_t)(row % (a.i1 - a.i0));
        const uint64_t src = ((uint64_t)l * a.max_seq + a.n_keep + a.n_discard + i) * a.kv_dim;
        const uint64_t dst = ((uint64_t)l * a.max_seq + a.n_keep + i) * a.kv_dim;
        const uint32_t h = p / half, j = p - h * half;
        const uint32_t ia = h * a.head_dim + (a.neox ? j : 2 * j), ib = h * a.head_dim + (a.neox ? j + half : 2 * j + 1);
        const float x0 = __half2float(__ushort_as_half(a.kc[src + ia]));
        const float x1 = __half2float(__ushort_as_half(a.kc[src + ib]));
        const float ang = __fmul_rn(pos, a.inv_freq[j]);
        const float sn = gm_sinf(ang), cs = gm_cosf(ang);
        a.kc[dst + ia] = __half_as_ushort(__float2half_rn(__fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn))));
        a.kc[dst + ib] = __half_as_ushort(__float2half_rn(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs))));
        a.vc[dst + ia] = a.vc[src + ia];
        a.vc[dst + ib] = a.vc[src + ib];
    }
}

}  // namespace sg
