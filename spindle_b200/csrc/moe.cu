// moe.cu — router and combine kernels of the MoE layer (see moe.cuh).
#include <cooperative_groups.h>

#include "moe.cuh"
#include "tiled_block.cuh"

namespace cg = cooperative_groups;

namespace sg {
using namespace tiled;

namespace {

// Rust's f32::max: the other operand when one is NaN.
__device__ __forceinline__ float rmax(float a, float b) { return isnan(a) ? b : isnan(b) ? a : (a > b ? a : b); }

// f32::total_cmp's order as a signed integer key.
__device__ __forceinline__ int32_t total_key(float f) {
    const int32_t i = __float_as_int(f);
    return i ^ (int32_t)((uint32_t)(i >> 31) >> 1);
}

__device__ __forceinline__ float block_rmax(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = rmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
    for (uint32_t w = 1; w < blockDim.x / 32; w++) m = rmax(m, red[w]);
    return m;
}

}  // namespace

// Softmax, top-k, prune and weights of smollm_chat.rs:1199-1240 over the
// logits P[0..ne) in shared memory, by one CTA.  K: ne sort keys; sc: scratch.
static __device__ __forceinline__ void router_select(const RouterArgs &a, float *P, int32_t *K, uint32_t *sc) {
    const uint32_t ne = a.n_expert, k = a.n_used, tid = threadIdx.x, nt = blockDim.x;
    float *red = reinterpret_cast<float *>(sc);        // [0..4): block reduction
    int32_t *top = reinterpret_cast<int32_t *>(sc + 8); // [8..24): top-k in order
    float *sum_s = reinterpret_cast<float *>(sc + 24);
    // max folded with f32::max (NaN ignored): any order gives the same value
    float m = -INFINITY;
    for (uint32_t e = tid; e < ne; e += nt) m = rmax(m, P[e]);
    const float mx = block_rmax(m, red);
    for (uint32_t e = tid; e < ne; e += nt) P[e] = expf_cr(__fsub_rn(P[e], mx));
    __syncthreads();
    if (tid == 0) {
        float s = 0.0f;  // sequential, as Iterator::sum
        for (uint32_t e = 0; e < ne; e++) s = __fadd_rn(s, P[e]);
        *sum_s = s;
    }
    __syncthreads();
    const float sum = *sum_s;
    for (uint32_t e = tid; e < ne; e += nt) {
        P[e] = __fdiv_rn(P[e], sum);
        K[e] = total_key(P[e]);
        if (a.probs) a.probs[e] = P[e];
    }
    __syncthreads();
    // rank of e = experts before it in (probability descending, index
    // ascending) order; the first k ranks are the top-k in order
    for (uint32_t e = tid; e < ne; e += nt) {
        const int32_t key = K[e];
        uint32_t cnt = 0;
        for (uint32_t j = 0; j < ne && cnt < k; j++) {
            const int32_t kj = K[j];
            cnt += (kj > key) | ((kj == key) & (j < e));
        }
        if (cnt < k) top[cnt] = (int32_t)e;
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t keep = k;
        if (a.prune > 0.0f && k > 2) {
            const uint32_t min_keep = k / 2 > 2 ? k / 2 : 2;
            if (a.prune >= 1.0f) {
                // `prune as usize` (saturating), clamped to [min_keep, k]
                const uint32_t p = a.prune >= 4294967040.0f ? 0xFFFFFFFFu : (uint32_t)a.prune;
                keep = p < min_keep ? min_keep : (p > k ? k : p);
            } else {
                float top_sum = 0.0f;
                for (uint32_t i = 0; i < k; i++) top_sum = __fadd_rn(top_sum, P[top[i]]);
                const float target = __fmul_rn(top_sum, __fsub_rn(1.0f, a.prune));
                float cum = 0.0f;
                uint32_t i = 0;
                while (i < k && (i < min_keep || cum < target)) {
                    cum = __fadd_rn(cum, P[top[i]]);
                    i++;
                }
                keep = i;
            }
        }
        float wsum = 0.0f;
        for (uint32_t i = 0; i < keep; i++) wsum = __fadd_rn(wsum, P[top[i]]);
        sg_moe_choice *s = a.sel;
        for (uint32_t i = 0; i < MOE_MAXK; i++) {
            const bool on = i < keep;
            s->id[i] = on ? top[i] : 0;
            s->weight[i] = on ? (a.norm ? __fdiv_rn(P[top[i]], wsum) : P[top[i]]) : 0.0f;
        }
        s->pad_[0] = s->pad_[1] = s->pad_[2] = 0;
        s->n = keep;
        if (a.shared_sel) {
            sg_moe_choice *t = a.shared_sel;
            for (uint32_t i = 0; i < MOE_MAXK; i++) {
                t->id[i] = 0;
                t->weight[i] = i == 0 ? 1.0f : 0.0f;
            }
            t->pad_[0] = t->pad_[1] = t->pad_[2] = 0;
            t->n = 1;
        }
    }
}

__global__ void __launch_bounds__(ROUTER_THREADS) moe_router_kernel(const __grid_constant__ RouterArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank(), tid = threadIdx.x;
    const uint32_t dim = a.dim, ne = a.n_expert;
    // Uniform over the cluster (same arguments everywhere): a bad launch
    // returns from every CTA before any cluster barrier.
    if (router_smem_bytes(dim, a.rc, a.rows_per_cta, ne) > dynamic_smem_size() || a.rc == 0 || a.rc > 16 ||
        blockDim.x != ROUTER_THREADS || cluster.num_blocks() != ROUTER_CLUSTER || gridDim.x != ROUTER_CLUSTER ||
        ne == 0 || ne > ROUTER_MAX_EXPERTS || a.n_used == 0 || a.n_used > MOE_MAXK || a.n_used > ne || dim % 8 ||
        a.rows_per_cta * ROUTER_CLUSTER < ne) {
        if (tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    grid_launch_dependents();
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);  // [0], [1]: ring stages; [2]: x; [3]: shared gate
    float *xs = reinterpret_cast<float *>(smem + 64);
    float *gs = xs + dim;
    uint8_t *ring = smem + 64 + 2u * dim * 4u;
    const uint32_t rstride = router_row_stride(dim), rowb = dim * 4u;
    float *logit = reinterpret_cast<float *>(ring + router_ring_bytes(dim, a.rc, ne));
    const bool gate_cta = rank == ROUTER_CLUSTER - 1 && a.shared_scale && a.shared_gate;
    const uint32_t e0 = rank * a.rows_per_cta;
    const uint32_t nrows = e0 < ne ? min(a.rows_per_cta, ne - e0) : 0u;
    const uint32_t nchunks = (nrows + a.rc - 1) / a.rc;

    auto issue = [&](uint32_t c) {
        const uint32_t r0 = c * a.rc, n = min(a.rc, nrows - r0);
        uint64_t *bar = &bars[c & 1u];
        mbar_arrive_expect_tx(bar, n * rowb);
        for (uint32_t q = 0; q < n; q++)
            bulk_g2s(ring + (c & 1u) * a.rc * rstride + q * rstride, a.w + (uint64_t)(e0 + r0 + q) * dim, rowb, bar);
    };
    // router weights first; x once the kernel that wrote it is done
    if (tid == 0) {
        for (int b = 0; b < 4; b++) mbar_init(&bars[b], 1);
        fence_mbar_init();
        for (uint32_t c = 0; c < nchunks && c < 2; c++) issue(c);
        if (gate_cta) {
            mbar_arrive_expect_tx(&bars[3], rowb);
            bulk_g2s(gs, a.shared_gate, rowb, &bars[3]);
        }
    }
    grid_dependency_wait();
    if (tid == 0) {
        mbar_arrive_expect_tx(&bars[2], rowb);
        bulk_g2s(xs, a.x, rowb, &bars[2]);
    }
    __syncthreads();
    bool ok = mbar_wait_bounded(&bars[2], 0, WAIT_LIMIT_NS);
    const uint32_t q = tid >> 3, j = tid & 7u;
    for (uint32_t c = 0; c < nchunks; c++) {
        if (ok) ok = mbar_wait_bounded(&bars[c & 1u], (c >> 1) & 1u, WAIT_LIMIT_NS);
        const uint32_t n = min(a.rc, nrows - c * a.rc);
        // lane j of row q: the FMA chain of AVX lane j (elements j, j+8, ...)
        float acc = 0.0f;
        if (q < n && ok) {
            const float *row = reinterpret_cast<const float *>(ring + (c & 1u) * a.rc * rstride + q * rstride);
#pragma unroll 8
            for (uint32_t i = j; i < dim; i += 8) acc = __fmaf_rn(row[i], xs[i], acc);
        }
        // hsum_avx2: ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)), then + the empty tail (0.0)
        const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
        const float u = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 1));
        const float v = __fadd_rn(u, __shfl_down_sync(0xffffffffu, u, 2));
        if (q < n && j == 0) logit[c * a.rc + q] = __fadd_rn(v, 0.0f);
        __syncthreads();
        if (tid == 0 && ok && c + 2 < nchunks) {
            fence_proxy_async();
            issue(c + 2);
        }
    }
    if (!ok && (tid & 31u) == 0) atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
    const bool cta_ok = __syncthreads_and(ok);

    cluster.sync();  // every CTA's logits are in its shared memory
    float *P = reinterpret_cast<float *>(ring);
    int32_t *K = reinterpret_cast<int32_t *>(ring + ne * 4u);
    uint32_t *sc = reinterpret_cast<uint32_t *>(ring + ne * 8u);
    if (rank == 0 && cta_ok) {
        for (uint32_t e = tid; e < ne; e += blockDim.x) {
            const uint32_t src = e / a.rows_per_cta;
            P[e] = cluster.map_shared_rank(logit, src)[e - src * a.rows_per_cta];
        }
    }
    cluster.sync();  // the other CTAs may exit now
    if (rank == 0) {
        if (cta_ok) {
            __syncthreads();
            router_select(a, P, K, sc);
        } else if (tid == 0) {
            a.sel->n = 0;  // the error is in g_dev_status; run no expert
        }
    }
    // The shared expert's gate: sigmoid(sum over c of w[c] * x[c]), summed in
    // order as the reference's iterator does (smollm_chat.rs:1374-1377).
    if (rank == ROUTER_CLUSTER - 1 && tid == 0 && a.shared_scale) {
        float gsc = 1.0f;
        if (gate_cta) {
            const bool got = mbar_wait_bounded(&bars[3], 0, WAIT_LIMIT_NS);
            if (cta_ok && got) {
                float z = 0.0f;
#pragma unroll 8
                for (uint32_t c = 0; c < dim; c++) z = __fadd_rn(z, __fmul_rn(gs[c], xs[c]));
                gsc = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-z)));
            } else {
                atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                gsc = __int_as_float(0x7fc00000);
            }
        }
        *a.shared_scale = gsc;
    }
}

__global__ void moe_combine_kernel(const __grid_constant__ CombineArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float w[MOE_MAXK];
    __shared__ uint32_t n_s;
    if (threadIdx.x < MOE_MAXK) w[threadIdx.x] = a.sel->weight[threadIdx.x];
    if (threadIdx.x == 0) n_s = min(a.sel->n, a.max_slots);
    __syncthreads();
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.dim) return;
    const uint32_t n = n_s;
    // ffns_fused on a zeroed output: acc = 0 + w_0*y_0 + w_1*y_1 + ...
    float acc = 0.0f;
    for (uint32_t i = 0; i < n; i++) acc = __fadd_rn(acc, __fmul_rn(w[i], a.y[(uint64_t)i * a.dim + r]));
    if (a.ysh) {
        // shared expert: ffns_fused with weight 1 on a zeroed buffer, then out += g * tmp
        const float tmp = __fadd_rn(0.0f, __fmul_rn(1.0f, a.ysh[r]));
        acc = __fadd_rn(acc, __fmul_rn(*a.shared_scale, tmp));
    }
    a.out[r] = acc;
}

}  // namespace sg
