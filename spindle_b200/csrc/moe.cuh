// moe.cuh — the top-k MoE layer of spindle (moe_forward, smollm_chat.rs:1178-1382,
// with the fused expert FFNs of ffns_fused, :382-442) as a chain of kernels
// on one stream, the expert choice staying on the device:
//   1. moe_router_kernel: one cluster of ROUTER_CLUSTER CTAs.  Each CTA computes
//      the logits of its share of the router rows (F32 GEMV with the lane order
//      of dot_f32_2rows_avx2, quant.rs:1461-1483), the cluster syncs, and CTA 0
//      gathers all logits through distributed shared memory and runs softmax,
//      top-k, prune and the mixing weights (smollm_chat.rs:1199-1240).
//   2. gemv_tiled_kernel<., 1, IN_MOE_X>: gate and up of every chosen expert.
//   3. gemv_tiled_kernel<., 1, IN_MOE_H>: down of every chosen expert.
//   (2 and 3 again for the shared expert, with a one-slot choice.)
//   4. moe_combine_kernel: out[r] = sum over the choice, in router order, of
//      w_i * y_i[r] (smollm_chat.rs:431-438), plus g * shared[r] (:1370-1382).
#pragma once

#include "gemv_tiled.cuh"

namespace sg {

constexpr uint32_t ROUTER_CLUSTER = 8;   // CTAs of the router (one cluster)
constexpr uint32_t ROUTER_THREADS = 128; // 16 rows at a time, 8 threads (AVX lanes) per row
constexpr uint32_t ROUTER_MAX_EXPERTS = 4096;
constexpr uint32_t ROUTER_ROW_PAD = 32;  // bytes between staged rows (spreads rows over banks)

struct RouterArgs {
    const float *w;        // F32 [n_expert][dim]
    const float *x;        // [dim]
    uint32_t dim, n_expert, n_used;
    uint32_t rows_per_cta; // ceil(n_expert / ROUTER_CLUSTER)
    uint32_t rc;           // rows per ring stage (<= 16)
    int32_t norm;
    float prune;
    float *probs;          // optional: softmax probabilities [n_expert]
    sg_moe_choice *sel;
    sg_moe_choice *shared_sel;  // optional: written as {1, id 0, weight 1}
    const float *shared_gate;   // optional F32 [dim]
    float *shared_scale;        // sigmoid(shared_gate . x), or 1 without a gate
};

// bars (64) | x (dim floats) | shared gate (dim floats) | ring: 2 stages of rc rows | logits
__host__ __device__ inline uint32_t router_row_stride(uint32_t dim) { return dim * 4u + ROUTER_ROW_PAD; }
__host__ __device__ inline uint32_t router_ring_bytes(uint32_t dim, uint32_t rc, uint32_t n_expert) {
    const uint32_t ring = 2u * rc * router_row_stride(dim);
    // CTA 0 reuses the ring for the softmax (probabilities and sort keys)
    const uint32_t sel_area = n_expert * 8u + 256u;
    return ring > sel_area ? ring : sel_area;
}
__host__ __device__ inline uint32_t router_smem_bytes(uint32_t dim, uint32_t rc, uint32_t rows_per_cta,
                                                      uint32_t n_expert) {
    return 64u + 2u * dim * 4u + router_ring_bytes(dim, rc, n_expert) + ((rows_per_cta * 4u + 15u) & ~15u);
}

struct CombineArgs {
    const sg_moe_choice *sel;
    const float *y;        // slot s at y + s * dim
    const float *ysh;      // shared expert output or null
    const float *shared_scale;
    float *out;
    uint32_t dim;
    uint32_t max_slots;    // slots y holds (n_used)
};

__global__ void moe_router_kernel(const __grid_constant__ RouterArgs a);
__global__ void moe_combine_kernel(const __grid_constant__ CombineArgs a);

}  // namespace sg
