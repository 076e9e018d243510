// moe.cuh — the top-k MoE layer of spindle (moe_forward, smollm_chat.rs:1178-1382,
// with the fused expert FFNs of ffns_fused, :382-442) as a chain of kernels
// on one stream, the expert choice staying on the device:
//   1. moe_router_kernel: the router logits (F32 GEMV with the lane order of
//      dot_f32_2rows_avx2, quant.rs:1461-1483), a few rows per CTA over the
//      whole GPU; one more CTA computes the shared expert's gate.
//   2. gemv_tiled_kernel<., 1, IN_MOE_X>: every CTA makes the choice from the
//      logits (softmax, top-k, prune, weights: smollm_chat.rs:1199-1240), CTA 0
//      publishes it, and the gate and up rows of the chosen experts run.
//   3. gemv_tiled_kernel<., 1, IN_MOE_H>: down rows of the chosen experts.
//   (2 and 3 again for the shared expert, with a one-slot choice.)
//   4. moe_combine_kernel: out[r] = sum over the choice, in router order, of
//      w_i * y_i[r] (smollm_chat.rs:431-438), plus g * shared[r] (:1370-1382).
#pragma once

#include "gemv_tiled.cuh"
#include "moe_select.cuh"

namespace sg {

constexpr uint32_t ROUTER_MAX_EXPERTS = 4096;
constexpr uint32_t ROUTER_ROW_PAD = 32;  // bytes between staged rows (spreads rows over banks)
constexpr uint32_t ROUTER_MAX_ROWS = 16; // rows per CTA (8 threads each)
constexpr uint32_t ROUTER_MAX_THREADS = 256;

struct RouterArgs {
    const float *w;             // F32 [n_expert][dim]
    const float *x;             // token t at x + t * ldx, [dim]
    uint32_t dim, n_expert;
    uint32_t rows_per_cta;      // CTA b < row_ctas computes rows [b * rows_per_cta, ...)
    uint32_t row_ctas;
    float *logits;              // token t at logits + t * n_expert
    uint8_t *qx;                // optional: Q8_K images of the tokens, act_bytes(dim / 256) apart
    // shared expert (CTA row_ctas, when shared_scale is set)
    sg_moe_choice *shared_sel;  // written as {1, id 0, weight 1}
    const float *shared_gate;   // F32 [dim] or null
    float *shared_scale;        // per token: sigmoid(shared_gate . x), or 1 without a gate
    uint32_t n_tok;             // tokens (1 for moe_forward)
    uint64_t ldx;
    uint32_t tok_chunk;         // tokens staged in shared memory at a time
    unsigned *zero_word;        // optional: set to 0 (the batch select kernel's ticket)
};

// Batched MoE (moe_forward_batch): every token's choice from its logits (one
// warp per token, select_warp), then the flat slot table: token t's chosen
// experts, in router order, are slots slot_base[t] .. + n_t as (expert, t).
struct SelectBatchArgs {
    const float *logits;        // [n_tok][n_expert]
    uint32_t n_tok, n_expert, n_used;
    int32_t norm;
    float prune;
    sg_moe_choice *choices;     // [n_tok]
    uint32_t *slot_base;        // [n_tok]
    int32_t *slots;             // [n_tok * n_used][2]
    uint32_t *n_slots;
    int32_t *slots_sh;          // shared expert: [n_tok][2] = (0, t), or null
    uint32_t *n_slots_sh;
    // expert parallelism (slots_local set): the slots whose expert is in
    // [ep_lo, ep_hi), as (expert - ep_lo, token), and their global slot indices
    int32_t *slots_local;
    uint32_t *slot_global;
    uint32_t *n_local;
    uint32_t ep_lo, ep_hi;
    unsigned *ticket;           // 0 at launch (the router kernel zeroes it); back to 0 after
    // optional: the slots grouped by expert into jobs of at most job_max
    // slots (moe_batch_fused's union jobs, smollm_chat.rs:1040-1120): job j
    // is jobs[j * MOE_JOB_INTS ..] = {expert, n, slot_0 .. slot_{n-1}}, the
    // jobs of an expert consecutive, *n_jobs of them
    int32_t *jobs;
    uint32_t *n_jobs;
    uint32_t job_max;           // slots per job, 1 .. MOE_JOB_MAX
    uint32_t jobs_cap;          // jobs the table holds
};
constexpr uint32_t MOE_JOB_MAX = 8;
constexpr uint32_t MOE_JOB_INTS = 2 + MOE_JOB_MAX;
constexpr uint32_t SELECT_BATCH_THREADS = 128;  // one warp per token, ceil(n_tok / 4) CTAs
// per warp: 256 floats and a Choice; then the token bases (n_tok + 1), the
// job build's per-expert counts and job bases (256 each) and per-slot ranks,
// and every token's slot count and experts (the last CTA stages them once)
__host__ __device__ inline uint32_t select_batch_smem(uint32_t n_tok) {
    return (SELECT_BATCH_THREADS / 32) * (256u * 4u + (uint32_t)sizeof(moe::Choice)) + (n_tok + 1u) * 4u +
           2u * 256u * 4u + n_tok * MOE_MAXK * 4u + n_tok * (1u + MOE_MAXK) * 4u;
}

struct CombineBatchArgs {
    const sg_moe_choice *choices;
    const uint32_t *slot_base;
    const float *y;             // slot s at y + s * dim
    const float *ysh;           // shared expert: token t at ysh + t * dim, or null
    const float *shared_scale;  // [n_tok]
    float *out;                 // token t at out + t * ldo
    uint64_t ldo;
    uint32_t dim, n_used;
    // expert parallelism (recv set): slot s row r arrives as the pair
    // (epoch << 32 | value) at recv[(e & 1) * half + s * dim + r], e =
    // *epoch + 1; the last CTA to finish stores e in *epoch
    const unsigned long long *recv;
    uint64_t half;
    unsigned *ticket;
    unsigned *epoch;
};

// bars (64) | x of tok_chunk tokens (dim floats each) | rows (rows_per_cta,
// padded) ; the gate CTA puts the gate vector where the rows go.
__host__ __device__ inline uint32_t router_row_stride(uint32_t dim) { return dim * 4u + ROUTER_ROW_PAD; }
__host__ __device__ inline uint32_t router_smem_bytes(uint32_t dim, uint32_t rows_per_cta, uint32_t tok_chunk) {
    return 64u + (tok_chunk ? tok_chunk : 1u) * dim * 4u + (rows_per_cta ? rows_per_cta : 1u) * router_row_stride(dim);
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
__global__ void moe_select_batch_kernel(const __grid_constant__ SelectBatchArgs a);
__global__ void moe_combine_batch_kernel(const __grid_constant__ CombineBatchArgs a);

}  // namespace sg
