// gemv_q8k.cuh — Q4_K / Q6_K weight x Q8_K activation GEMV for B200.
//
// Replaces quant_q8k::rows<B,T> / matmul_rows (quant_q8k.rs:166-295) with the
// same fp32 results bit for bit.
//
// Data flow per CTA (persistent over row tiles):
//   HBM --cp.async.bulk (TMA engine, mbarrier ring of S stages)--> shared
//   memory --LDS--> registers --dp4a--> exact int32 lane sums (phase A) -->
//   shared scratch --> per-(row, vector, lane) fp32 FMA chain over the row's
//   super-blocks in block order, 8-lane tree, minus the sequential correction
//   (phase B) --> fp32 out.
//
// Exactness: the reference's output for row r and vector b is
//   hsum(acc) - corr, acc_l = fma(d_i*xd_i, float(sumi_{i,l}), acc_l) over
//   blocks i in order, hsum = ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)),
//   corr = sum_i in order of (dmin_i*xd_i)*float(s_i)   [Q4_K]
//                          or (d_i*xd_i)*float(32*s_i)  [Q6_K].
// The int32 lane sums sumi_{i,l} = sum_k sc_k(l) * sum_{j=4l..4l+3} w_k[j]*y_k[j]
// cannot overflow (|sumi| < 2^31; products fit dp4a), so any summation order
// gives the same integers, and every float step below is the same IEEE
// operation with explicit _rn intrinsics (no contraction).
#pragma once

#include "common.cuh"

namespace sg {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_MAXV = 16;  // vectors per launch (more = several launches)
enum { DT_Q4K = 0, DT_Q6K = 1 };

struct GemvArgs {
    const uint8_t *w;     // row 0 of the tensor, 16-byte aligned
    uint64_t tma_limit;   // bulk copies stay below w + tma_limit (16-aligned end of the tensor)
    uint32_t nb;          // super-blocks per row
    uint32_t rb;          // bytes per row
    uint32_t r0, nrows;   // rows r0 .. r0 + nrows
    uint32_t R;           // rows per tile
    uint32_t ntiles;
    uint32_t stage_bytes;
    uint32_t nstages;
    uint32_t sum_stride;  // int32 entries per (row, vector) in the lane-sum scratch
    uint32_t nvec;
    const float *xd[GEMV_MAXV];
    const int8_t *xs[GEMV_MAXV];
    const int16_t *xb[GEMV_MAXV];
    float *out[GEMV_MAXV];
    int32_t *dbg_sums;    // lane-sum export for vector 0 (sg_block_sums), else null
};

// Shared-memory bytes of one launch, beside the stages: lane sums + corrections.
__host__ __device__ inline uint32_t gemv_scratch_bytes(uint32_t R, uint32_t nv, uint32_t nb, uint32_t stride) {
    return R * nv * stride * 4u + R * nv * nb * 4u;
}

template <int DT, int NV, int CPT, bool DBG>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_q8k_kernel(const __grid_constant__ GemvArgs a);

}  // namespace sg
