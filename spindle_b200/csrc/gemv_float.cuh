// gemv_float.cuh — the float matvec kernels on GGUF rows: matvec_rows_avx2
// (quant.rs:939-1094, one vector) and rows_multi (quant_multi.rs:126-217,
// several vectors sharing one decode of each weight block) for F32, F16, Q8_0,
// Q4_K and Q6_K.
//
// The reference keeps eight fp32 accumulator lanes per row (one AVX register)
// and runs every lane as a sequential FMA chain over the row; the two
// algorithms differ in how a lane's chain is formed, so the same vector gives
// different bits through them, and both are restated here:
//
//   single (matvec_rows_avx2): lane l takes element l of every 8-wide chunk.
//     F32/F16: acc = fma(w, x, acc), then hsum_avx2(acc) + the scalar tail
//     (products and sums rounded separately).  Q8_0: per 32-block
//     s = fma chain of q*x over its four chunks from 0, acc = fma(d, s, acc).
//     Q4_K (presum form): per 32-value half-chunk s = fma chain from 0,
//     acc = fma(d*sc, s, acc); the mins go into a separate scalar
//     total_min += (sum_k mn_k * subsum_k) * dmin; result hsum(acc) - total_min.
//     Q6_K: per block acc_b = fma chain of (q*sc)*x from 0 over the block,
//     total = fma(d, acc_b, total); result hsum(total).
//   multi (rows_multi): each block is first decoded to fp32 weights
//     (Q4_K w = fma(d*sc, q, -(dmin*mn)); Q6_K w = (d*sc)*q), then two
//     accumulator sets a0/a1 take the even and odd 8-wide chunks of every 16;
//     Q8_0 alternates a0/a1 per 32-block.  Result hsum(a0 + a1), whose tree
//     pairs lanes (0,2),(1,3) where hsum_avx2 pairs (0,1),(2,3).
//
// On the GPU the eight lanes of a row are eight threads; a warp holds four
// rows.  Integer weights become floats exactly by the 2^23 bias trick (no
// conversion unit), every float operation is an explicit _rn intrinsic, and the
// two horizontal trees are restated with xor shuffles.
#pragma once

#include "common.cuh"

namespace sg {

constexpr uint32_t FGEMV_THREADS = 256;         // 8 warps, 4 rows each
constexpr uint32_t FGEMV_ROWS = FGEMV_THREADS / 8;
constexpr uint32_t FGEMV_MAXV = 8;

struct FGemvArgs {
    const uint8_t *w;       // row 0 of the matrix (GGUF rows)
    uint64_t row_bytes;
    uint32_t n;             // cols
    uint32_t r0, r1;
    uint32_t nvec;          // <= the instantiation's NV
    const float *x;         // x_b = x + b * ldx
    uint64_t ldx;
    float *out;             // out_b[r] = out[b * ldo + r]
    uint64_t ldo;
    uint32_t stage_x;       // one vector: copy x into shared memory first (fgemv_smem_bytes counts it)
};

// dtype codes of the kernel template (the C ABI's SG_* values)
enum : int { FDT_F32 = 0, FDT_F16 = 1, FDT_Q8_0 = 8, FDT_Q4_K = 12, FDT_Q6_K = 14 };

// Q4_K single-vector path: sums of x over each 32 values, per vector, in shared memory
__host__ __device__ inline uint32_t fgemv_presum_floats(int dt, bool multi, uint32_t nv, uint32_t n) {
    return (dt == FDT_Q4_K && !multi) ? ((nv * (n / 32) + 3u) & ~3u) : 0u;
}
// x staged in shared memory for one vector up to this many columns
constexpr uint32_t FGEMV_STAGE_X_MAX = 8192;
// Q6_K one vector with x staged: 8-block row spans (1680 bytes + 16 of
// padding) for the 4 rows of each warp, after x
constexpr uint32_t FGEMV_Q6_STAGE_BYTES = (FGEMV_THREADS / 32) * 4u * (8u * 210u + 16u);
__host__ __device__ inline uint32_t fgemv_smem_bytes(int dt, bool multi, uint32_t nv, uint32_t n, bool stage_x = false) {
    return fgemv_presum_floats(dt, multi, nv, n) * 4u + (stage_x ? n * 4u : 0u) +
           (stage_x && dt == FDT_Q6_K && !multi ? FGEMV_Q6_STAGE_BYTES : 0u);
}

template <int DT, int NV, bool MULTI>
__global__ void gemv_float_kernel(const __grid_constant__ FGemvArgs a);

}  // namespace sg
