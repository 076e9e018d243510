// gemm_tc.cuh — Q4_K / Q6_K weights x Q8_K activations for a batch of up to 128
// vectors on the 5th-generation tensor cores (tcgen05.mma, accumulators in
// TMEM), bit for bit the GEMV's and the reference's matmul_rows
// (quant_q8k.rs:166-295, block layouts of q4k_gemv.rs:26-31 and quant.rs:34-39).
//
// The reference's dot keeps, per row and super-block, eight int32 "AVX lanes":
// lane L holds sum_j sc_j * sum_e q[32j + 4L + e] * y[32j + 4L + e] over the
// eight 32-element sub-blocks j (e = 0..3), and folds each lane into its own
// fp32 chain acc_L = fma(d * xd, float(lane), acc_L).  Those integer lane sums
// are what this kernel moves onto the tensor cores, exactly:
//   * A (weights, 128 rows per CTA): the element sc_j * q, at most 63 * 15 =
//     945, is an exact f16; K is permuted so lane L's 32 elements are
//     contiguous (position 32L + 4j + e), so one K=32 product is one lane;
//   * B (activations, 16 tokens per CTA): the Q8_K byte y, an exact f16;
//   * D (fp32 in TMEM): every product and every partial sum is an integer
//     below 32 * 945 * 128 < 2^24, so the fp32 accumulation is exact in any
//     order and D holds the int32 lane sum as a float, the very value the
//     reference converts.
// The CUDA cores do what stays scalar: the f16 staging (one HFMA2 per two
// elements), the per-lane fp32 FMA chain over super-blocks in order, the
// min correction (integer sum of mins x bsums) and the 8-lane tree
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) minus the correction.
#pragma once

#include "common.cuh"
#include "gemm_batch.cuh"
#include "gemv_tiled.cuh"

namespace sg {

constexpr uint32_t TC_ROWS = 128;     // M: eight 16-row TILED16 tiles
constexpr uint32_t TC_TOK = 16;       // N: tokens per CTA (blockIdx.y = token group)
constexpr uint32_t TC_THREADS = 256;  // 8 warps: staging, then the epilogue (4 TMEM lane quarters x 2 lane sets)
constexpr uint32_t TC_TMEM_COLS = 256;  // two buffers of 8 lanes x 16 tokens
constexpr uint32_t TC_A_BYTES = TC_ROWS * 256u * 2u;
constexpr uint32_t TC_B_BYTES = TC_TOK * 256u * 2u;
// two operand stages A | B; the block's token scalars bs2[16][8] (int32: bsum
// 2j + bsum 2j+1) | xd[16] in three slots (block i mod 3): a warp may stage
// block i + 1 while another still runs the epilogue of block i - 1
constexpr uint32_t TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr uint32_t TC_XS_BYTES = 1024;
constexpr uint32_t TC_HDR_BYTES = 1024 + 3u * TC_XS_BYTES;
constexpr uint32_t TC_SMEM = TC_HDR_BYTES + 2u * TC_STAGE_BYTES;

// Q6_K: sc * w (|sc| <= 128, w <= 63) needs 13 bits and a lane sum can reach
// 32 * 8064 * 128 > 2^24, so w = 16 w_hi + w_lo gives two exact products per
// lane, A_lo = sc * w_lo (|.| <= 1920) and A_hi = sc * w_hi (|.| <= 384), each
// summed below 2^23 in its own TMEM accumulator; lane = 16 hi + lo in int32.
// A super-block is staged in two units of four lanes (lanes 4u..4u+3, the
// TILED16 chunks of parity u): A_lo | A_hi | B of one unit in 68 KB.
constexpr uint32_t TC6_A_BYTES = TC_ROWS * 128u * 2u;
constexpr uint32_t TC6_B_BYTES = TC_TOK * 128u * 2u;
constexpr uint32_t TC6_STAGE_BYTES = 2u * TC6_A_BYTES + TC6_B_BYTES;
constexpr uint32_t TC6_XS_BYTES = 2048;  // bsum[16][16] (int32) | xd[16]
constexpr uint32_t TC6_HDR_BYTES = 1024 + 3u * TC6_XS_BYTES;
constexpr uint32_t TC6_SMEM = TC6_HDR_BYTES + 2u * TC6_STAGE_BYTES;
constexpr uint32_t TC6_TMEM_COLS = 512;  // two buffers of (lo, hi) x 8 lanes x 16 tokens

struct GemmTcArgs {
    const uint8_t *w;           // TILED16 Q4_K tiles (16-byte aligned)
    uint32_t nb;                // super-blocks per row
    uint32_t t0, ntiles;        // tiles t0 .. t0 + ntiles
    uint32_t r0, r1;            // rows written
    const uint8_t *qb;          // QB image of the ntok vectors (gemm_batch.cuh)
    uint32_t ntok;
    float *out;                 // vector t, row r at out + t * ldo + r
    uint64_t ldo;
    uint32_t swiglu;            // as GemmBatchArgs::swiglu
};

__global__ void gemm_tc_q4k_kernel(const __grid_constant__ GemmTcArgs a);
__global__ void gemm_tc_q6k_kernel(const __grid_constant__ GemmTcArgs a);

}  // namespace sg
