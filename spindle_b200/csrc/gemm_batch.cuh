// gemm_batch.cuh — Q4_K / Q6_K weights x Q8_K activations for a batch of up
// to 64 vectors per launch (matvec_multi / matmul_rows with many vectors,
// smollm_chat.rs:447-512, quant_q8k.rs:255-295): the prefill chunks and the
// verify batches of forward_batch_slice.
//
// The GEMV kernels (gemv_tiled.cu) take at most 8 vectors per launch, so a
// 64-token chunk made 8 launches that each read the whole matrix again and
// ran the vector loop in spilled registers.  Here one launch reads every
// weight column once for all tokens:
//   * thread 0 streams, per item, one super-block column of `tps`
//     16-row tiles (TILED16, contiguous) plus that block's Q8_K data of all
//     tokens (block-major QB image, one contiguous run) into a ring of stages
//     with bulk copies (TMA engine), full/empty mbarriers, bounded waits;
//   * the warps each own one tile of the step and TPW tokens (8 warps of 8
//     or 16 of 4): thread (g, r) keeps AVX lanes 4g..4g+3 of row r for its
//     tokens, exactly as the GEMV's single-slot path does (same int32 lane sums, same fp32 FMA
//     chain over blocks in order, same correction sum, same 8-lane tree), so
//     every output is bit for bit the GEMV's (and the reference's).
// A step covers tps = consumers / nq tiles, nq = the token groups of TPW
// (a power of two).
#pragma once

#include "common.cuh"
#include "gemv_tiled.cuh"

namespace sg {

constexpr uint32_t GB_MAX_TOK = 64;    // vectors of one gemm_batch_kernel launch (one QB group)
constexpr uint32_t QB_MAX_TOK = 128;   // vectors of one QB image (prefill chunks of feed, smollm_chat.rs:3090)
constexpr uint32_t GB_MAX_STAGES = 6;
// warps per CTA for TPW vectors per warp
__host__ __device__ constexpr uint32_t gb_consumers(int tpw) { return 64u / (uint32_t)tpw; }
constexpr uint32_t GB_BAR_BYTES = 128;

// QB: Q8_K images of n vectors, block-major, in groups of QB_GROUP vectors.
// Group q (vectors 64q .. 64q + n_q - 1, n_q = min(64, n - 64q)) starts at qb
// + q * nb * qb_block_bytes(64); its block i is at + i * qb_block_bytes(n_q):
// qs[n_q][256] | bsums[n_q][16] (int16) | d[n_q] (float), padded to 16
// bytes.  With n <= 64 there is one group, the plain block-major image.
constexpr uint32_t QB_GROUP = 64;
__host__ __device__ inline uint32_t qb_block_bytes(uint32_t n) { return (n * 292u + 15u) & ~15u; }
__host__ __device__ inline uint64_t qb_group_offset(uint32_t q, uint32_t nb) {
    return (uint64_t)q * nb * qb_block_bytes(QB_GROUP);
}
__host__ __device__ inline uint32_t qb_group_tokens(uint32_t n, uint32_t q) {
    return n - q * QB_GROUP < QB_GROUP ? n - q * QB_GROUP : QB_GROUP;
}
__host__ __device__ inline uint64_t qb_image_bytes(uint32_t n, uint32_t nb) {
    const uint32_t full = n / QB_GROUP, rem = n % QB_GROUP;
    return qb_group_offset(full, nb) + (rem ? (uint64_t)nb * qb_block_bytes(rem) : 0u);
}

// One warp per (vector, block): x_t = x + t * ldx (cols = 256 * nb floats,
// 16-byte aligned rows), the exact Q8K::quantize of quant_q8k.rs:84-121.
struct QbArgs {
    const float *x;
    uint64_t ldx;
    uint32_t n, nb;
    uint8_t *qb;
};

struct GemmBatchArgs {
    const uint8_t *w;           // TILED16 tiles (16-byte aligned)
    uint32_t nb;                // super-blocks per row
    uint32_t t0, ntiles;        // tiles t0 .. t0 + ntiles
    uint32_t r0, r1;            // rows written
    const uint8_t *qb;          // QB image of the ntok vectors
    uint32_t ntok, nq, tps;     // vectors; groups of TPW vectors; tiles per step (nq * tps = consumer warps)
    uint32_t nstages, stage_bytes;  // stage: tps weight columns | one QB block
    float *out;                 // vector t, row r at out + t * ldo + r
    uint64_t ldo;
    // swiglu: each tile holds 8 gate rows then the 8 up rows of the same
    // outputs (the packed gate/up layout); output j = tile * 8 + r of vector t
    // is silu(gate) * up at out + t * ldo + j, for 2 j < r1
    uint32_t swiglu;
};

__global__ void q8k_batch_kernel(const __grid_constant__ QbArgs a);
template <int DT, int TPW>
__global__ void gemm_batch_kernel(const __grid_constant__ GemmBatchArgs a);

}  // namespace sg
