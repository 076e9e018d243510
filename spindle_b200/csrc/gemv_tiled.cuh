// gemv_tiled.cuh — Q4_K / Q6_K x Q8_K GEMV over the TILED16 weight layout.
//
// TILED16 is a byte permutation of the GGUF rows, made once at upload
// (sg_repack_tiled16): rows are grouped in tiles of 16; a tile stores its
// super-block column i as contiguous planes, all 16-byte aligned:
//   Q4_K (2304 B per column): qs[16][128] | head[16][16]   (head = d, dmin, scales[12])
//   Q6_K (3360 B per column): qlqh[16][192] | scales[16][16] | d[16][2]
// Rows beyond the matrix (last tile) are zero.  The bytes per row and block
// are the GGUF ones, so the arithmetic is unchanged.
//
// Kernel: one warp owns a 16-row tile and walks its super-blocks in order;
// thread (g, r) = (lane / 16, lane % 16) computes AVX lanes 4g..4g+3 of row r.
// The exact per-lane fp32 FMA chain over blocks (quant_q8k.rs:243) therefore
// lives in registers, and the 8-lane tree + correction finish the row
// (quant_q8k.rs:246-248).  Weights stream HBM -> shared memory through a
// per-warp ring of bulk copies (TMA engine); activations are read through L1.
#pragma once

#include "common.cuh"

namespace sg {

constexpr int TGEMV_WARPS = 4;         // warps per CTA
constexpr int TGEMV_MAXV = 8;          // vectors per launch
constexpr uint32_t TILE_ROWS = 16;

__host__ __device__ constexpr uint32_t tiled_col_bytes(int dt) { return dt == 0 ? 2304u : 3360u; }

struct TGemvArgs {
    const uint8_t *w;     // TILED16 buffer (16-byte aligned)
    uint32_t nb;          // super-blocks per row
    uint32_t t0, ntiles;  // tiles t0 .. t0 + ntiles
    uint32_t r0, r1;      // rows written (others of the tiles are skipped)
    uint32_t bc;          // super-block columns per stage
    uint32_t nstages;
    uint32_t stage_bytes;
    uint32_t nvec;
    const float *xd[TGEMV_MAXV];
    const int8_t *xs[TGEMV_MAXV];
    const int16_t *xb[TGEMV_MAXV];
    float *out[TGEMV_MAXV];
};

template <int DT, int NV>
__global__ void __launch_bounds__(TGEMV_WARPS * 32) gemv_tiled_kernel(const __grid_constant__ TGemvArgs a);

__global__ void repack_tiled16_kernel(int dt, const uint8_t *src, uint64_t rows, uint32_t nb, uint8_t *dst,
                                      int inverse);

}  // namespace sg
