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
// Kernel: S warps share a 16-row tile; warp slot s owns the super-blocks
// [s*nb/S, (s+1)*nb/S).  Thread (g, r) = (lane / 16, lane % 16) computes AVX
// lanes 4g..4g+3 of row r.  Slot 0 keeps the exact per-lane fp32 FMA chain of
// quant_q8k.rs:243 in registers; slots 1..S-1 hand it, through shared memory,
// float(lane sum), d*xd and the correction term of each of their blocks, and
// slot 0 continues the chain over them in block order.  The 8-lane tree and
// the correction finish the row (quant_q8k.rs:246-248).
//
// Data movement: weights stream HBM -> shared memory through a per-warp ring
// of bulk copies (TMA engine), issued before the kernel waits on the grid it
// depends on (programmatic dependent launch), so weight streaming overlaps the
// kernel that produced the activations.  The Q8_K activations are then staged
// once per CTA in shared memory.
#pragma once

#include "common.cuh"

namespace sg {

constexpr int TGEMV_WARPS = 16;        // most warps per CTA (launches use 8 or 16)
constexpr int TGEMV_MAXV = 8;          // vectors per launch
constexpr uint32_t TILE_ROWS = 16;
constexpr uint32_t CHAIN_FLOATS = 160; // per (block, vector): 16 rows x (8 lane floats + d*xd + corr term)
constexpr uint32_t TGEMV_BAR_BYTES = 1024;

__host__ __device__ constexpr uint32_t tiled_col_bytes(int dt) { return dt == 0 ? 2304u : 3360u; }

// Shared-memory image of one Q8_K vector: qs[cols] | bsums[nb*16] | d[nb] (16-aligned).
__host__ __device__ inline uint32_t act_bytes(uint32_t nb) { return nb * 256u + nb * 32u + ((nb * 4u + 15u) & ~15u); }

struct TGemvArgs {
    const uint8_t *w;     // TILED16 buffer (16-byte aligned)
    uint32_t nb;          // super-blocks per row
    uint32_t t0, ntiles;  // tiles t0 .. t0 + ntiles
    uint32_t r0, r1;      // rows written (others of the tiles are skipped)
    uint32_t S;           // warps per tile (1, 2, 4 or 8)
    uint32_t bc;          // super-blocks per stage
    uint32_t nstages;
    uint32_t stage_bytes;
    uint32_t slot_blocks; // max super-blocks of one slot (chain scratch sizing)
    uint32_t nvec;
    const float *x[TGEMV_MAXV];   // fp32 inputs, when the kernel quantizes them itself (QX)
    const float *xd[TGEMV_MAXV];
    const int8_t *xs[TGEMV_MAXV];
    const int16_t *xb[TGEMV_MAXV];
    float *out[TGEMV_MAXV];
};

// Dynamic shared memory of one CTA of `warps` warps:
// barriers | activations | rings | chain scratch.
__host__ __device__ inline uint32_t tiled_smem_bytes(uint32_t warps, uint32_t S, uint32_t nstages,
                                                     uint32_t stage_bytes, uint32_t slot_blocks, uint32_t nv,
                                                     uint32_t nb) {
    const uint32_t groups = warps / S;
    return TGEMV_BAR_BYTES + nv * act_bytes(nb) + warps * nstages * stage_bytes +
           groups * (S - 1) * slot_blocks * nv * CHAIN_FLOATS * 4u;
}

// QX = true: the inputs are fp32 (a.x) and every CTA quantizes them to Q8_K
// in shared memory (the reference's matvec = Q8K::quantize + matmul_rows, in
// one kernel).  QX = false: the inputs are Q8_K vectors (a.xd, a.xs, a.xb).
template <int DT, int NV, bool QX>
__global__ void __launch_bounds__(TGEMV_WARPS * 32, 1) gemv_tiled_kernel(const __grid_constant__ TGemvArgs a);

__global__ void repack_tiled16_kernel(int dt, const uint8_t *src, uint64_t rows, uint32_t nb, uint8_t *dst,
                                      int inverse);

}  // namespace sg
