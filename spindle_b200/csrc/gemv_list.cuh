// gemv_list.cuh — several independent TILED16 GEMVs in one persistent launch.
//
// The reference runs a decode step's matvecs one after another, each a
// parallel-for over rows (smollm_chat.rs:309-318, quant_q8k.rs:255-295).  On
// the GPU one launch per matrix drains HBM at every launch boundary: a CTA of
// the next kernel cannot become resident (one 16-warp CTA per SM with most of
// the shared memory) before this kernel's CTA on that SM exits, so each
// boundary costs the DRAM latency again.  gemv_list_kernel takes a list of
// matrices instead: every warp's ring of bulk copies runs on from its last
// item of matrix j into its first item of matrix j + 1, so the copies of the
// next matrix are in flight while this one's last blocks are dotted.
//
// Per matrix the work is gemv_tiled_kernel's with one vector: S_j warps share
// a 16-row tile, warp slot s owns super-blocks [s*nb/S, (s+1)*nb/S), slot 0
// keeps the per-lane fp32 chain and continues it over the other slots' blocks
// in block order, then the 8-lane tree and the correction (quant_q8k.rs:
// 243-248).  So every output is bit for bit the one sg_matvec writes.  x_j
// is staged in one of two buffers: quantized by the CTA (fp32 input), or one
// bulk copy of its Q8_K image issued while matrix j - 1 is still in work;
// the CTA synchronizes once per matrix.  Each matrix's remainder tiles start
// where the previous matrix's ended, so that no CTA takes every remainder.
#pragma once

#include "gemv_tiled.cuh"

namespace sg {

constexpr uint32_t GL_MAX = 16;  // matrices per launch (SG_LIST_MAX)

struct GlMat {
    const uint8_t *w;    // TILED16 buffer (16-byte aligned)
    const float *x;      // fp32 input, 256 * nb values (16-byte aligned), or
    const uint8_t *img;  // its Q8_K image (act_bytes(nb) bytes, 16-byte aligned)
    float *out;          // rows outputs
    uint32_t dt;         // 0: Q4_K, 1: Q6_K
    uint32_t nb;         // super-blocks per row
    uint32_t ntiles;     // 16-row tiles
    uint32_t rows;
    uint32_t S, s_log2;     // warps per tile (a power of two)
    uint32_t bc;            // super-blocks per ring stage
    uint32_t slot_blocks;   // ceil(nb / S)
    uint32_t tiles_q, tiles_r;  // ntiles = tiles_q * (gridDim.x * warps / S) + tiles_r
    uint32_t rot;           // tile group g (CTA-minor numbering) takes the tiles of group
                            // (g + rot) % (gridDim.x * warps / S): the remainder tiles
                            // of successive matrices go to different CTAs
};

struct GlArgs {
    uint32_t n;
    uint32_t nstages, stage_bytes;  // the rings (the same for every matrix)
    uint32_t act_bytes;             // one of the two activation buffers
    uint32_t chain_floats;          // the CTA's chain scratch
    GlMat m[GL_MAX];
};

// The barrier area: the rings' mbarriers from 0, the two activation buffers'
// (image copies) at GL_IMG_BAR_OFF.
constexpr uint32_t GL_IMG_BAR_OFF = 512;

// Dynamic shared memory: barriers | two activation buffers | rings | chain scratch.
__host__ __device__ inline uint32_t list_smem_bytes(uint32_t warps, uint32_t nstages, uint32_t stage_bytes,
                                                    uint32_t act_bytes, uint32_t chain_floats) {
    return TGEMV_BAR_BYTES + 2u * act_bytes + warps * nstages * stage_bytes + chain_floats * 4u;
}

// Chain scratch of one matrix in a CTA of `warps` warps: every worker
// slot of every group hands slot_blocks blocks (CHAIN_FLOATS each) to its slot 0.
__host__ __device__ inline uint32_t list_chain_floats(uint32_t warps, uint32_t S, uint32_t slot_blocks) {
    return (warps / S) * (S - 1u) * slot_blocks * CHAIN_FLOATS;
}

__global__ void __launch_bounds__(TGEMV_WARPS * 32, 1) gemv_list_kernel(const __grid_constant__ GlArgs a);

// Q8_K images of a list of fp32 vectors in one launch: vector j (nb[j]
// super-blocks at x[j]) to img[j] = qs[256 nb] | bsums[16 nb] (int16) | d[nb]
// (f32, padded to 16 bytes): the shared-memory image of act_bytes, so that a
// GEMV stages it with one bulk copy.  One warp per super-block, Q8K::quantize
// bit for bit (q8k_block.cuh).
struct QImgArgs {
    uint32_t n;
    const float *x[GL_MAX];
    uint8_t *img[GL_MAX];
    uint32_t nb[GL_MAX];
    uint32_t blk0[GL_MAX + 1];  // prefix sums of nb
};
__global__ void q8k_images_kernel(const __grid_constant__ QImgArgs a);

}  // namespace sg
