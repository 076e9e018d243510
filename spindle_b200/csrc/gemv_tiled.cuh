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

// What the kernel reads as its vectors, and where its tiles come from.
//   IN_Q8K:   Q8_K vectors (xd, xs, xb).
//   IN_F32:   fp32 vectors x, quantized to Q8_K by every CTA in shared memory
//             (the reference's matvec = Q8K::quantize + matmul_rows in one kernel).
//   IN_MOE_X: grouped over the chosen experts: launch tile tt is tile
//             tt % tiles_per_mat of expert id[tt / tiles_per_mat] (slot s =
//             tt / tiles_per_mat), whose matrix is at w + id * mat_stride; one
//             fp32 vector x[0], quantized as in IN_F32; slot s's rows go to
//             out[0] + s * out_stride.  With `logits`, every CTA makes the
//             choice itself from the router's logits (softmax, top-k, prune,
//             weights) and CTA 0 publishes it in sel_out; without, it runs `sel`.
//             With qx_image, x arrives already quantized (an act_bytes(nb)
//             shared-memory image made by the router) in one bulk copy.
//             With swiglu, each tile holds 8 gate rows then the 8 up rows of
//             the same outputs, and the kernel writes h = silu(gate) * up
//             (8 outputs per tile) instead of the 16 rows.
//   IN_MOE_H: grouped like IN_MOE_X over `sel`; slot s's vector is the fp32
//             h at gu + s * gu_stride, quantized by each CTA for the slots its
//             tiles belong to.
// In the MoE modes each CTA takes a contiguous range of the launch's tiles.
constexpr int IN_Q8K = 0, IN_F32 = 1, IN_MOE_X = 2, IN_MOE_H = 3;
constexpr uint32_t MOE_MAXK = SG_MOE_MAX_USED;

constexpr uint32_t TP_MAX_RANKS = 8;

struct TGemvArgs {
    const uint8_t *w;     // TILED16 buffer (16-byte aligned)
    uint32_t nb;          // super-blocks per row
    uint32_t t0, ntiles;  // tiles t0 .. t0 + ntiles
    uint32_t r0, r1;      // rows written (others of the tiles are skipped)
    uint32_t S;           // warps per tile (1, 2, 4, 8 or 16)
    uint32_t s_log2;      // log2(S)
    uint32_t tiles_q, tiles_r;  // GEMV: ntiles = tiles_q * (gridDim.x * warps / S) + tiles_r
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
    // IN_MOE_X / IN_MOE_H only
    const sg_moe_choice *sel;   // the choice to run (IN_MOE_H; IN_MOE_X without logits)
    sg_moe_choice *sel_out;     // IN_MOE_X with logits: CTA 0 writes the choice here
    const float *logits;        // IN_MOE_X: router logits [n_expert], or null
    float *probs;               // optional: CTA 0 writes the softmax here
    uint32_t n_used;            // top-k
    int32_t norm;
    float prune;
    uint32_t nact;              // IN_MOE_H: activation images per CTA
    uint32_t swiglu;            // IN_MOE_X: interleaved gate/up tiles, h out
    const uint8_t *qx_image;    // IN_MOE_X: Q8_K image of x, or null
    uint64_t mat_stride;
    uint64_t out_stride;
    uint32_t tiles_per_mat;
    uint32_t max_slots;   // slots the launch was sized for (n_used)
    uint32_t n_expert;
    uint32_t n_ff;        // IN_MOE_H
    const float *gu;      // IN_MOE_H
    uint64_t gu_stride;   // IN_MOE_H, floats
    // Batched MoE (several tokens): the slots are (expert, token) pairs in
    // device memory, *n_slots of them (at most max_slots), instead of one
    // token's choice; IN_MOE_X stages each slot's token image from qx_tokens
    // (act_bytes(nb) apart).
    const int32_t *slots;
    const uint32_t *n_slots;
    const uint8_t *qx_tokens;
    // expert parallelism (IN_MOE_H with slots, npeers > 0): row r of local
    // slot j goes as the pair (epoch << 32 | value) to peer_recv[p][(e & 1) *
    // ep_half + slot_global[j] * out_stride + r] on every rank, e = *epoch + 1
    const uint32_t *slot_global;
    uint64_t ep_half;
    // Row-split tensor parallelism (IN_Q8K / IN_F32, npeers > 0).  The call's
    // epoch e is *epoch + 1.  Row r of vector v is stored as the pair
    // (e << 32 | value bits) at peer_recv[p][h*nvec*tp_rows + v*tp_rows +
    // row_off + r] on every rank p, h = e & 1; then every CTA reads its share
    // of this rank's receive buffer, waiting for each pair to carry e, into
    // out[0][v * out_stride + row]; the last CTA to finish stores e in *epoch.
    uint32_t npeers;
    uint32_t row_off;
    uint32_t tp_rows;     // rows of the whole matrix
    unsigned long long *peer_recv[TP_MAX_RANKS];
    const unsigned long long *my_recv;  // this rank's receive buffer
    unsigned *ticket;
    unsigned *epoch;
    // Jobs mode (MoE with a slot table, NV > 1): the launch's units are jobs
    // of the select kernel's table (SelectBatchArgs::jobs: {expert, n,
    // slot_0 ..}, MOE_JOB_INTS ints each, *n_jobs of them, at most
    // max_slots): every weight block of a job's expert is decoded once for
    // its n slots; slot s's vector is its token's image (IN_MOE_X) or h at
    // gu + s * gu_stride (IN_MOE_H), its rows go to out[0] + s * out_stride.
    const int32_t *jobs;
    const uint32_t *n_jobs;
    uint32_t job_ints;
    uint32_t pf_x;        // IN_F32: fetch the fp32 inputs into L2 before the dependency wait
};

// In the MoE modes the choice is kept at the top of the barrier area: n at
// MOE_SEL_OFF, ids 64 bytes after it; the barrier of the x image copy sits
// just below (MOE_QX_BAR_OFF), and the rings' barriers below that.
constexpr uint32_t MOE_SEL_OFF = TGEMV_BAR_BYTES - 128;
constexpr uint32_t MOE_QX_BAR_OFF = MOE_SEL_OFF - 8;

// Shared memory the in-kernel expert choice borrows from the rings (before
// any weight copy is issued): probabilities, sort keys and a little scratch.
__host__ __device__ inline uint32_t moe_select_bytes(uint32_t n_expert) { return 2u * ((n_expert * 4u + 15u) & ~15u) + 512u; }

// Activation images staged per CTA.
__host__ __device__ inline uint32_t tiled_nact(int mode, uint32_t nv, uint32_t nact) {
    return (mode == IN_MOE_H || mode == IN_MOE_X) ? (nact ? nact : 1u) : nv;
}

// Dynamic shared memory of one CTA of `warps` warps:
// barriers | activations (nact images) | rings | chain scratch.
__host__ __device__ inline uint32_t ilog2u(uint32_t v) {
#ifdef __CUDA_ARCH__
    return 31u - (uint32_t)__clz(v);
#else
    return 31u - (uint32_t)__builtin_clz(v);
#endif
}

// (S a power of two, as the kernel requires)
__host__ __device__ inline uint32_t tiled_smem_bytes(uint32_t warps, uint32_t S, uint32_t nstages,
                                                     uint32_t stage_bytes, uint32_t slot_blocks, uint32_t nv,
                                                     uint32_t nb, uint32_t nact, uint32_t job_bytes = 0) {
    const uint32_t groups = S ? warps >> ilog2u(S) : 0u;
    return TGEMV_BAR_BYTES + nact * act_bytes(nb) + job_bytes + warps * nstages * stage_bytes +
           groups * (S - 1) * slot_blocks * nv * CHAIN_FLOATS * 4u;
}

// Jobs mode (TGemvArgs::jobs): per local job its slot count and NV slot
// indices, after the activation images (MOE_MAXK local jobs at most).
__host__ __device__ constexpr uint32_t tiled_job_bytes(uint32_t nv) { return MOE_MAXK * (1u + nv) * 4u; }

template <int DT, int NV, int MODE>
__global__ void __launch_bounds__(TGEMV_WARPS * 32, 1) gemv_tiled_kernel(const __grid_constant__ TGemvArgs a);

// GGUF row `row` is row (row / rpg) * dgr + off + row % rpg of the TILED16
// buffer (plain matrices: rpg = rows, dgr = off = 0; stacked expert tensors:
// rpg = rows per expert, dgr = padded rows per stacked expert).
__global__ void repack_tiled16_kernel(int dt, const uint8_t *src, uint64_t rows, uint32_t nb, uint8_t *dst,
                                      int inverse, uint64_t rpg, uint64_t dgr, uint64_t off);

}  // namespace sg
