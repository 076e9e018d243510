// decode.cuh — the kernels of one decoder step besides the GEMVs and the MoE
// layer (forward_slice, smollm_chat.rs:3371-3552), one token at a time.  The
// token and its position live in device memory (state[0], state[1]) so that a
// whole step can be captured once and replayed: the argmax kernel writes the
// next token and advances the position.
//
// Every fp32 operation follows the reference's order: the RMSNorm and head-norm
// sums of squares are sequential, the attention recurrence runs position by
// position, the GEMVs and MoE passes are the exact integer kernels, and
// sin/cos/exp are glibc's sinf/cosf/expf bit for bit (glibc_math.h), the
// functions the reference's f32::sin_cos / f32::exp call on Linux.  The step
// is therefore bit-identical to the oracle's restatement of forward_slice
// with the host's glibc; the reference holds no golden vectors for it.
#pragma once

#include "common.cuh"

namespace sg {

constexpr uint32_t NORM_THREADS = 1024;
constexpr uint32_t ARGMAX_THREADS = 512;
constexpr uint32_t ARGMAX_CTAS = 128;

// x = dequant_row(embed[token]) * scale (dequant_row, quant.rs:1527-1660).
struct EmbedArgs {
    const uint8_t *embed;   // GGUF rows [vocab][dim]
    int32_t dtype;          // SG_F32, SG_F16, SG_Q4_K or SG_Q6_K
    uint32_t dim, vocab;
    float scale;
    const int32_t *state;   // state[0] = token
    float *x;
    // batch (grid.y tokens): token blockIdx.y is tokens[blockIdx.y], its x at x + blockIdx.y * dim;
    // block (0, 0) also stores the token count in *n_out when set
    const int32_t *tokens;
    uint32_t *n_out;
};

// x += rs * add (when add); xn = (x * inv) * w with inv = 1 / sqrt(mean(x^2) + eps);
// qx (when set) = Q8_K image of xn in the GEMV's shared-memory layout.
struct NormArgs {
    float *x;
    const float *add;
    float rs;
    const float *w;
    float eps;
    uint32_t n;
    float *xn;
    uint8_t *qx;
    // batch: CTA t normalizes token t (x, add, xn at + t * n; qx at + t * act_bytes(n / 256))
    // Optional, one token: add is the combine of the MoE layer before, made
    // here with moe_combine_kernel's arithmetic (sum over csel's slots of
    // w_i * cy_i[r] in router order, then + cscale * cysh[r]).
    const sg_moe_choice *csel;
    const float *cy;            // slot s at cy + s * n
    const float *cysh;          // shared expert output, or null
    const float *cscale;
    uint32_t cmax_slots;
};

// Batch: this position's QK-norm, RoPE and f16 K/V rows of token blockIdx.y
// (position *pos + blockIdx.y), one warp per head (q heads, then kv heads);
// q is rotated in place.  Tokens are qkv_stride floats apart in q, k and v.
struct RopeBatchArgs {
    float *q;
    const float *k, *v;
    uint64_t qkv_stride;
    const float *qn_w, *kn_w;
    float eps;
    const float *inv_freq;
    uint32_t head_dim, n_heads, n_kv;
    int32_t neox;
    const int32_t *pos;
    uint16_t *kc, *vc;
    uint32_t max_seq;
};

// One query head of grouped-query attention over positions 0..pos, with this
// position's part done in the same kernel: the per-head RMSNorm of q and k
// (when weights are given), RoPE on both, and K and V rounded to f16 (round to
// nearest even).  The first query head of each KV group writes this position's
// K and V rows into the caches; every head uses its own copy of them.
struct AttnArgs {
    const float *q, *k, *v;     // this position: [n_heads*hd], [n_kv*hd], [n_kv*hd]
    const float *qn_w, *kn_w;   // [head_dim] or null
    float eps;
    const float *inv_freq;      // [head_dim / 2], from the host (glibc powf)
    uint32_t head_dim, n_heads, n_kv, max_seq;
    int32_t neox;
    float scale;
    const int32_t *state;       // state[1] = pos
    uint16_t *kc, *vc;          // this layer's caches: [max_seq][n_kv * head_dim]
    float *out;                 // [n_heads * head_dim]
    // batch ("prepared"): token blockIdx.y at position state[0] + blockIdx.y,
    // q already normed and rotated at q + blockIdx.y * q_stride, this position's
    // K/V rows already in the caches; out at out + blockIdx.y * n_heads * head_dim
    uint32_t prepared;
    uint64_t q_stride;
    uint32_t nbuf;              // chunk buffers in shared memory (2..ATTN_MAX_BUF)
    uint32_t chunk;             // positions per chunk: 64 or 128 (smaller chunks, more CTAs per SM)
    uint32_t ntok;              // attention_batch_kernel: tokens of the batch
};

// Batch attention with the K/V rows shared (attention_batch_kernel): one CTA
// per (KV head, block of ATTN_PAIRS / group tokens) computes the group's
// ATTN_PAIRS (query head, token) pairs, staging each chunk of ATTN_BCH
// positions of the KV head's K and V rows once for all of them.
constexpr uint32_t ATTN_PAIRS = 16;
constexpr uint32_t ATTN_BCH = 32;
__host__ __device__ inline uint32_t attn_batch_threads(uint32_t head_dim) { return 2u * head_dim; }
// q (f32, rows padded by 4) | K, V f16 x 2 buffers | K, V f32 | scores | (p, alpha) | l, running max
__host__ __device__ inline uint32_t attn_batch_smem(uint32_t head_dim) {
    return ATTN_PAIRS * (head_dim + 4u) * 4u + 2u * 2u * ATTN_BCH * head_dim * 2u + 2u * ATTN_BCH * head_dim * 4u +
           ATTN_PAIRS * ATTN_BCH * 4u + ATTN_PAIRS * ATTN_BCH * 8u + 2u * ATTN_PAIRS * 4u;
}

// The greedy token (f32::total_cmp, last maximum on ties), written as the next
// step's token; the position advances.  ARGMAX_CTAS blocks each reduce a
// strided share to one (key, index) pair in partial[]; the last block to
// finish (ticket count) reduces those and resets the count to 0.
struct ArgmaxArgs {
    const float *logits;
    uint32_t n;
    int32_t *state;
    int64_t *out;               // optional: the token, also kept here
    unsigned long long *partial;  // [ARGMAX_CTAS]
    unsigned *count;            // 0 before the launch, 0 after it
    // batch (grid.y tokens): token t's logits at logits + t * ldl, partial +
    // t * ARGMAX_CTAS, count + t; out[t] gets its greedy token; state untouched
    uint32_t batch;
    uint64_t ldl;
};

// Positions of K and V staged in shared memory at a time, and the padding of a
// staged row (spreads the rows of one warp's positions over the banks).
constexpr uint32_t ATTN_CHUNK = 128;     // largest chunk (a.chunk: 64 or 128)
constexpr uint32_t ATTN_ROW_PAD = 16;

__host__ __device__ inline uint32_t attn_threads(uint32_t head_dim) { return head_dim < 256 ? 256u : 288u; }

constexpr uint32_t ATTN_MAX_BUF = 4;
// reserved (32 B), 1/l and the inverse norms (16 B), pad | q | q, k before RoPE |
// scores, then p | alpha | nbuf chunk buffers of K or V rows | this
// position's K, V (f16); every part 16-byte aligned
__host__ __device__ inline uint32_t attn_seq4(uint32_t max_seq) { return (max_seq + 3u) & ~3u; }
__host__ __device__ inline uint32_t attn_smem_bytes(uint32_t head_dim, uint32_t max_seq, uint32_t nbuf,
                                                    uint32_t chunk = ATTN_CHUNK) {
    return 64u + 3u * head_dim * 4u + 2u * attn_seq4(max_seq) * 4u + nbuf * chunk * (2u * head_dim + ATTN_ROW_PAD) +
           2u * head_dim * 2u;
}

// Pipeline link between two ranks (forward_slice stages on different GPUs):
// the sender stores n floats as (epoch << 32 | value) pairs into the
// receiver's buffer (two halves by epoch parity), after the receiver has
// acknowledged the call two before (so the half is free); the receiver waits
// for each pair, writes the plain floats, and its last block acknowledges the
// epoch in the sender's comm block.
struct PipeArgs {
    const float *src;               // send: the values
    float *dst;                     // recv: the values
    unsigned long long *recv;       // send: the receiver's buffer; recv: this rank's
    uint64_t n, half;               // values; pairs per half
    unsigned *epoch;                // this rank's epoch of the link (comm block)
    unsigned *ticket;               // this rank's ticket
    unsigned *ack;                  // send: this rank's ack word (written by the receiver);
                                    // recv: the sender's ack word (a peer address)
};
__global__ void pipe_send_kernel(const __grid_constant__ PipeArgs a);
__global__ void pipe_recv_kernel(const __grid_constant__ PipeArgs a);

// out = x + rs * add (the residual add of the last layer of a pipeline stage)
__global__ void residual_kernel(const float *x, const float *add, float rs, float *out, uint64_t n);

// The sliding-window KV shift (shift_kv, smollm_chat.rs:2942-2972): for
// layers [l0, l1) and kept positions i in [i0, i1), the K row at n_keep +
// n_discard + i is widened to f32, rotated by -n_discard (Rope::rotate,
// :1408-1419) and rounded back to f16 at n_keep + i; the V row is copied.
// Launches run in waves of at most n_discard rows, each reading only rows no
// earlier wave writes and writing only rows earlier waves have read.
struct KvShiftArgs {
    uint16_t *kc, *vc;          // the caches [n_layers][max_seq][kv_dim]
    const float *inv_freq;      // [head_dim / 2]
    uint32_t l0, l1, max_seq, kv_dim, head_dim, neox;
    uint32_t n_keep, n_discard, i0, i1;
};
__global__ void kv_shift_kernel(const __grid_constant__ KvShiftArgs a);

__global__ void embed_kernel(const __grid_constant__ EmbedArgs a);
__global__ void rmsnorm_kernel(const __grid_constant__ NormArgs a);
template <int HD>
__global__ void attention_batch_kernel(const __grid_constant__ AttnArgs a);
template <int HD, int CHK>
__global__ void attention_kernel(const __grid_constant__ AttnArgs a);
__global__ void argmax_kernel(const __grid_constant__ ArgmaxArgs a);
__global__ void rope_kv_batch_kernel(const __grid_constant__ RopeBatchArgs a);

}  // namespace sg
