/*
 * sg_oracle.h — CPU restatement of spindle's quantized matvec path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the CUDA path is
 * compared against (tests/, __graft_entry__.smoke()) and the CPU baseline that
 * bench.py times.  The product (spindle_b200/) never links or calls it.
 *
 * Every function restates one piece of the reference Rust crate (WiseHax/spindle
 * 1.1.0, src/...) with the same arithmetic in the same order, so that its fp32
 * results are bit-identical to the reference's AVX2 code:
 *   - the x86 AVX2/FMA/F16C operations are the same instructions the reference's
 *     `std::arch` intrinsics lower to;
 *   - the file is compiled with -ffp-contract=off (rustc never fuses a*b+c; gcc
 *     would), so every FMA here is an explicit one.
 *
 * Parity anchoring: the reference ships no golden vectors or fixture files.  The
 * oracle is checked against every known-answer comparator its tests hold for
 * this path (tests/test_oracle.py ports them: quant_q8k.rs:343-442,
 * quant.rs:1728-1771, quant_multi.rs:372-417), using the same seeded generators.
 */
#ifndef SG_ORACLE_H
#define SG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, gguf_loader.rs:25-65. */
enum {
    OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7,
    OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14, OR_BF16 = 30
};

/* quant.rs:914-935 `Mat`. */
typedef struct {
    int32_t dtype;
    uint32_t _pad;
    uint64_t offset;
    uint64_t cols;
    uint64_t rows;
} or_mat;

/* ---- test-input generators (quant_q8k.rs:302-336, quant.rs:1666-1723) ---- */
uint64_t or_rng_next(uint64_t *state);
float or_rng_f(uint64_t *state, float lo, float hi);
void or_rng_fill_f32(uint64_t *state, float lo, float hi, float *out, size_t n);
uint16_t or_f16_trunc(float v);        /* quant_q8k.rs:315-321 */
uint16_t or_f16_trunc_flush(float v);  /* quant.rs:1680-1690 */
/* quant_q8k.rs:323-336 (Q4_K, Q6_K) and quant_multi.rs:301-322 (Q8_0, F32). */
int or_random_matrix(int32_t dtype, size_t cols, size_t rows, uint64_t *rng, uint8_t *out);
/* quant.rs:1693-1723 (every format of the float test). */
int or_random_row(int32_t dtype, size_t cols, uint64_t *rng, uint8_t *out);

/* ---- formats (quant.rs:877-899, :1527-1660, q4k_gemv.rs:75-85) ---- */
int64_t or_row_bytes(int32_t dtype, uint64_t cols);
float or_f16_to_f32(uint16_t h);
void or_unpack_q4k_scales(const uint8_t sc12[12], uint8_t sc[8], uint8_t mn[8]);
int or_dequant_row(int32_t dtype, const uint8_t *row, size_t cols, float *out);

/* ---- the build's own f32 -> K-quant weight quantizer (kquant.c) ---- */
void or_quantize_q4k(const float *x, size_t n, uint8_t *out);
void or_quantize_q6k(const float *x, size_t n, uint8_t *out);

/* ---- integer path (quant_q8k.rs) ---- */
/* Q8K::quantize, quant_q8k.rs:73-121.  n % 256 == 0. */
void or_q8k_quantize(const float *x, size_t n, float *d, int8_t *qs, int16_t *bsums);
/* matmul_rows, quant_q8k.rs:255-295.  Vector b: xd[b] (n/256 floats),
 * xs[b] (n int8), xb[b] (n/16 int16); row r of vector b -> outs[b][r]. */
int or_matmul_rows(const uint8_t *base, const or_mat *m, size_t n_vec,
                   const float *const *xd, const int8_t *const *xs,
                   const int16_t *const *xb, float *const *outs,
                   size_t r0, size_t r1);
/* The int32 lane sums of rows<B,T> (quant_q8k.rs:235-242) for one vector:
 * out[(r - r0) * nb * 8 + i * 8 + l] = lane l of `sumi` for block i of row r. */
int or_block_sums(const uint8_t *base, const or_mat *m, const int8_t *xs,
                  size_t r0, size_t r1, int32_t *out);

/* ---- float path (quant.rs:939-1094, quant_multi.rs:232-273) ---- */
/* matvec_rows_avx2: rows r0..r0+n_rows of W*x -> out[0..n_rows]. */
int or_matvec_rows(const uint8_t *base, const or_mat *m, const float *x,
                   float *out, size_t r0, size_t n_rows);
/* quant_multi::matmul_rows_avx2: rows r0..r1 of W*xs[b] -> outs[b][r]. */
int or_matmul_rows_multi(const uint8_t *base, const or_mat *m, size_t n_vec,
                         const float *const *xs, float *const *outs,
                         size_t r0, size_t r1);

/* ---- FFN / MoE layer (smollm_chat.rs:382-442, :1178-1392) ---- */
typedef struct {
    or_mat router;           /* F32, rows = n_expert, cols = dim */
    or_mat gate, up, down;   /* expert 0; expert e starts e * rows * row_bytes later */
    uint32_t n_expert, n_used;
    int32_t norm;
    float moe_prune;
    int32_t has_shared, has_shared_gate;
    or_mat sh_gate, sh_up, sh_down;
    uint64_t shared_gate_offset; /* F32[dim] */
} or_moe;
int or_ffns_fused(const uint8_t *base, const or_mat *gate, const or_mat *up, const or_mat *down,
                  const float *weights, size_t k, const float *x, float *out, int int_on);
/* Router, softmax, top-k and prune: probs[n_expert], then the chosen experts
 * in order with their weights. */
int or_moe_route(const uint8_t *base, const or_moe *m, const float *x, float *probs, int32_t *chosen,
                 float *weights, uint32_t *n_chosen);
int or_moe_forward(const uint8_t *base, const or_moe *m, const float *x, float *out, int int_on,
                   int32_t *chosen_out, float *weights_out, uint32_t *n_chosen_out);

/* ---- worker pool (worker_pool.rs:38-139, smollm_chat.rs:309-349) ---- */
/* matvec / matvec_multi on the integer kernels with the reference's row split
 * [R*t/T, R*(t+1)/T) over n_threads persistent spinning workers.  xs is
 * n_vec x cols (row-major), outs is n_vec x rows.  Quantizes inside. */
int or_pool_create(int n_threads);
void or_pool_destroy(void);
int or_pool_threads(void);
int or_pool_matvec_multi(const uint8_t *base, const or_mat *m, size_t n_vec,
                         const float *xs, float *outs);

int or_cpu_has_avx2(void);

/* ---- decoder forward pass (smollm_chat.rs:3371-3552 forward_slice,
 * :569-584 rmsnorm, :1397-1420 Rope, :3565-3602 greedy sampling) ---- */
float or_dot_f16_row(const uint8_t *row, const float *x, size_t n);
typedef struct {
    uint64_t attn_norm, ffn_norm;   /* F32[dim] offsets */
    uint64_t q_norm, k_norm;        /* F32[head_dim] offsets, or UINT64_MAX when absent */
    or_mat wq, wk, wv, wo;
    int32_t is_moe;
    or_moe moe;                     /* is_moe */
    or_mat gate, up, down;          /* dense SwiGLU FFN */
} or_layer;
typedef struct {
    uint32_t dim, n_heads, n_kv_heads, head_dim, n_layers, vocab, max_seq;
    int32_t rope_neox;
    float rope_theta, rms_eps, residual_scale, embedding_scale;
    float attn_scale;               /* 0: 1/sqrt(head_dim) */
    or_mat embed, lm_head;
    uint64_t output_norm;           /* F32[dim] */
    const or_layer *layers;         /* n_layers */
} or_model;
/* rmsnorm: out[i] = (x[i] * inv) * w[i], inv = 1 / sqrt(sum of squares / n + eps). */
void or_rmsnorm(const float *x, const float *w, float *out, size_t n, float eps);
/* Rope inverse frequencies 1 / theta^(2i / head_dim), i < head_dim / 2. */
void or_rope_freqs(float theta, uint32_t head_dim, float *inv_freq);
/* Rope::rotate: every head of v (len values) rotated to position pos. */
void or_rope_rotate(float *v, size_t len, uint32_t head_dim, const float *inv_freq, int neox, float pos);
/* shift_kv (smollm_chat.rs:2942-2972) over layers [l0, l1); returns the new position. */
uint32_t or_kv_shift(const or_model *m, uint16_t *kcache, uint16_t *vcache, uint32_t l0, uint32_t l1, uint32_t n_keep,
                     uint32_t n_discard, uint32_t cur_pos);
/* One token at position pos through every layer: the KV caches (f16,
 * [n_layers][max_seq][n_kv_heads * head_dim]) get this position's K and V;
 * hidden_out (optional) = the output-normed hidden state, logits_out
 * (optional) = the LM head on it.  int_on selects the integer kernels. */
int or_forward(const uint8_t *base, const or_model *m, uint16_t *kcache, uint16_t *vcache, int64_t token,
               const float *in_hidden, uint32_t pos, int int_on, float *hidden_out, float *logits_out);
/* Greedy choice: the index of the largest logit under f32::total_cmp, the
 * last one on ties (Iterator::max_by). */
int64_t or_argmax(const float *logits, size_t n);

/* exp / sin / cos of the restatements (libm.c): the host's glibc expf / sinf /
 * cosf, what f32::exp / sin / cos call on Linux. */
float or_expf(float x);
float or_sinf(float x);
float or_cosf(float x);

/* The reference's synthetic benchmark kernels (synth.c): q4k_gemv.rs,
 * moe_engine.rs route_moe_top2, transformer.rs flash decoding. */
float or_synth_f16(uint16_t h);
float or_q4k_block_dot(const uint8_t *blk, const float *act);
uint64_t or_q4k_gemv_4row(const uint8_t *chunk, uint64_t chunk_len, const float *x, float *y, uint64_t row_offset);
void or_q4k_gemm_spec4(const uint8_t *chunk, uint64_t r0, uint64_t r1, const float *x4, float *y4, uint64_t base);
void or_route_moe_top2(const float *x, const float *gates, uint64_t layer, int32_t *experts, float *weights);
void or_kvcache_init(int8_t *k, int8_t *v, float *ks, float *vs, uint64_t init_ctx);
void or_flash_gqa_spec4(float *q_spec, int8_t *kq, int8_t *vq, float *ks, float *vs, uint64_t seq_len,
                        uint64_t layer);

#ifdef __cplusplus
}
#endif
#endif
