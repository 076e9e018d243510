/*
 * spindle_gpu.h — C ABI of spindle-b200, the B200 (sm_100a) implementation of
 * spindle's quantized matvec path.
 *
 * The reference (WiseHax/spindle 1.1.0, Rust) has no plugin system: its drop-in
 * boundary is the crate-internal kernel API that the engine calls.  Each entry
 * point below replaces one of those functions; the comment names it by
 * file:line under the reference's src/.
 *
 * Conventions
 *   - Every function returns sg_status (0 = SG_OK) and never aborts the process.
 *   - Pointers named d_* are device pointers (cudaMalloc'd, or from sg_alloc);
 *     pointers named h_* are host pointers.  All memory is caller-owned unless
 *     an sg_* function allocated it.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls are
 *     asynchronous with respect to the host unless stated otherwise.
 *   - Weight tensors keep the GGUF byte layout verbatim: row r starts at
 *     d_base + m->offset + r * row_bytes(dtype, cols), and the tensor start
 *     must be 16-byte aligned (GGUF aligns tensors to 32 bytes).
 */
#ifndef SPINDLE_GPU_H
#define SPINDLE_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SG_API __attribute__((visibility("default")))
#else
#define SG_API
#endif

typedef int32_t sg_status;
#define SG_OK 0
#define SG_ERR_INVALID 1   /* null pointer, bad count or range */
#define SG_ERR_DTYPE 2     /* format not on this path (the reference panics, quant.rs:1092) */
#define SG_ERR_SHAPE 3     /* cols not a multiple of the block, or above SG_MAX_COLS */
#define SG_ERR_ALIGN 4     /* tensor start not 16-byte aligned */
#define SG_ERR_CUDA 5      /* a CUDA runtime call failed; see sg_last_error_string() */
#define SG_ERR_NCCL 6
#define SG_ERR_TIMEOUT 7   /* a bounded device-side wait gave up */
#define SG_ERR_NOMEM 8
#define SG_ERR_NOALLOC_LIMIT 9 /* request larger than the static scratch of sg_matvec_static */

/* GGML type ids (gguf_loader.rs:25-65). */
#define SG_F32 0
#define SG_F16 1
#define SG_Q8_0 8
#define SG_Q4_K 12
#define SG_Q6_K 14

/* Weight layouts (sg_mat.layout).  GGUF: the file's rows, verbatim.
 * TILED16: the same bytes permuted once at upload by sg_repack_tiled16 so that
 * the GEMV streams aligned 16-row tiles (see sg_repack_tiled16). */
#define SG_LAYOUT_GGUF 0
#define SG_LAYOUT_TILED16 1

/* Widest row the integer kernels take (256 super-blocks). */
#define SG_MAX_COLS 65536

/* A weight matrix inside a device buffer: quant.rs:914-935 `Mat`. */
typedef struct sg_mat {
    int32_t dtype;
    uint32_t layout; /* SG_LAYOUT_GGUF (0) or SG_LAYOUT_TILED16 */
    uint64_t offset; /* bytes from the base pointer to row 0 */
    uint64_t cols;
    uint64_t rows;
} sg_mat;

/* One Q8_K activation vector in device memory: quant_q8k.rs:61-65 `Q8K`.
 * d: n/256 floats, qs: n int8, bsums: n/16 int16. */
typedef struct sg_q8k {
    float *d;
    int8_t *qs;
    int16_t *bsums;
    uint64_t n;
} sg_q8k;

/* ---- status, formats, device memory ------------------------------------ */

SG_API const char *sg_status_string(sg_status s);
/* Text of the last CUDA error seen by this thread's calls. */
SG_API const char *sg_last_error_string(void);
/* quant.rs:1527-1542 `row_bytes`: SG_ERR_DTYPE / SG_ERR_SHAPE when undefined. */
SG_API sg_status sg_row_bytes(int32_t dtype, uint64_t cols, uint64_t *out);
/* quant_q8k.rs:55-57 `supports`: 1 when m runs on the integer kernels. */
SG_API int32_t sg_supports(const sg_mat *m);
/* quant_q8k.rs:22-24 `set_enabled` (the --float-kernels switch), process-wide. */
SG_API void sg_set_int_kernels(int32_t on);
SG_API int32_t sg_int_kernels_enabled(void);
/* Bytes of one Q8_K vector of n values (d + qs + bsums), and carving of a
 * 16-byte aligned buffer of that size into an sg_q8k. */
SG_API uint64_t sg_q8k_bytes(uint64_t n);
SG_API sg_status sg_q8k_view(void *d_buf, uint64_t n, sg_q8k *out);

/* Device memory helpers for callers without a CUDA binding.  sg_upload pads
 * the allocation to 256 bytes so that 16-byte bulk copies never leave it. */
SG_API sg_status sg_alloc(uint64_t bytes, void **d_out);
SG_API sg_status sg_free(void *d_ptr);
SG_API sg_status sg_upload(const void *h_src, uint64_t bytes, void **d_out);
SG_API sg_status sg_memcpy_h2d(void *d_dst, const void *h_src, uint64_t bytes, void *stream);
SG_API sg_status sg_memcpy_d2h(void *h_dst, const void *d_src, uint64_t bytes, void *stream);
SG_API sg_status sg_stream_sync(void *stream);
/* Reads and clears the device-side status word that bounded waits set. */
SG_API sg_status sg_device_status(void);

/* ---- integer path: quant_q8k.rs ------------------------------------------ */

/* Q8K::quantize (quant_q8k.rs:73-121) of n_vec vectors: vector b is read from
 * d_x + b*ldx and written to outs[b] (outs is a host array).  n % 256 == 0.
 * Bit-identical to the reference, including non-finite and all-zero blocks. */
SG_API sg_status sg_q8k_quantize(const float *d_x, uint64_t n, uint64_t n_vec, uint64_t ldx,
                          const sg_q8k *outs, void *stream);

/* quant_q8k::matmul_rows (quant_q8k.rs:255-295): rows r0..r1 of
 * outs[b] = W * xq[b] for b < n_vec; row r of vector b goes to outs[b][r]
 * (outs[b] points at the START of a full output).  xq and outs are host arrays
 * of device descriptors / pointers.  dtype Q4_K or Q6_K, cols % 256 == 0,
 * cols <= SG_MAX_COLS, either layout.  Bit-identical fp32 results to the
 * reference for any n_vec and any row split. */
SG_API sg_status sg_matmul_rows(const uint8_t *d_base, const sg_mat *m, const sg_q8k *xq,
                         float *const *outs, uint64_t n_vec, uint64_t r0, uint64_t r1,
                         void *stream);

/* TILED16 layout (no reference counterpart; the reference reads the mmap'd
 * GGUF rows).  Rows are grouped in tiles of 16; tile t stores super-block
 * column i of its 16 rows as aligned planes: Q4_K qs[16][128] then
 * head[16][16] (d, dmin, scales); Q6_K qlqh[16][192], scales[16][16], d[16][2].
 * The last tile is zero-padded.  Only bytes move: results are bit-identical
 * to the GGUF layout.  sg_tiled16_bytes gives the buffer size;
 * sg_repack_tiled16 / sg_unpack_tiled16 convert between the two layouts
 * (device buffers, no overlap). */
SG_API sg_status sg_tiled16_bytes(int32_t dtype, uint64_t rows, uint64_t cols, uint64_t *out);
SG_API sg_status sg_repack_tiled16(int32_t dtype, const uint8_t *d_gguf, uint64_t rows, uint64_t cols,
                                   uint8_t *d_tiled, void *stream);
SG_API sg_status sg_unpack_tiled16(int32_t dtype, const uint8_t *d_tiled, uint64_t rows, uint64_t cols,
                                   uint8_t *d_gguf, void *stream);

/* matvec / matvec_multi on the integer path (smollm_chat.rs:309-318 and
 * :447-512): out_b = W * x_b for b < n_vec, rows r0..r1, where x_b = d_x +
 * b*ldx holds cols fp32 values (16-byte aligned) and row r of out_b is
 * d_out[b*ldo + r].  The Q8_K quantization of x_b runs inside the GEMV kernel
 * (no scratch memory, one launch); the bits equal sg_q8k_quantize followed by
 * sg_matmul_rows.  TILED16 weights only (SG_ERR_INVALID for GGUF rows). */
SG_API sg_status sg_matvec(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                           uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, void *stream);

/* Several matvecs in one launch: entry j computes d_out[j][r] = W_j * x_j for
 * every row r of mats[j] (TILED16 Q4_K / Q6_K, based at d_base[j]), x_j =
 * d_x[j] holding cols_j fp32 values (16-byte aligned); d_base, mats, d_x and
 * d_out are host arrays of n <= SG_LIST_MAX entries.  The entries are
 * independent (no output may be another entry's input).  One persistent
 * kernel streams the matrices one after another without a launch boundary
 * between them (each warp's copies of the next matrix are in flight while it
 * finishes the current one); every output is bit for bit the one sg_matvec
 * writes for that entry (smollm_chat.rs:309-318 per entry). */
#define SG_LIST_MAX 16
SG_API sg_status sg_matvec_list(const uint8_t *const *d_base, const sg_mat *mats, const float *const *d_x,
                                float *const *d_out, uint64_t n, void *stream);

/* The same list with Q8_K activations (quant_q8k.rs:255-295 matmul_rows per
 * entry): entry j reads its vector as a Q8_K image d_img[j] made by
 * sg_q8k_images (or by any producer writing that layout), staged by one bulk
 * copy instead of being quantized in every CTA.  Bit for bit sg_matvec_list
 * on the vectors the images were made from. */
SG_API sg_status sg_matvec_list_q8k(const uint8_t *const *d_base, const sg_mat *mats, const uint8_t *const *d_img,
                                    float *const *d_out, uint64_t n, void *stream);

/* Q8_K image of a vector of cols fp32 values (Q8K::quantize, quant_q8k.rs:
 * 73-121, bit for bit): one buffer of sg_q8k_image_bytes(cols) bytes holding
 * qs[cols] (int8), then bsums[cols / 16] (int16), then d[cols / 256] (f32,
 * padded with zero bytes to a multiple of 16 bytes).  sg_q8k_images quantizes n <= SG_LIST_MAX
 * vectors (d_x[j]: cols[j] values, 16-byte aligned) into d_img[j] (16-byte
 * aligned) in one launch; host arrays of n entries.  0 for a cols that is not
 * a multiple of 256 in 256..SG_MAX_COLS. */
SG_API uint64_t sg_q8k_image_bytes(uint64_t cols);
SG_API sg_status sg_q8k_images(const float *const *d_x, const uint64_t *cols, uint8_t *const *d_img, uint64_t n,
                               void *stream);

/* Many vectors at once (matvec_multi, smollm_chat.rs:447-512, over
 * quant_q8k.rs:255-295 matmul_rows): the rows r0..r1 of a TILED16 Q4_K/Q6_K
 * matrix for n_vec <= SG_BATCH_MAX_VEC fp32 vectors (x_b = d_x + b*ldx),
 * out_b[r] = d_out[b*ldo + r]; each vector is quantized to Q8_K once and every
 * weight column is read once for all of them (one quantize launch plus one
 * GEMM launch).  Bit for bit the results of sg_matvec (and of the reference's
 * integer kernel).  Scratch: sg_matmul_batch_scratch_bytes(m, n_vec) device
 * bytes, 16-byte aligned, caller-owned; ldx % 4 == 0. */
#define SG_BATCH_MAX_VEC 128
SG_API uint64_t sg_matmul_batch_scratch_bytes(const sg_mat *m, uint64_t n_vec);
SG_API sg_status sg_matmul_batch(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                 float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                 void *d_scratch, uint64_t scratch_bytes, void *stream);

/* The float path (quant.rs:939-1094 matvec_rows_avx2; quant_multi.rs:232-273
 * matmul_rows_avx2), for formats or switches that keep a matrix off the integer
 * kernels: out_b[r] = d_out[b*ldo + r] for r in r0..r1, x_b = d_x + b*ldx (cols
 * fp32).  GGUF rows only, base + offset 16-byte aligned for Q4_K, 4 for F32,
 * 2 otherwise.  Formats: SG_F32, SG_F16 (any cols), SG_Q8_0 (cols % 32),
 * SG_Q4_K and SG_Q6_K (cols % 256), cols <= SG_MAX_COLS.
 * sg_matvec_rows_float runs every vector through matvec_rows_avx2 (the
 * single-vector algorithm; also what matvec_multi does for F32 matrices,
 * smollm_chat.rs:455-463).  sg_matmul_rows_float is matmul_rows_avx2: for
 * n_vec > 1 and a format with a shared-decode kernel (F32 cols % 8, Q8_0,
 * Q4_K, Q6_K) the rows_multi algorithm, whose bits differ from the
 * single-vector ones exactly as in the reference.  Both are bit-identical to
 * the reference (NaN payloads aside). */
SG_API sg_status sg_matvec_rows_float(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                      float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                      void *stream);
SG_API sg_status sg_matmul_rows_float(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                      float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                      void *stream);

/* ---- Row-split tensor parallelism over NVLink (one process per GPU) --------
 *
 * par_rows (smollm_chat.rs:332-337) splits a matvec's rows across threads;
 * sg_matvec_tp splits them across GPUs the same way (rank p of P owns rows
 * [R*p/P, R*(p+1)/P); results do not depend on the split, quant_q8k.rs:393-394)
 * and fuses the gather that follows into the same kernel: the GEMV epilogue
 * stores each row of its shard, tagged with the call's epoch, straight into
 * every rank's receive buffer (8-byte peer stores over NVLink through CUDA IPC
 * mappings; no copy kernel, no NCCL call, no memory fence), and each rank's
 * blocks then read their share of its own receive buffer, each row as soon as
 * it carries the epoch, into the plain output.  After the call every rank
 * holds the whole output.  Every rank must make the same sequence of calls
 * (the epoch counts them); a wait that runs out (2 s) writes NaN and makes
 * sg_device_status return SG_ERR_TIMEOUT.
 *
 * Set-up, per rank: a comm block of sg_tp_comm_bytes() (device memory, 256-byte
 * aligned, zeroed by sg_tp_comm_init), kept for all calls; per output, a
 * receive buffer of sg_tp_recv_bytes(n_vec, rows) (cudaMalloc / sg_alloc,
 * zeroed) shared with the other ranks through sg_ipc_get_handle /
 * sg_ipc_open (the handle is sg_ipc_handle_bytes() long; the exchange itself
 * is the caller's, e.g. an all-gather over its process group). */
#define SG_TP_MAX_RANKS 8
#define SG_TP_COMM_BYTES 256
typedef struct {
    uint32_t n_ranks, rank;
    void *recv[SG_TP_MAX_RANKS];   /* the output's receive buffer on every rank (this rank's own at [rank]) */
    void *comm;                    /* this rank's comm block */
} sg_tp_group;
SG_API uint64_t sg_ipc_handle_bytes(void);
SG_API sg_status sg_ipc_get_handle(void *d_ptr, void *handle_out);
SG_API sg_status sg_ipc_open(const void *handle, void **d_out);
SG_API sg_status sg_ipc_close(void *d_ptr);
SG_API uint64_t sg_tp_comm_bytes(void);
SG_API sg_status sg_tp_comm_init(void *d_comm, void *stream);
SG_API uint64_t sg_tp_recv_bytes(uint64_t n_vec, uint64_t rows);
/* This rank's shard (TILED16, m->rows rows = global rows row0 .. row0 +
 * m->rows of a rows-row matrix) times x_b (fp32, b < n_vec <= 8, 16-byte
 * aligned, ldx apart); afterwards d_out[b*ldo + r] = row r of W x_b for every
 * r < rows, on every rank. */
SG_API sg_status sg_matvec_tp(const uint8_t *d_shard, const sg_mat *m, const float *d_x, uint64_t ldx,
                              uint64_t n_vec, uint64_t row0, uint64_t rows, float *d_out, uint64_t ldo,
                              const sg_tp_group *grp, void *stream);

/* The same matvec for either layout with the Q8_K images in caller-owned
 * scratch (the reference keeps them in thread-local scratch, quant_q8k.rs:
 * 123-142): quantizes x_b into d_scratch (>= sg_matvec_scratch_bytes(cols,
 * n_vec) bytes, 16-byte aligned), then runs sg_matmul_rows on it.  Same bits
 * as sg_matvec. */
SG_API uint64_t sg_matvec_scratch_bytes(uint64_t cols, uint64_t n_vec);
SG_API sg_status sg_matvec_scratch(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                   float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                   void *d_scratch, uint64_t scratch_bytes, void *stream);

/* sg_matvec_scratch for callers that cannot allocate device memory (hosts
 * without their own CUDA allocator, or paths where a cudaMalloc would stall
 * the device).  No counterpart in the reference, whose scratch is ordinary
 * thread-local heap memory.  The Q8_K scratch is a static device array of
 * SG_NOALLOC_SCRATCH_BYTES bytes inside the library: requests needing more
 * (sg_matvec_scratch_bytes(cols, n_vec)) return SG_ERR_NOALLOC_LIMIT; it
 * allocates nothing.  The first call on a device (and the first after a
 * device reset) looks the array up: make it before any stream capture.  All
 * calls share the array, so calls that overlap on the GPU race and must be
 * serialized by the caller. */
#define SG_NOALLOC_SCRATCH_BYTES 262144
SG_API sg_status sg_matvec_static(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                  float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                  void *stream);

/* The int32 lane sums of rows<B,T> (quant_q8k.rs:235-242) for one vector, as
 * the kernel computes them: d_out[(r-r0)*nb*8 + i*8 + l] = lane l of block i
 * of row r.  Exists to check per-super-block sums bit for bit.  GGUF layout only. */
SG_API sg_status sg_block_sums(const uint8_t *d_base, const sg_mat *m, const sg_q8k *xq,
                        int32_t *d_out, uint64_t r0, uint64_t r1, void *stream);

/* The kernels' expf / sinf / cosf (fn 0 / 1 / 2): glibc's single-precision
 * functions, which f32::exp and f32::sin_cos call on Linux (smollm_chat.rs:
 * 586-588 SiLU, :1200-1203 router softmax, :1397-1420 RoPE, :3463-3495
 * attention), restated for the device.  d_out[i] = f(the float whose bits are
 * (start + i * stride) mod 2^32), i < count.  Exists to check the device build
 * against the host's libm. */
SG_API sg_status sg_libm_eval(int32_t fn, uint64_t start, uint64_t stride, uint64_t count, float *d_out,
                              void *stream);

/* The architecture the runtime loaded the library's kernels for, as
 * major * 10 + minor (cudaFuncAttributes.binaryVersion): 100 on B200 (the
 * library ships sm_100a code only).  No counterpart in the reference. */
SG_API sg_status sg_binary_version(int32_t *out);

/* ---- MoE layer (smollm_chat.rs:1178-1382, moe_forward with the fused expert
 * FFNs of ffns_fused, :382-442) ------------------------------------------------
 *
 * One token through a top-k MoE feed-forward layer, with the expert choice kept
 * on the device (no host round trip between router and experts):
 *   logits = router x (F32 rows, the float path's lane order);
 *   p = softmax(logits); top n_used by p (descending; equal p: lower index
 *   first); pruned by moe_prune; weight_i = norm ? p_i / sum(kept p) : p_i;
 *   out = sum_i weight_i * down_i(silu(gate_i x) * up_i x), in router order,
 *   plus the shared expert (times sigmoid(shared_gate . x) when given).
 * The expert matrices run on the integer path: x and each h are quantized to
 * Q8_K exactly as the reference does (dim and n_ff multiples of 256). */
#define SG_MOE_MAX_USED 16

/* The router's choice (device memory, written by sg_moe_forward). */
typedef struct {
    uint32_t n;                       /* experts kept after pruning */
    uint32_t pad_[3];
    int32_t id[SG_MOE_MAX_USED];      /* router order */
    float weight[SG_MOE_MAX_USED];
} sg_moe_choice;

/* Device weights of one MoE layer (struct Moe, smollm_chat.rs:152-167).
 * Expert e's gate and up (n_ff rows each, dim cols) are one TILED16 matrix of
 * 2 * n_ff rows at gate_up + e * gate_up_stride, interleaved in groups of 8:
 * rows 16q..16q+7 are gate rows 8q..8q+7 and rows 16q+8..16q+15 the up rows
 * 8q..8q+7, so that each 16-row tile yields 8 outputs of silu(gate) * up.  Its
 * down (dim rows, n_ff cols) is TILED16 at down + e * down_stride.
 * sg_moe_pack_gate_up and sg_moe_pack_down build both from the GGUF expert
 * tensors; the strides are sg_tiled16_bytes(dtype, 2 * n_ff, dim) and
 * sg_tiled16_bytes(dtype, dim, n_ff). */
typedef struct {
    const float *router;              /* F32 [n_expert][dim] (ffn_gate_inp) */
    const uint8_t *gate_up;
    const uint8_t *down;
    int32_t gate_up_dtype, down_dtype;    /* SG_Q4_K or SG_Q6_K */
    uint64_t gate_up_stride, down_stride;
    uint64_t dim, n_ff, n_expert, n_used;
    int32_t norm;                     /* expert_norm */
    float moe_prune;                  /* 0 = off; (0,1) = keep mass 1-prune; >= 1 = keep that many */
    /* Shared expert (Qwen2-MoE): NULL shared_gate_up = none. */
    const uint8_t *shared_gate_up;    /* TILED16 gate/up, interleaved as above, 2 * shared_n_ff rows */
    const uint8_t *shared_down;       /* TILED16, dim rows x shared_n_ff cols */
    int32_t shared_gate_up_dtype, shared_down_dtype;
    uint64_t shared_n_ff;
    const float *shared_gate;         /* F32 [dim] (ffn_gate_inp_shexp) or NULL */
} sg_moe;

/* Repack the GGUF expert tensors ffn_gate_exps and ffn_up_exps ([n_expert]
 * matrices of n_ff x dim, same dtype; n_ff a multiple of 8) into the
 * interleaved TILED16 form above. */
SG_API sg_status sg_moe_pack_gate_up(int32_t dtype, const uint8_t *d_gate_exps, const uint8_t *d_up_exps,
                                     uint64_t n_expert, uint64_t n_ff, uint64_t dim, uint8_t *d_out, void *stream);
/* Repack ffn_down_exps ([n_expert] matrices of dim x n_ff) into TILED16 per expert. */
SG_API sg_status sg_moe_pack_down(int32_t dtype, const uint8_t *d_down_exps, uint64_t n_expert, uint64_t dim,
                                  uint64_t n_ff, uint8_t *d_out, void *stream);
/* Device scratch that sg_moe_forward needs for this layer (0 for an invalid m). */
SG_API uint64_t sg_moe_scratch_bytes(const sg_moe *m);
/* out[dim] = moe_forward(x[dim]) (smollm_chat.rs:1178).  d_scratch: at least
 * sg_moe_scratch_bytes(m) bytes, 256-byte aligned, not shared with a call that
 * may overlap on the GPU.  d_choice and d_probs (float[n_expert], the softmax
 * probabilities) are optional outputs.  Four kernel launches, no host sync. */
SG_API sg_status sg_moe_forward(const sg_moe *m, const float *d_x, float *d_out, void *d_scratch,
                                uint64_t scratch_bytes, sg_moe_choice *d_choice, float *d_probs, void *stream);

/* moe_forward_batch (smollm_chat.rs:928-1174): n_tok tokens through the same
 * layer, out_t = moe_forward(x_t), bit for bit what n_tok one-token calls give
 * (the reference's batch is one-token-identical too, :4699-4736).  x_t =
 * d_x + t*ldx (16-byte aligned), out_t = d_out + t*ldo; n_tok <= 128 and
 * n_expert <= 256.  The router runs once over all tokens, one launch makes
 * every token's choice and a table of (expert, token) slots, and the gate/up
 * and down passes each run over all slots in one launch (each block stages
 * the Q8_K image of every token its slots use).  d_choices (optional,
 * [n_tok]) receives the choices. */
#define SG_MOE_MAX_BATCH 128
SG_API uint64_t sg_moe_batch_scratch_bytes(const sg_moe *m, uint64_t n_tok);
SG_API sg_status sg_moe_forward_batch(const sg_moe *m, const float *d_x, uint64_t ldx, uint64_t n_tok, float *d_out,
                                      uint64_t ldo, void *d_scratch, uint64_t scratch_bytes,
                                      sg_moe_choice *d_choices, void *stream);

/* Expert parallelism for the batched layer (experts shard across GPUs, the
 * router stays replicated): rank p keeps experts [expert_lo,
 * expert_hi) -- m->gate_up / m->down hold only those, packed as usual, while
 * m->router and m->n_expert stay whole -- and computes the choices of every
 * token (identically on every rank) but only the slots whose expert it owns.
 * The down pass stores each of those slot outputs, tagged with the call's
 * epoch, straight into every rank's receive buffer at the slot's place (8-byte
 * peer stores over NVLink, the protocol of sg_matvec_tp), and every rank's
 * combine sums all slots of a token in router order as they arrive: bit for
 * bit the one-GPU result.  Set-up per rank: a zeroed comm block
 * (sg_tp_comm_bytes, sg_tp_comm_init) and a zeroed receive buffer of
 * sg_moe_ep_recv_bytes(m, n_tok_max) bytes shared through sg_ipc_get_handle /
 * sg_ipc_open; every rank makes the same sequence of calls. */
typedef struct {
    uint32_t n_ranks, rank;
    uint64_t expert_lo, expert_hi;
    uint64_t recv_slots;                /* n_tok_max * n_used: the receive buffers' slots per half */
    void *recv[SG_TP_MAX_RANKS];        /* every rank's receive buffer (this rank's own at [rank]) */
    void *comm;                         /* this rank's comm block */
} sg_moe_ep;
SG_API uint64_t sg_moe_ep_recv_bytes(const sg_moe *m, uint64_t n_tok_max);
SG_API sg_status sg_moe_forward_batch_ep(const sg_moe *m, const sg_moe_ep *ep, const float *d_x, uint64_t ldx,
                                         uint64_t n_tok, float *d_out, uint64_t ldo, void *d_scratch,
                                         uint64_t scratch_bytes, sg_moe_choice *d_choices, void *stream);

/* ---- Decoder step (forward_slice, smollm_chat.rs:3371-3552, with greedy
 * sampling, :3565-3602 and :3661-3671) -----------------------------------------
 *
 * One token through every layer: embedding, then per layer RMSNorm, Q/K/V,
 * per-head Q/K norm, RoPE, the f16 KV cache, grouped-query attention, output
 * projection and residual, RMSNorm, dense SwiGLU FFN or MoE layer and residual;
 * then the output norm, the LM head and the greedy token.  The token and its
 * position are device state (int32 state[2] = {token, pos}); the step writes
 * the greedy token into state[0] and advances state[1], so a captured step can
 * be replayed token after token.  Matrices are TILED16; the GEMVs and expert
 * passes are the reference's bits, the rest matches within tolerance (see
 * spindle_b200/csrc/decode.cuh). */
typedef struct {
    const float *attn_norm, *ffn_norm;      /* F32 [dim] */
    const float *q_norm, *k_norm;           /* F32 [head_dim] (Qwen3 per-head norms), or NULL */
    const uint8_t *wq, *wk, *wv, *wo;       /* TILED16 */
    int32_t wq_dtype, wk_dtype, wv_dtype, wo_dtype;
    int32_t is_moe;
    sg_moe moe;                             /* when is_moe */
    const uint8_t *ffn_gate_up, *ffn_down;  /* dense FFN: one expert as sg_moe_pack_gate_up / _down pack it */
    int32_t ffn_gate_up_dtype, ffn_down_dtype;
    uint64_t n_ff;
} sg_layer;

typedef struct {
    uint32_t dim, n_heads, n_kv_heads, head_dim, n_layers, vocab, max_seq;
    int32_t rope_neox;                      /* NEOX pairs (i, i + head_dim/2), else (2i, 2i+1) */
    float rope_theta, rms_eps, residual_scale, embedding_scale;
    float attn_scale;                       /* 0: 1/sqrt(head_dim) */
    const uint8_t *embed;                   /* GGUF rows [vocab][dim]: F32, F16, Q4_K or Q6_K */
    int32_t embed_dtype;
    const uint8_t *lm_head;                 /* TILED16 [vocab][dim] */
    int32_t lm_head_dtype;
    const float *output_norm;               /* F32 [dim] */
    const sg_layer *layers;                 /* host array of n_layers */
} sg_model;

/* Device scratch of sg_forward (0 for an invalid model), and the f16 K and V
 * caches ([n_layers][max_seq][n_kv_heads * head_dim] each). */
SG_API uint64_t sg_model_scratch_bytes(const sg_model *m);
SG_API uint64_t sg_model_kv_bytes(const sg_model *m);
/* Fills the scratch's constant part (RoPE frequencies from the host's powf);
 * once per model and scratch, before sg_forward. */
SG_API sg_status sg_model_prepare(const sg_model *m, void *d_scratch, uint64_t scratch_bytes, void *stream);
/* One decoder step on the device state {token, pos}.  d_hidden (optional):
 * the output-normed hidden state [dim]; d_logits (optional): [vocab];
 * d_token (optional): the greedy token also as int64. */
SG_API sg_status sg_forward(const sg_model *m, int32_t *d_state, void *d_kv, void *d_scratch, uint64_t scratch_bytes,
                            float *d_hidden, float *d_logits, int64_t *d_token, void *stream);

/* The decoder step with expert parallelism (moe_forward under the layer split
 * of cluster_net.rs:776-795 and smollm_chat.rs:1178-1392, the experts spread
 * over GPUs instead of over PCs): every rank holds the whole model except the
 * experts -- each MoE layer's m->layers[l].moe keeps only this rank's experts
 * [eps[l].expert_lo, eps[l].expert_hi), packed, with the whole router and
 * n_expert -- and runs the same step on the same state.  Each MoE layer is
 * sg_moe_forward_batch_ep for one token: every rank computes the choice, runs
 * its own experts' slots and stores their outputs into every rank's receive
 * buffer over NVLink, and every rank sums them in router order, so every rank
 * ends the step with the same logits and greedy token as sg_forward on one
 * GPU, bit for bit.  eps: host array [n_layers] (entries of dense layers are
 * not read), each set up as for sg_moe_forward_batch_ep with n_tok_max >= 1.
 * Scratch: sg_model_ep_scratch_bytes(m) bytes, prepared by sg_model_prepare. */
SG_API uint64_t sg_model_ep_scratch_bytes(const sg_model *m);
SG_API sg_status sg_forward_ep(const sg_model *m, const sg_moe_ep *eps, int32_t *d_state, void *d_kv,
                               void *d_scratch, uint64_t scratch_bytes, float *d_hidden, float *d_logits,
                               int64_t *d_token, void *stream);

/* forward_batch_slice + compute_logits_batch (smollm_chat.rs:3146-3362,
 * :3591-3620): the n tokens d_tokens[0..n) at positions *d_pos .. *d_pos +
 * n - 1 (device int32, left unchanged; the caller advances it) through every
 * layer, each attending to every earlier position, its own batch included;
 * their K/V rows go into the caches.  Per token, bit for bit the one-token
 * sg_forward step at that position.  d_logits (optional): [n][ldl] floats;
 * d_greedy (optional): int64[n], each token's greedy next token.  Scratch:
 * sg_model_batch_scratch_bytes(m, n_max) bytes made ready once by
 * sg_model_batch_prepare; n <= n_max <= 128, feed's chunk (smollm_chat.rs:3090)
 * (MoE layers: n_expert <= 256). */
SG_API uint64_t sg_model_batch_scratch_bytes(const sg_model *m, uint64_t n_max);
SG_API sg_status sg_model_batch_prepare(const sg_model *m, uint64_t n_max, void *d_scratch, uint64_t scratch_bytes,
                                        void *stream);
SG_API sg_status sg_forward_batch(const sg_model *m, const int32_t *d_tokens, uint64_t n, const int32_t *d_pos,
                                  void *d_kv, void *d_scratch, uint64_t scratch_bytes, uint64_t n_max,
                                  float *d_logits, uint64_t ldl, int64_t *d_greedy, void *stream);

/* The sliding-window KV shift (shift_kv, smollm_chat.rs:2942-2972; the
 * policy, ensure_kv_room at :2924-2940, stays with the caller): drops
 * n_discard positions right after the n_keep pinned ones (at most cur_pos -
 * n_keep), moving positions [n_keep + n_discard, cur_pos) down to n_keep; each
 * moved K row is re-rotated by -n_discard (RoPE rotations compose) through f32
 * and back to f16, V rows are copied.  Layers [l0, l1) only (a pipeline stage
 * shifts its own).  d_scratch: sg_forward's scratch, prepared (its RoPE
 * frequencies).  The caller then continues at position cur_pos - n_discard. */
SG_API sg_status sg_kv_shift(const sg_model *m, void *d_kv, const void *d_scratch, uint32_t l0, uint32_t l1,
                             uint32_t n_keep, uint32_t n_discard, uint32_t cur_pos, void *stream);

/* The stages of a layer split over ranks (forward_slice with a layer range,
 * smollm_chat.rs:3371-3552; the two-PC split of docs/cluster.md): layers
 * [l0, l1) of sg_forward_batch.  l0 > 0: the input is d_hidden_in [n][dim],
 * the raw residual of the stage before (d_tokens unused); l1 < n_layers: the
 * output is the raw residual d_hidden_out [n][dim] (no output norm, no head,
 * d_logits / d_greedy unused).  l1 == n_layers: d_hidden_out (optional) gets
 * the output-normed hidden states [n][dim] (forward_batch_slice's return
 * value), and the LM head and argmax run only when d_logits or d_greedy is
 * given (a prompt fed through feed(), smollm_chat.rs:3042-3106, needs no
 * logits).  A stage's KV cache rows are its own layers'.
 * Continuing on one scratch: l1 < n_layers with d_hidden_out null leaves the
 * layers' state in d_scratch, and a following call with l0 equal to that l1,
 * d_hidden_in null, the same scratch, tokens and positions picks it up (so a
 * prompt can go through a layer at a time, e.g. two chunks on two streams,
 * without moving the residual); the results are those of one call. */
SG_API sg_status sg_forward_batch_range(const sg_model *m, uint32_t l0, uint32_t l1, const int32_t *d_tokens,
                                        const float *d_hidden_in, uint64_t n, const int32_t *d_pos, void *d_kv,
                                        void *d_scratch, uint64_t scratch_bytes, uint64_t n_max,
                                        float *d_hidden_out, float *d_logits, uint64_t ldl, int64_t *d_greedy,
                                        void *stream);
/* A one-way link between two ranks for the residual between stages (the STEP /
 * PREFILL frames of cluster_net.rs, over NVLink): sg_pipe_send stores n <=
 * n_max floats as epoch-tagged pairs into the receiver's buffer
 * (sg_pipe_recv_bytes(n_max), zeroed, IPC-shared), after the receiver has
 * taken the call two before (the buffer alternates halves); sg_pipe_recv waits
 * for them, writes them to d_dst and acknowledges to the sender (d_peer_comm:
 * the sender's comm block, IPC-mapped).  Each side has its own zeroed comm
 * block (sg_tp_comm_bytes) per link; both make the same sequence of calls;
 * waits are bounded (2 s, then SG_ERR_TIMEOUT from sg_device_status). */
SG_API uint64_t sg_pipe_recv_bytes(uint64_t n_max);
SG_API sg_status sg_pipe_send(const float *d_src, uint64_t n, uint64_t n_max, void *d_peer_recv, void *d_comm,
                              void *stream);
SG_API sg_status sg_pipe_recv(float *d_dst, uint64_t n, uint64_t n_max, void *d_recv, void *d_comm, void *d_peer_comm,
                              void *stream);

/* ---- the reference's synthetic benchmark kernels ----------------------------
 * Prototypes driven by the reference's early benchmark (main.rs), not by its
 * chat engine; fixed shapes (4096-wide rows of 16 Q4_K blocks, 8 experts, 32
 * query / 8 KV heads of 128, 32 layers, 512 positions); results bit for bit
 * the AVX2 kernels'. */
/* q4k_gemv_4row_avx2 (q4k_gemv.rs:183-226): rows of d_chunk[chunk_len] in
 * whole groups of four (*rows_done, optional, host), y[(row_offset + r) &
 * 4095] += the row's dot with x (float [4096]); weights' d / dmin decoded by
 * the module's own f16 conversion (q4k_gemv.rs:37-68, exponents clamped). */
SG_API sg_status sg_q4k_gemv_4row(const uint8_t *d_chunk, uint64_t chunk_len, const float *d_x, float *d_y,
                                  uint64_t row_offset, uint64_t *rows_done, void *stream);
/* q4k_gemm_spec4_slice_avx2 (q4k_gemv.rs:361-403): rows [r0, r1) against four
 * vectors x4 [4][4096], y4[k][(base + r) & 4095] += each row's dot. */
SG_API sg_status sg_q4k_gemm_spec4(const uint8_t *d_chunk, uint64_t r0, uint64_t r1, const float *d_x4,
                                   float *d_y4, uint64_t base, void *stream);
/* route_moe_top2 (moe_engine.rs:124-164): the top 2 of 8 experts for x
 * [4096] against gates [8][4096] (every 16th element), softmax weights. */
SG_API sg_status sg_route_moe_top2(const float *d_x, const float *d_gates, uint64_t layer, int32_t *d_experts,
                                   float *d_weights, void *stream);
/* flash_decoding_gqa_spec4_avx2 (transformer.rs:541-600) on q_spec [4][4096]
 * (replaced by the attention output) and the int8 KV cache of
 * QuantizedKvCache (k, v: [32][512][1024] int8; ks, vs: [32][512][8] f32):
 * the four tokens' K/V rows appended at seq_len (clamped to 508), then
 * online-softmax attention over positions 0..seq_len + k. */
SG_API sg_status sg_flash_gqa_spec4(float *d_q_spec, int8_t *d_kq, int8_t *d_vq, float *d_ks, float *d_vs,
                                    uint64_t seq_len, uint64_t layer, void *stream);

/* ---- weight quantizer (no reference counterpart: its tests use random bytes)
 * f32 [rows, cols] -> Q4_K or Q6_K rows, deterministic; cols % 256 == 0. */
SG_API sg_status sg_quantize_weights(int32_t dtype, const float *d_w, uint64_t rows, uint64_t cols,
                              uint8_t *d_out, void *stream);

#ifdef __cplusplus
}
#endif
#endif
