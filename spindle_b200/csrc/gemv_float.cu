// gemv_float.cu — float matvec kernels on GGUF rows (see gemv_float.cuh).
#include "gemv_float.cuh"
#include "tiled_block.cuh"

namespace sg {
using namespace tiled;

namespace {

// Byte k of word as an exact float: 2^23 + byte, minus 2^23 (no I2F).
__device__ __forceinline__ float byte_f(uint32_t word, uint32_t k) {
    return __fsub_rn(__int_as_float(__byte_perm(word, 0x4B000000u, 0x7440u | k)), 8388608.0f);
}
// Byte k as a signed int8.
__device__ __forceinline__ float sbyte_f(uint32_t word, uint32_t k) {
    return __fsub_rn(__int_as_float(__byte_perm(word ^ 0x80808080u, 0x4B000000u, 0x7440u | k)), 8388736.0f);
}
// Byte k (a 6-bit Q6_K code) minus 32.
__device__ __forceinline__ float q6_f(uint32_t word, uint32_t k) {
    return __fsub_rn(__int_as_float(__byte_perm(word, 0x4B000000u, 0x7440u | k)), 8388640.0f);
}

__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }

// Loads through generic pointers (global or shared memory): a 2-byte value,
// and bytes l, 8+l, 16+l, 24+l of the 32-byte span at p packed into one word
// (the four values AVX lane l of the reference takes from such a span).
__device__ __forceinline__ uint32_t gu16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
__device__ __forceinline__ uint32_t gld4(const uint8_t *p, uint32_t l) {
    return (uint32_t)p[l] | ((uint32_t)p[8 + l] << 8) | ((uint32_t)p[16 + l] << 16) | ((uint32_t)p[24 + l] << 24);
}

// Stage the next `pieces` 16-byte pieces of this row (from rp) into dst:
// thread l of the row's 8 takes pieces l, l + 8, ...; P pieces per thread at most.
template <int P>
__device__ __forceinline__ void stage_row(const uint8_t *rp, uint8_t *dst, uint32_t pieces, uint32_t l) {
    uint4 v[P];
#pragma unroll
    for (int p = 0; p < P; p++)
        if (l + 8u * p < pieces) v[p] = __ldg(reinterpret_cast<const uint4 *>(rp) + l + 8u * p);
#pragma unroll
    for (int p = 0; p < P; p++)
        if (l + 8u * p < pieces) reinterpret_cast<uint4 *>(dst)[l + 8u * p] = v[p];
}

// The same as asynchronous copies (cp.async, 16 bytes each, L2 only), so
// that a row's next span lands while the current one is used: the issuing
// thread's copies are complete after cp_wait<N> (N later groups may still be
// in flight), and a __syncwarp then shows them to the row's other threads.
template <int P>
__device__ __forceinline__ void stage_row_async(const uint8_t *rp, uint8_t *dst, uint32_t pieces, uint32_t l) {
#pragma unroll
    for (int p = 0; p < P; p++)
        if (l + 8u * p < pieces)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + 16u * (l + 8u * p))),
                         "l"(rp + 16u * (l + 8u * p))
                         : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// x: global memory or the CTA's shared copy (a generic load serves both)
__device__ __forceinline__ float xld(const float *p) { return *p; }

// hsum_avx2 (quant.rs:903-908) over the 8 lanes of a row group:
// ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)); every lane gets the sum.
__device__ __forceinline__ float hsum_hadd8(float v) {
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// hsum of quant_multi.rs:35-40: ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).
__device__ __forceinline__ float hsum_shuf8(float v) {
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
}

// unpack_q4k_scales (q4k_gemv.rs:75-85) from the 12 scale bytes s0..s2.
__device__ __forceinline__ void q4k_scales(uint32_t s0, uint32_t s1, uint32_t s2, float sc[8], float mn[8]) {
    const uint32_t s[3] = {s0, s1, s2};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        auto byte = [&](int i) { return (s[i >> 2] >> (8 * (i & 3))) & 0xFFu; };
        uint32_t a, m;
        if (j < 4) {
            a = byte(j) & 63u;
            m = byte(j + 4) & 63u;
        } else {
            a = (byte(j + 4) & 0xFu) | ((byte(j - 4) >> 6) << 4);
            m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
        }
        sc[j] = (float)a;
        mn[j] = (float)m;
    }
}

template <int DT>
__device__ __forceinline__ float wload(const uint8_t *row, uint32_t j) {
    if constexpr (DT == FDT_F32) return __ldg(reinterpret_cast<const float *>(row) + j);
    else return h2f(__ldg(reinterpret_cast<const unsigned short *>(row) + j));
}

}  // namespace

template <int DT, int NV, bool MULTI>
__global__ void __launch_bounds__(FGEMV_THREADS, NV == 1 && !MULTI ? 3 : 1) gemv_float_kernel(const __grid_constant__ FGemvArgs a) {
    extern __shared__ __align__(16) float fsums[];
    grid_dependency_wait();
    const uint32_t l = threadIdx.x & 7u, n = a.n, nv = a.nvec;
    uint32_t row = a.r0 + blockIdx.x * FGEMV_ROWS + (threadIdx.x >> 3);
    const bool valid = row < a.r1;
    if (!valid) row = a.r1 - 1;  // computes a real row, writes nothing
    const float *xv[NV];
#pragma unroll
    for (int b = 0; b < NV; b++) xv[b] = a.x + (uint64_t)((uint32_t)b < nv ? b : 0) * a.ldx;
    if (a.stage_x) {
        // one vector: x is read by every row of the CTA, so it is copied once
        // into shared memory (after the Q4_K sub-block sums' area)
        float *xs = fsums + fgemv_presum_floats(DT, MULTI, nv, n);
        for (uint32_t i = threadIdx.x; i < n / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(xs)[i] = __ldg(reinterpret_cast<const float4 *>(a.x) + i);
        __syncthreads();
        xv[0] = xs;
    }
    const uint8_t *rp = a.w + (uint64_t)row * a.row_bytes;
    float acc[NV], acc1[NV], extra[NV];
#pragma unroll
    for (int b = 0; b < NV; b++) acc[b] = acc1[b] = extra[b] = 0.0f;

    if constexpr (DT == FDT_F32 || DT == FDT_F16) {
        if constexpr (!MULTI) {
            // dot_f32_avx2 / dot_f16_row_avx2 (quant.rs:863-874, :1412-1425)
            const uint32_t steps = n / 8;
            // one vector: more steps' weights in flight per thread (2-byte loads)
            constexpr uint32_t U = NV == 1 ? 32 : 8;
            uint32_t i = 0;
            // With 16-byte aligned rows the weights move in 64-element spans:
            // each thread of the row's 8 loads 16 bytes (a span of F16, half
            // of one of F32), QS spans at a time, into this warp's part of
            // shared memory; lane l then reads elements l, l+8, ... of each
            // span from there, so the FMA chain is unchanged.
            // (two buffers of QS spans: the next QS spans are copied in
            // asynchronously while the current ones are used)
            constexpr uint32_t EB = DT == FDT_F32 ? 4u : 2u, SPAN_B = 64u * EB, RSTR = SPAN_B + 16u,
                           QS = NV <= 2 ? (DT == FDT_F16 ? 4u : 2u) : 1u;
            __shared__ __align__(16) uint8_t wsm[2][FGEMV_THREADS / 32][QS][4][RSTR];
            const bool vec = ((reinterpret_cast<uintptr_t>(a.w) | a.row_bytes) & 15u) == 0;
            if (vec) {
                const uint32_t rw = (threadIdx.x >> 3) & 3u, wp = threadIdx.x >> 5, nit = steps / (8 * QS);
                auto issue = [&](uint32_t it) {
                    if (it < nit)
#pragma unroll
                        for (uint32_t u = 0; u < QS; u++)
                            stage_row_async<SPAN_B / 128>(rp + (uint64_t)(64 * QS * it + 64 * u) * EB,
                                                          &wsm[it & 1u][wp][u][rw][0], SPAN_B / 16, l);
                    cp_commit();
                };
                issue(0);
                for (uint32_t it = 0; it < nit; it++, i += 8 * QS) {
                    issue(it + 1);
                    cp_wait<1>();
                    __syncwarp();
                    const uint32_t bf = it & 1u;
#pragma unroll
                    for (uint32_t u = 0; u < QS; u++)
#pragma unroll
                        for (uint32_t j = 0; j < 8; j++) {
                            const uint32_t e = 8 * j + l;  // element of the span
                            const float w = DT == FDT_F32 ? *reinterpret_cast<const float *>(&wsm[bf][wp][u][rw][4 * e])
                                                          : h2f(*reinterpret_cast<const unsigned short *>(&wsm[bf][wp][u][rw][2 * e]));
#pragma unroll
                            for (int b = 0; b < NV; b++)
                                if ((uint32_t)b < nv) acc[b] = __fmaf_rn(w, xld(xv[b] + 8 * (i + 8 * u + j) + l), acc[b]);
                        }
                    __syncwarp();  // done with this buffer before it is refilled
                }
            }
            for (; i + U <= steps; i += U) {
                float wv[U];
#pragma unroll
                for (uint32_t u = 0; u < U; u++) wv[u] = wload<DT>(rp, 8 * (i + u) + l);
#pragma unroll
                for (uint32_t u = 0; u < U; u++)
#pragma unroll
                    for (int b = 0; b < NV; b++)
                        if ((uint32_t)b < nv) acc[b] = __fmaf_rn(wv[u], xld(xv[b] + 8 * (i + u) + l), acc[b]);
            }
            for (; i < steps; i++) {
                const float w = wload<DT>(rp, 8 * i + l);
#pragma unroll
                for (int b = 0; b < NV; b++)
                    if ((uint32_t)b < nv) acc[b] = __fmaf_rn(w, xld(xv[b] + 8 * i + l), acc[b]);
            }
            for (uint32_t j = steps * 8; j < n; j++) {  // scalar tail, every lane alike
                const float w = wload<DT>(rp, j);
#pragma unroll
                for (int b = 0; b < NV; b++)
                    if ((uint32_t)b < nv) extra[b] = __fadd_rn(extra[b], __fmul_rn(w, xld(xv[b] + j)));
            }
        } else {
            // rows_multi F32 arm (quant_multi.rs:139-157): n % 8 == 0
            uint32_t j = 0;
#pragma unroll 4
            for (; j + 16 <= n; j += 16) {
                const float w0 = wload<DT>(rp, j + l), w1 = wload<DT>(rp, j + 8 + l);
#pragma unroll
                for (int b = 0; b < NV; b++)
                    if ((uint32_t)b < nv) {
                        acc[b] = __fmaf_rn(w0, xld(xv[b] + j + l), acc[b]);
                        acc1[b] = __fmaf_rn(w1, xld(xv[b] + j + 8 + l), acc1[b]);
                    }
            }
            if (j < n) {
                const float w0 = wload<DT>(rp, j + l);
#pragma unroll
                for (int b = 0; b < NV; b++)
                    if ((uint32_t)b < nv) acc[b] = __fmaf_rn(w0, xld(xv[b] + j + l), acc[b]);
            }
        }
    } else if constexpr (DT == FDT_Q8_0) {
        // dot_q8_0_row_avx2 (quant.rs:51-71) / rows_multi Q8_0 arm (quant_multi.rs:158-176)
        const uint32_t nbk = n / 32;
        // block k at bp (global or shared memory)
        auto q8_block = [&](const uint8_t *bp, uint32_t k) {
            const float d = h2f(gu16(bp));
            const uint32_t qw = gld4(bp + 2, l);
            float q[4];
#pragma unroll
            for (uint32_t i = 0; i < 4; i++) q[i] = sbyte_f(qw, i);
#pragma unroll
            for (int b = 0; b < NV; b++)
                if ((uint32_t)b < nv) {
                    const float *xb = xv[b] + 32 * k + l;
                    float s = __fmaf_rn(q[0], xld(xb), 0.0f);
#pragma unroll
                    for (uint32_t i = 1; i < 4; i++) s = __fmaf_rn(q[i], xld(xb + 8 * i), s);
                    if (MULTI && (k & 1u)) acc1[b] = __fmaf_rn(d, s, acc1[b]);
                    else acc[b] = __fmaf_rn(d, s, acc[b]);
                }
        };
        uint32_t k = 0;
        // 16-byte aligned rows: spans of 8 blocks (272 bytes = 17 pieces), two
        // at a time, staged through this warp's part of shared memory
        // (two buffers: the next two spans are copied in asynchronously
        // while the current two are used)
        constexpr uint32_t KB = 8, SB = KB * 34, SP = SB / 16;
        __shared__ __align__(16) uint8_t qsm[2][FGEMV_THREADS / 32][2][4][SB + 16];
        if (((reinterpret_cast<uintptr_t>(a.w) | a.row_bytes) & 15u) == 0) {
            const uint32_t rw = (threadIdx.x >> 3) & 3u, wp = threadIdx.x >> 5, nit = nbk / (2 * KB);
            auto issue = [&](uint32_t it) {
                if (it < nit) {
                    stage_row_async<3>(rp + 34 * (2 * KB * it), qsm[it & 1u][wp][0][rw], SP, l);
                    stage_row_async<3>(rp + 34 * (2 * KB * it + KB), qsm[it & 1u][wp][1][rw], SP, l);
                }
                cp_commit();
            };
            issue(0);
            for (uint32_t it = 0; it < nit; it++, k += 2 * KB) {
                issue(it + 1);
                cp_wait<1>();
                __syncwarp();
#pragma unroll 4
                for (uint32_t kk = 0; kk < 2 * KB; kk++)
                    q8_block(&qsm[it & 1u][wp][kk / KB][rw][34 * (kk % KB)], k + kk);
                __syncwarp();  // done with this buffer before it is refilled
            }
        }
        for (; k < nbk; k++) q8_block(rp + k * 34, k);
    } else if constexpr (DT == FDT_Q4_K) {
        const uint32_t nbk = n / 256, ns = n / 32;
        if constexpr (!MULTI) {
            // compute_subblock_sums_32 (quant.rs:167-178) of every vector, once per CTA
            for (uint32_t i = threadIdx.x; i < nv * ns; i += blockDim.x) {
                const uint32_t b = i / ns, sb = i - b * ns;
                const float *p = a.x + (uint64_t)b * a.ldx + 32u * sb;
                float u[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    u[j] = __fadd_rn(__fadd_rn(p[j], p[8 + j]), __fadd_rn(p[16 + j], p[24 + j]));
                fsums[i] = __fadd_rn(__fadd_rn(__fadd_rn(u[0], u[4]), __fadd_rn(u[1], u[5])),
                                     __fadd_rn(__fadd_rn(u[2], u[6]), __fadd_rn(u[3], u[7])));
            }
            __syncthreads();
        }
        // block k at bp (global or shared memory)
        auto q4_block = [&](const uint8_t *bp, uint32_t k) {
            const uint4 hd = *reinterpret_cast<const uint4 *>(bp);
            const float d = h2f(hd.x & 0xFFFFu), dmin = h2f(hd.x >> 16);
            float sc[8], mn[8];
            q4k_scales(hd.y, hd.z, hd.w, sc, mn);
            uint32_t lo[4], hi[4];
#pragma unroll
            for (uint32_t c = 0; c < 4; c++) {
                const uint32_t qw = gld4(bp + 16 + 32 * c, l);
                lo[c] = qw & 0x0F0F0F0Fu;
                hi[c] = (qw >> 4) & 0x0F0F0F0Fu;
            }
            if constexpr (!MULTI) {
                // dot_q4_k_row_avx2_presum (quant.rs:250-290)
#pragma unroll
                for (int b = 0; b < NV; b++)
                    if ((uint32_t)b < nv) {
                        const float *sm = fsums + b * ns + 8 * k;
                        float mt = 0.0f;
#pragma unroll
                        for (int j = 0; j < 8; j++) mt = __fadd_rn(mt, __fmul_rn(mn[j], sm[j]));
                        extra[b] = __fadd_rn(extra[b], __fmul_rn(mt, dmin));
                    }
#pragma unroll
                for (uint32_t c = 0; c < 4; c++) {
                    const float ds0 = __fmul_rn(d, sc[2 * c]), ds1 = __fmul_rn(d, sc[2 * c + 1]);
#pragma unroll
                    for (int b = 0; b < NV; b++)
                        if ((uint32_t)b < nv) {
                            const float *xb = xv[b] + 256 * k + 64 * c + l;
                            float s = __fmaf_rn(byte_f(lo[c], 0), xld(xb), 0.0f);
                            s = __fmaf_rn(byte_f(lo[c], 1), xld(xb + 8), s);
                            s = __fmaf_rn(byte_f(lo[c], 2), xld(xb + 16), s);
                            s = __fmaf_rn(byte_f(lo[c], 3), xld(xb + 24), s);
                            acc[b] = __fmaf_rn(ds0, s, acc[b]);
                            s = __fmaf_rn(byte_f(hi[c], 0), xld(xb + 32), 0.0f);
                            s = __fmaf_rn(byte_f(hi[c], 1), xld(xb + 40), s);
                            s = __fmaf_rn(byte_f(hi[c], 2), xld(xb + 48), s);
                            s = __fmaf_rn(byte_f(hi[c], 3), xld(xb + 56), s);
                            acc[b] = __fmaf_rn(ds1, s, acc[b]);
                        }
                }
            } else {
                // deq_q4k (quant_multi.rs:55-72), then the a0/a1 chains
#pragma unroll
                for (uint32_t c = 0; c < 4; c++) {
                    const float s0 = __fmul_rn(d, sc[2 * c]), o0 = __fmul_rn(dmin, mn[2 * c]);
                    const float s1 = __fmul_rn(d, sc[2 * c + 1]), o1 = __fmul_rn(dmin, mn[2 * c + 1]);
                    float w[8];
#pragma unroll
                    for (uint32_t i = 0; i < 4; i++) {
                        w[i] = __fmaf_rn(s0, byte_f(lo[c], i), -o0);
                        w[4 + i] = __fmaf_rn(s1, byte_f(hi[c], i), -o1);
                    }
#pragma unroll
                    for (int b = 0; b < NV; b++)
                        if ((uint32_t)b < nv) {
                            const float *xb = xv[b] + 256 * k + 64 * c + l;
#pragma unroll
                            for (uint32_t i = 0; i < 8; i += 2) {
                                acc[b] = __fmaf_rn(w[i], xld(xb + 8 * i), acc[b]);
                                acc1[b] = __fmaf_rn(w[i + 1], xld(xb + 8 * i + 8), acc1[b]);
                            }
                        }
                }
            }
        };
        uint32_t k = 0;
        // 16-byte aligned rows: spans of 4 blocks (576 bytes = 36 pieces)
        // staged through this warp's part of shared memory
        // (two buffers: the next span is copied in asynchronously while the
        // current one is used)
        constexpr uint32_t KB = 4, SB = KB * 144, SP = SB / 16;
        __shared__ __align__(16) uint8_t qsm[2][FGEMV_THREADS / 32][4][SB + 16];  // padded: rows on other banks
        if (((reinterpret_cast<uintptr_t>(a.w) | a.row_bytes) & 15u) == 0) {
            const uint32_t rw = (threadIdx.x >> 3) & 3u, wp = threadIdx.x >> 5, nit = nbk / KB;
            auto issue = [&](uint32_t it) {
                if (it < nit) stage_row_async<5>(rp + 144 * (KB * it), qsm[it & 1u][wp][rw], SP, l);
                cp_commit();
            };
            issue(0);
            for (uint32_t it = 0; it < nit; it++, k += KB) {
                issue(it + 1);
                cp_wait<1>();
                __syncwarp();
#pragma unroll 2
                for (uint32_t kk = 0; kk < KB; kk++) q4_block(&qsm[it & 1u][wp][rw][144 * kk], k + kk);
                __syncwarp();  // done with this buffer before it is refilled
            }
        }
        for (; k < nbk; k++) q4_block(rp + k * 144, k);
    } else {  // FDT_Q6_K
        const uint32_t nbk = n / 256;
        // block k at bp (global or shared memory)
        auto q6_block = [&](const uint8_t *bp, uint32_t k) {
            const float d = h2f(gu16(bp + 208));
            float sc[16];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t v = gu16(bp + 192 + 2 * j);
                sc[2 * j] = (float)(int)(int8_t)(v & 0xFFu);
                sc[2 * j + 1] = (float)(int)(int8_t)(v >> 8);
            }
            float blk[NV];
#pragma unroll
            for (int b = 0; b < NV; b++) blk[b] = 0.0f;
#pragma unroll
            for (uint32_t h = 0; h < 2; h++) {
                // q6_groups (quant.rs:574-607) for positions l, 8+l, 16+l, 24+l of this half
                const uint32_t A = gld4(bp + 64 * h, l), B = gld4(bp + 64 * h + 32, l), H = gld4(bp + 128 + 32 * h, l);
                const uint32_t Q[4] = {(A & 0x0F0F0F0Fu) | ((H & 0x03030303u) << 4),
                                       (B & 0x0F0F0F0Fu) | (((H >> 2) & 0x03030303u) << 4),
                                       ((A >> 4) & 0x0F0F0F0Fu) | (((H >> 4) & 0x03030303u) << 4),
                                       ((B >> 4) & 0x0F0F0F0Fu) | (((H >> 6) & 0x03030303u) << 4)};
                if constexpr (!MULTI) {
                    // dot_q6_k_row_avx2 (quant.rs:552-616): l-steps outer, groups inner
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; kk++)
#pragma unroll
                        for (uint32_t g = 0; g < 4; g++) {
                            const float w = __fmul_rn(q6_f(Q[g], kk), sc[8 * h + (kk >> 1) + 2 * g]);
#pragma unroll
                            for (int b = 0; b < NV; b++)
                                if ((uint32_t)b < nv)
                                    blk[b] = __fmaf_rn(w, xld(xv[b] + 256 * k + 128 * h + 32 * g + 8 * kk + l), blk[b]);
                        }
                } else {
                    // deq_q6k (quant_multi.rs:77-110), then the a0/a1 chains
#pragma unroll
                    for (uint32_t g = 0; g < 4; g++) {
                        const float s0 = __fmul_rn(d, sc[8 * h + 2 * g]), s1 = __fmul_rn(d, sc[8 * h + 1 + 2 * g]);
                        const float w0 = __fmul_rn(s0, q6_f(Q[g], 0)), w1 = __fmul_rn(s0, q6_f(Q[g], 1));
                        const float w2 = __fmul_rn(s1, q6_f(Q[g], 2)), w3 = __fmul_rn(s1, q6_f(Q[g], 3));
#pragma unroll
                        for (int b = 0; b < NV; b++)
                            if ((uint32_t)b < nv) {
                                const float *xb = xv[b] + 256 * k + 128 * h + 32 * g + l;
                                acc[b] = __fmaf_rn(w0, xld(xb), acc[b]);
                                acc1[b] = __fmaf_rn(w1, xld(xb + 8), acc1[b]);
                                acc[b] = __fmaf_rn(w2, xld(xb + 16), acc[b]);
                                acc1[b] = __fmaf_rn(w3, xld(xb + 24), acc1[b]);
                            }
                    }
                }
            }
            if constexpr (!MULTI) {
#pragma unroll
                for (int b = 0; b < NV; b++) acc[b] = __fmaf_rn(d, blk[b], acc[b]);
            }
        };
        uint32_t k = 0;
        if constexpr (!MULTI) {
            // one vector with x staged: spans of 8 blocks (1680 bytes = 105
            // pieces, 16-byte aligned in 16-byte aligned rows) staged through
            // this warp's part of the dynamic shared memory, after x
            if (a.stage_x && ((reinterpret_cast<uintptr_t>(a.w) | a.row_bytes) & 15u) == 0) {
                constexpr uint32_t KB = 8, SB = KB * 210, SP = SB / 16, RST = SB + 16;
                const uint32_t rw = (threadIdx.x >> 3) & 3u, wp = threadIdx.x >> 5;
                uint8_t *buf = reinterpret_cast<uint8_t *>(fsums + fgemv_presum_floats(DT, MULTI, nv, n) + n) +
                               (wp * 4u + rw) * RST;
                for (; k + KB <= nbk; k += KB) {
                    __syncwarp();
                    stage_row<14>(rp + 210 * k, buf, SP, l);
                    __syncwarp();
#pragma unroll 1
                    for (uint32_t kk = 0; kk < KB; kk++) q6_block(buf + 210 * kk, k + kk);
                }
            }
        }
        constexpr int UQ6 = NV == 1 ? 2 : 1;
#pragma unroll UQ6
        for (; k < nbk; k++) q6_block(rp + k * 210, k);
    }

    // the next kernel may launch now: its CTAs would otherwise sit on this
    // kernel's SMs waiting, taking the occupancy its loads need
    grid_launch_dependents();
    float res[NV];
#pragma unroll
    for (int b = 0; b < NV; b++) {
        if constexpr (MULTI) {
            res[b] = hsum_shuf8(__fadd_rn(acc[b], acc1[b]));
        } else {
            const float h = hsum_hadd8(acc[b]);
            res[b] = DT == FDT_Q4_K ? __fsub_rn(h, extra[b]) : DT == FDT_F32 || DT == FDT_F16 ? __fadd_rn(h, extra[b]) : h;
        }
    }
    if (valid) {
#pragma unroll
        for (int b = 0; b < NV; b++)
            if ((uint32_t)b == l && (uint32_t)b < nv) a.out[(uint64_t)b * a.ldo + row] = res[b];
    }
}

#define SG_FGEMV_INST(DT, NV, M) template __global__ void gemv_float_kernel<DT, NV, M>(const __grid_constant__ FGemvArgs);
#define SG_FGEMV_NV(DT, M) SG_FGEMV_INST(DT, 1, M) SG_FGEMV_INST(DT, 2, M) SG_FGEMV_INST(DT, 4, M) SG_FGEMV_INST(DT, 8, M)
SG_FGEMV_NV(FDT_F32, false)
SG_FGEMV_NV(FDT_F32, true)
SG_FGEMV_NV(FDT_F16, false)
SG_FGEMV_NV(FDT_Q8_0, false)
SG_FGEMV_NV(FDT_Q8_0, true)
SG_FGEMV_NV(FDT_Q4_K, false)
SG_FGEMV_NV(FDT_Q4_K, true)
SG_FGEMV_NV(FDT_Q6_K, false)
SG_FGEMV_NV(FDT_Q6_K, true)

}  // namespace sg
