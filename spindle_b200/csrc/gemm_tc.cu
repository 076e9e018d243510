// gemm_tc.cu — the tcgen05 batch kernel of gemm_tc.cuh.
#include <cuda_fp16.h>

#include "gemm_tc.cuh"
#include "tiled_block.cuh"

namespace sg {
using namespace tiled;

namespace {

// Shared-memory operand layout (K-major, no swizzle): 8x8 f16 core matrices
// of 128 contiguous bytes (8 rows of 16 bytes); the 32 core matrices along
// K of one 8-row group follow each other (LBO = 128), 8-row groups are
// TC_SBO apart.  Element (row, k) is at (row / 8) * TC_SBO + (k / 8) * 128 +
// (row % 8) * 16 + (k % 8) * 2.
constexpr uint32_t TC_SBO = 32u * 128u;
// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B f16
// (bits 7-9, 10-12 = 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t TC_IDESC = (1u << 4) | ((TC_TOK >> 3) << 17) | ((TC_ROWS >> 4) << 24);

// Shared-memory matrix descriptor: start >> 4 (bits 0-13), LBO >> 4
// (16-29), SBO >> 4 (32-45), version 1 (bits 46-47), no swizzle (61-63 = 0).
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t sbo = TC_SBO) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46);
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t ad, uint64_t bd, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(ad), "l"(bd), "r"(TC_IDESC), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive TMEM columns of this thread's lane (32x32b shape), waited for
// inside the same statement so no use of the registers can move above it.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive TMEM columns of this thread's lane, waited for in the same statement
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_splat(float v) {
    const uint32_t h = __half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
}

__device__ __forceinline__ uint4 ldg128(const uint8_t *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

// f16 pairs of the magic 0x6400 | n = 1024 + n (n < 1024): nibbles (bytes 0,
// 2) and (1, 3) of a word of four bytes, low or high nibble
constexpr uint32_t H1024 = 0x64006400u;
// -1152 in f16: 1024 + (y ^ 0x80) - 1152 = y for a signed byte y
constexpr uint32_t HM1152 = 0xE480E480u;


// After the last super-block (every MMA complete): the lane pairs x_m = a_m +
// a_{m+4} and the corrections meet in shared memory (scratch: 40 KB), then
// thread (rr, th) writes tokens 8th..8th+7 of row rr as
// ((x0 + x2) + (x1 + x3)) - corr, or silu(gate) * up for the packed gate/up
// layout.
__device__ __forceinline__ void tc_finish(const GemmTcArgs &a, uint8_t *scratch, const float (&acc)[TC_TOK][4],
                                          const float (&corr)[8], uint32_t th, uint32_t rr, uint32_t r, uint32_t T,
                                          bool tile_ok) {
    float *finx = reinterpret_cast<float *>(scratch);  // [4][16 tokens][128 rows]
    float *finc = finx + 4 * TC_TOK * TC_ROWS;          // [16 tokens][128 rows]
#pragma unroll
    for (int t = 0; t < (int)TC_TOK; t++) {
        finx[((2 * th + 0) * TC_TOK + t) * TC_ROWS + rr] = __fadd_rn(acc[t][0], acc[t][2]);
        finx[((2 * th + 1) * TC_TOK + t) * TC_ROWS + rr] = __fadd_rn(acc[t][1], acc[t][3]);
    }
#pragma unroll
    for (int t8 = 0; t8 < 8; t8++) finc[(8 * th + t8) * TC_ROWS + rr] = corr[t8];
    __syncthreads();
#pragma unroll
    for (int t8 = 0; t8 < 8; t8++) {
        const uint32_t t = 8u * th + t8, tok = blockIdx.y * TC_TOK + t;
        const float x0 = finx[(0 * TC_TOK + t) * TC_ROWS + rr], x1 = finx[(1 * TC_TOK + t) * TC_ROWS + rr];
        const float x2 = finx[(2 * TC_TOK + t) * TC_ROWS + rr], x3 = finx[(3 * TC_TOK + t) * TC_ROWS + rr];
        const float yv = __fsub_rn(__fadd_rn(__fadd_rn(x0, x2), __fadd_rn(x1, x3)), finc[t * TC_ROWS + rr]);
        if (a.swiglu) {
            // rows r < 8 gate, r + 8 up of the same outputs (smollm_chat.rs:357-359)
            const float up = __shfl_down_sync(0xffffffffu, yv, 8);
            const uint32_t jo = T * 8 + r;
            if (tok < a.ntok && tile_ok && r < 8 && 2 * jo < a.r1) a.out[(uint64_t)tok * a.ldo + jo] = silu_mul(yv, up);
        } else {
            const uint32_t row = T * TILE_ROWS + r;
            if (tok < a.ntok && tile_ok && row >= a.r0 && row < a.r1) a.out[(uint64_t)tok * a.ldo + row] = yv;
        }
    }
}

__device__ __forceinline__ bool tc_alloc(uint32_t *slot, uint32_t cols, uint32_t warp) {
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                     "r"(cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return true;
}

__device__ __forceinline__ void tc_dealloc(uint32_t tbase, uint32_t cols, uint32_t warp) {
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(cols) : "memory");
    }
}

}  // namespace

// One CTA: rows of 8 tiles (blockIdx.x) x tokens 16 * blockIdx.y .. +16.
// Per super-block i (stage s = i & 1, TMEM buffer s):
//   all threads stage A (thread = row rr, half g: lanes 4g..4g+3) and B
//   (thread = token t, lane L, sub-blocks 4jj..4jj+3), then thread 0 issues
//   16 MMAs (lane L, K half h: D[s][L] (+)= A[:, 32L+16h..] B[:, 32L+16h..]^T)
//   and commits them to mma_done[s]; the epilogue of block i - 1 runs while
//   they execute.
// Epilogue thread (row rr = 32 (warp & 3) + lane, set th = warp >> 2) keeps
// lanes {2th, 2th+1, 2th+4, 2th+5} of its row for all 16 tokens and the
// correction of tokens 8th..8th+7.
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_tc_q4k_kernel(const __grid_constant__ GemmTcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *mma_done = reinterpret_cast<uint64_t *>(smem);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 64);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    constexpr uint32_t CB = 2304;  // tiled_col_bytes(Q4_K)
    if (blockDim.x != TC_THREADS || a.nb == 0 || a.ntok == 0 || a.ntok > QB_MAX_TOK ||
        gridDim.y * TC_TOK < a.ntok || dynamic_smem_size() < TC_SMEM) {
        if (tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    if (tid == 0) {
        mbar_init(&mma_done[0], 1);
        mbar_init(&mma_done[1], 1);
        fence_mbar_init();
    }
    tc_alloc(tmem_slot, TC_TMEM_COLS, warp);
    const uint32_t tbase = *tmem_slot;

    const uint64_t tile_bytes = (uint64_t)a.nb * CB;
    // this CTA's 16 tokens lie in QB group gq (TC_TOK divides QB_GROUP): its
    // image holds gn vectors, token xtok is its vector xtok - 64 gq
    const uint32_t gq = blockIdx.y * TC_TOK / QB_GROUP, gn = qb_group_tokens(a.ntok, gq);
    const uint8_t *qimg = a.qb + qb_group_offset(gq, a.nb);
    const uint32_t qbb = qb_block_bytes(gn);
    // staging roles
    const uint32_t rr = tid & 127u, g = tid >> 7, jt = rr >> 4, r = rr & 15u;
    const bool tile_ok = blockIdx.x * 8u + jt < a.ntiles;
    const uint32_t T = a.t0 + blockIdx.x * 8u + jt;
    const uint8_t *wrow = a.w + (uint64_t)(tile_ok ? T : a.t0) * tile_bytes;
    // token staging: 8 consecutive threads take 8 tokens of one core matrix
    // (one 128-byte shared-memory wavefront per store phase)
    const uint32_t xt = (tid & 7u) | ((tid >> 4) & 8u), xc = (tid >> 3) & 15u, xL = xc >> 1, xjj = xc & 1u;
    const uint32_t xtok = blockIdx.y * TC_TOK + xt, xu = xtok - gq * QB_GROUP;
    const bool xok = xtok < a.ntok;
    // epilogue roles
    const uint32_t q = warp & 3u, th = warp >> 2;

    uint4 qv[4], hd;
    auto load_w = [&](uint32_t i) {
        if (!tile_ok) return;
        const uint8_t *col = wrow + (uint64_t)i * CB;
        hd = ldg128(col + 2048 + 16 * r);
#pragma unroll
        for (int cc = 0; cc < 4; cc++) qv[cc] = ldg128(col + 128 * r + 16 * q4k_chunk(2 * cc + g, r));
    };
    uint32_t yw[4], bsw = 0;
    float xdv = 0.0f;
    auto load_x = [&](uint32_t i) {
        if (!xok) return;
        const uint8_t *blk = qimg + (uint64_t)i * qbb;
#pragma unroll
        for (int j = 0; j < 4; j++)
            yw[j] = __ldg(reinterpret_cast<const uint32_t *>(blk + 256u * xu + 32u * (4u * xjj + j) + 4u * xL));
        if (xc < 8) bsw = __ldg(reinterpret_cast<const uint32_t *>(blk + 256u * gn + 32u * xu + 4u * xc));
        if (xc == 8) xdv = __ldg(reinterpret_cast<const float *>(blk + 288u * gn) + xu);
    };
    auto stage = [&](uint32_t s) { return smem + TC_HDR_BYTES + s * TC_STAGE_BYTES; };
    auto xslot = [&](uint32_t i) { return reinterpret_cast<int32_t *>(smem + 1024 + (i % 3u) * TC_XS_BYTES); };

    auto store_a = [&](uint8_t *A) {
        uint8_t *dst = A + (rr >> 3) * TC_SBO + (rr & 7u) * 16u;
        if (!tile_ok) {
#pragma unroll
            for (int kk = 0; kk < 16; kk++)
                *reinterpret_cast<uint4 *>(dst + (16u * g + kk) * 128u) = make_uint4(0, 0, 0, 0);
            return;
        }
        const uint32_t sclo = hd.y & 0x3F3F3F3Fu, schi = (hd.w & M4) | ((hd.y >> 2) & B45);
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
            const int slo = ubyte(cc < 2 ? sclo : schi, (2 * cc) & 3), shi = ubyte(cc < 2 ? sclo : schi, (2 * cc + 1) & 3);
            const uint32_t s_lo = h2_splat((float)slo), n_lo = h2_splat(-1024.0f * (float)slo);
            const uint32_t s_hi = h2_splat((float)shi), n_hi = h2_splat(-1024.0f * (float)shi);
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const uint32_t wd = w4(qv[cc], m);
                uint4 o;
                o.x = hfma2((wd & 0x000F000Fu) | H1024, s_lo, n_lo);
                o.y = hfma2(((wd >> 8) & 0x000F000Fu) | H1024, s_lo, n_lo);
                o.z = hfma2(((wd >> 4) & 0x000F000Fu) | H1024, s_hi, n_hi);
                o.w = hfma2(((wd >> 12) & 0x000F000Fu) | H1024, s_hi, n_hi);
                const uint32_t kc = 4u * (4u * g + m) + cc;
                *reinterpret_cast<uint4 *>(dst + kc * 128u) = o;
            }
        }
    };
    auto store_x = [&](uint8_t *B, int32_t *bs2, float *xd) {
        uint8_t *dst = B + (xt >> 3) * TC_SBO + (xt & 7u) * 16u;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint4 o = make_uint4(0, 0, 0, 0);
            if (xok) {
                const uint32_t u0 = yw[2 * h] ^ 0x80808080u, u1 = yw[2 * h + 1] ^ 0x80808080u;
                o.x = hadd2((u0 & 0x00FF00FFu) | H1024, HM1152);
                o.y = hadd2(((u0 >> 8) & 0x00FF00FFu) | H1024, HM1152);
                o.z = hadd2((u1 & 0x00FF00FFu) | H1024, HM1152);
                o.w = hadd2(((u1 >> 8) & 0x00FF00FFu) | H1024, HM1152);
            }
            *reinterpret_cast<uint4 *>(dst + (4u * xL + 2u * xjj + h) * 128u) = o;
        }
        if (xc < 8) bs2[xt * 8 + xc] = xok ? (int32_t)(int16_t)(bsw & 0xFFFFu) + (int32_t)(int16_t)(bsw >> 16) : 0;
        if (xc == 8) xd[xt] = xok ? xdv : 0.0f;
    };

    float acc[TC_TOK][4], corr[8];
#pragma unroll
    for (int t = 0; t < (int)TC_TOK; t++)
#pragma unroll
        for (int l = 0; l < 4; l++) acc[t][l] = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; t++) corr[t] = 0.0f;
    bool failed = false;

    // eh: block i's row header (d, dmin, scales and mins), kept from its staging
    auto epilogue = [&](uint32_t i, const uint4 eh) {
        const uint32_t s = i & 1u;
        const int32_t *bs2 = xslot(i);
        const float *xd = reinterpret_cast<const float *>(bs2 + TC_TOK * 8);
        // warp-uniform outcome: the TMEM loads below are .sync.aligned
        const bool ok = mbar_wait_bounded(&mma_done[s], (i >> 1) & 1u, WAIT_LIMIT_NS);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
            failed = true;
        }
        tc_fence_after();
        if (failed) return;
        const float d = h2f_lo(eh.x), dmin = h2f_hi(eh.x);
        const uint32_t mlo = eh.z & 0x3F3F3F3Fu, mhi = ((eh.w >> 4) & M4) | ((eh.z >> 2) & B45);
        float cd[TC_TOK];
#pragma unroll
        for (int t = 0; t < (int)TC_TOK; t++) cd[t] = __fmul_rn(d, xd[t]);
        // lanes 2th, 2th+1 (then 2th+4, 2th+5) are 32 adjacent columns
#pragma unroll
        for (int pr = 0; pr < 2; pr++) {
            float v[32];
            tc_ld32(tbase + ((32u * q) << 16) + s * 128u + 16u * (2u * th + 4u * pr), v);
#pragma unroll
            for (int t = 0; t < (int)TC_TOK; t++) {
                acc[t][2 * pr] = __fmaf_rn(cd[t], v[t], acc[t][2 * pr]);
                acc[t][2 * pr + 1] = __fmaf_rn(cd[t], v[16 + t], acc[t][2 * pr + 1]);
            }
        }
#pragma unroll
        for (int t8 = 0; t8 < 8; t8++) {
            const uint32_t t = 8u * th + t8;
            const int4 b0 = *reinterpret_cast<const int4 *>(bs2 + 8 * t), b1 = *reinterpret_cast<const int4 *>(bs2 + 8 * t + 4);
            const int sp = ubyte(mlo, 0) * b0.x + ubyte(mlo, 1) * b0.y + ubyte(mlo, 2) * b0.z + ubyte(mlo, 3) * b0.w +
                           ubyte(mhi, 0) * b1.x + ubyte(mhi, 1) * b1.y + ubyte(mhi, 2) * b1.z + ubyte(mhi, 3) * b1.w;
            corr[t8] = __fadd_rn(corr[t8], __fmul_rn(__fmul_rn(dmin, xd[t]), __int2float_rn(sp)));
        }
        tc_fence_before();
    };

    hd = make_uint4(0, 0, 0, 0);
    load_w(0);
    grid_dependency_wait();
    load_x(0);
    uint4 hd_cur = hd, hd_prev = hd;
    for (uint32_t i = 0; i < a.nb; i++) {
        const uint32_t s = i & 1u;
        uint8_t *A = stage(s), *B = A + TC_A_BYTES;
        int32_t *bs2 = xslot(i);
        store_a(A);
        hd_prev = hd_cur;
        hd_cur = hd;
        store_x(B, bs2, reinterpret_cast<float *>(bs2 + TC_TOK * 8));
        if (i + 1 < a.nb) {
            load_w(i + 1);
            load_x(i + 1);
        }
        fence_proxy_async();
        tc_fence_before();
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
#pragma unroll
            for (uint32_t L = 0; L < 8; L++)
#pragma unroll
                for (uint32_t h = 0; h < 2; h++) {
                    const uint32_t koff = (4u * L + 2u * h) * 128u;
                    tc_mma(tbase + s * 128u + 16u * L, tc_desc(a0 + koff), tc_desc(b0 + koff), h);
                }
            tc_commit(&mma_done[s]);
        }
        if (i > 0) epilogue(i - 1, hd_prev);
    }
    if (!failed) epilogue(a.nb - 1, hd_cur);
    grid_launch_dependents();
    failed = __syncthreads_or(failed);

    if (!failed) tc_finish(a, stage(0), acc, corr, th, rr, r, T, tile_ok);
    tc_dealloc(tbase, TC_TMEM_COLS, warp);
}

// Q6_K: per super-block i (TMEM buffer b = i & 1) two units u = 0, 1 (stage
// u): lanes 4u..4u+3.  Staging thread (row rr, half h) builds sub-blocks
// 4h..4h+3 of those lanes from TILED16 chunks 4h+u, 4h+2+u, 8+2h+u; token
// thread (t, c) builds lane 4u + (c >> 2), sub-blocks 2(c & 3), 2(c & 3)+1.
// Thread 0 issues 16 MMAs per unit (lane, K half, lo / hi) into
// D_lo[L] = b*256 + 16L and D_hi[L] = b*256 + 128 + 16L.  A unit's stage is
// refilled once the MMAs of the same unit of the block before are complete.
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_tc_q6k_kernel(const __grid_constant__ GemmTcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *mma_done = reinterpret_cast<uint64_t *>(smem);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 64);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    constexpr uint32_t CB = 3360;  // tiled_col_bytes(Q6_K)
    constexpr uint32_t SBO6 = 16u * 128u;  // 16 core matrices along K per 8-row group
    if (blockDim.x != TC_THREADS || a.nb == 0 || a.ntok == 0 || a.ntok > QB_MAX_TOK ||
        gridDim.y * TC_TOK < a.ntok || dynamic_smem_size() < TC6_SMEM) {
        if (tid == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    if (tid == 0) {
        mbar_init(&mma_done[0], 1);
        mbar_init(&mma_done[1], 1);
        fence_mbar_init();
    }
    tc_alloc(tmem_slot, TC6_TMEM_COLS, warp);
    const uint32_t tbase = *tmem_slot;

    const uint64_t tile_bytes = (uint64_t)a.nb * CB;
    const uint32_t gq = blockIdx.y * TC_TOK / QB_GROUP, gn = qb_group_tokens(a.ntok, gq);  // as the Q4_K kernel
    const uint8_t *qimg = a.qb + qb_group_offset(gq, a.nb);
    const uint32_t qbb = qb_block_bytes(gn);
    const uint32_t rr = tid & 127u, h = tid >> 7, jt = rr >> 4, r = rr & 15u;
    const bool tile_ok = blockIdx.x * 8u + jt < a.ntiles;
    const uint32_t T = a.t0 + blockIdx.x * 8u + jt;
    const uint8_t *wrow = a.w + (uint64_t)(tile_ok ? T : a.t0) * tile_bytes;
    const uint32_t xt = tid >> 4, xc = tid & 15u, xm = xc >> 2, xq = xc & 3u;
    const uint32_t xtok = blockIdx.y * TC_TOK + xt, xu = xtok - gq * QB_GROUP;
    const bool xok = xtok < a.ntok;
    const uint32_t q = warp & 3u, th = warp >> 2;
    auto stage = [&](uint32_t u) { return smem + TC6_HDR_BYTES + u * TC6_STAGE_BYTES; };
    auto xslot = [&](uint32_t i) { return reinterpret_cast<int32_t *>(smem + 1024 + (i % 3u) * TC6_XS_BYTES); };

    uint4 L0, L1, HH, SC;
    uint32_t yw[2], bsw = 0;
    float xdv = 0.0f;
    auto load_w = [&](uint32_t i, uint32_t u) {
        if (!tile_ok) return;
        const uint8_t *col = wrow + (uint64_t)i * CB, *qrow = col + 192 * r;
        L0 = ldg128(qrow + 16 * q6k_chunk(4 * h + u, r));
        L1 = ldg128(qrow + 16 * q6k_chunk(4 * h + 2 + u, r));
        HH = ldg128(qrow + 16 * q6k_chunk(8 + 2 * h + u, r));
        SC = ldg128(col + 3072 + 16 * r);
    };
    auto load_x = [&](uint32_t i, uint32_t u) {
        if (!xok) return;
        const uint8_t *blk = qimg + (uint64_t)i * qbb;
        const uint32_t L = 4u * u + xm;
#pragma unroll
        for (int j = 0; j < 2; j++)
            yw[j] = __ldg(reinterpret_cast<const uint32_t *>(blk + 256u * xu + 32u * (2u * xq + j) + 4u * L));
        if (u == 0) {
            bsw = (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(blk + 256u * gn + 32u * xu) + xc);
            if (xc == 0) xdv = __ldg(reinterpret_cast<const float *>(blk + 288u * gn) + xu);
        }
    };
    // two 16-bit lanes holding n < 1024 -> f16 pair n * sc, exact (|n sc| <= 1920)
    auto cvt = [&](uint32_t v, uint32_t sc2) { return hmul2(hsub2(v | H1024, H1024), sc2); };
    auto store_a = [&](uint32_t u) {
        uint8_t *Alo = stage(u), *Ahi = Alo + TC6_A_BYTES;
        const uint32_t off = (rr >> 3) * SBO6 + (rr & 7u) * 16u;
        if (!tile_ok) {
#pragma unroll
            for (int m = 0; m < 4; m++)
#pragma unroll
                for (int c2 = 0; c2 < 2; c2++) {
                    const uint32_t kc = 4u * m + 2u * h + c2;
                    *reinterpret_cast<uint4 *>(Alo + off + kc * 128u) = make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4 *>(Ahi + off + kc * 128u) = make_uint4(0, 0, 0, 0);
                }
            return;
        }
        uint32_t sc2[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t si = 2u * (4u * h + j) + u;  // scale of sub-block 4h + j, lanes 4u..4u+3
            sc2[j] = h2_splat((float)sbyte(w4(SC, si >> 2), si & 3u));
        }
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const uint32_t l0 = w4(L0, m), l1 = w4(L1, m), hh = w4(HH, m);
            // sub-blocks 4h + j: low 4 bits and the 2 high bits of w
            const uint32_t lo[4] = {l0 & M4, l1 & M4, (l0 >> 4) & M4, (l1 >> 4) & M4};
            const uint32_t hi[4] = {hh & 0x03030303u, (hh >> 2) & 0x03030303u, (hh >> 4) & 0x03030303u,
                                    (hh >> 6) & 0x03030303u};
#pragma unroll
            for (int c2 = 0; c2 < 2; c2++) {
                const int j0 = 2 * c2, j1 = 2 * c2 + 1;
                const uint32_t kc = 4u * m + 2u * h + c2;
                uint4 o;
                o.x = cvt(lo[j0] & 0x000F000Fu, sc2[j0]);
                o.y = cvt((lo[j0] >> 8) & 0x000F000Fu, sc2[j0]);
                o.z = cvt(lo[j1] & 0x000F000Fu, sc2[j1]);
                o.w = cvt((lo[j1] >> 8) & 0x000F000Fu, sc2[j1]);
                *reinterpret_cast<uint4 *>(Alo + off + kc * 128u) = o;
                o.x = cvt(hi[j0] & 0x000F000Fu, sc2[j0]);
                o.y = cvt((hi[j0] >> 8) & 0x000F000Fu, sc2[j0]);
                o.z = cvt(hi[j1] & 0x000F000Fu, sc2[j1]);
                o.w = cvt((hi[j1] >> 8) & 0x000F000Fu, sc2[j1]);
                *reinterpret_cast<uint4 *>(Ahi + off + kc * 128u) = o;
            }
        }
    };
    auto store_x = [&](uint32_t i, uint32_t u) {
        uint8_t *B = stage(u) + 2u * TC6_A_BYTES;
        uint4 o = make_uint4(0, 0, 0, 0);
        if (xok) {
            const uint32_t u0 = yw[0] ^ 0x80808080u, u1 = yw[1] ^ 0x80808080u;
            o.x = hadd2((u0 & 0x00FF00FFu) | H1024, HM1152);
            o.y = hadd2(((u0 >> 8) & 0x00FF00FFu) | H1024, HM1152);
            o.z = hadd2((u1 & 0x00FF00FFu) | H1024, HM1152);
            o.w = hadd2(((u1 >> 8) & 0x00FF00FFu) | H1024, HM1152);
        }
        *reinterpret_cast<uint4 *>(B + (xt >> 3) * SBO6 + (4u * xm + xq) * 128u + (xt & 7u) * 16u) = o;
        if (u == 0) {
            int32_t *bs = xslot(i);
            bs[xt * 16 + xc] = xok ? (int32_t)(int16_t)bsw : 0;
            if (xc == 0) reinterpret_cast<float *>(bs + 256)[xt] = xok ? xdv : 0.0f;
        }
    };

    float acc[TC_TOK][4], corr[8];
#pragma unroll
    for (int t = 0; t < (int)TC_TOK; t++)
#pragma unroll
        for (int l = 0; l < 4; l++) acc[t][l] = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; t++) corr[t] = 0.0f;
    bool failed = false;
    auto wait_done = [&](uint32_t u, uint32_t parity) {
        const bool ok = mbar_wait_bounded(&mma_done[u], parity, WAIT_LIMIT_NS);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
            failed = true;
        }
        tc_fence_after();
    };
    // block i's MMAs are complete (the caller waited for its last unit)
    auto epilogue = [&](uint32_t i) {
        const uint32_t b = i & 1u;
        const int32_t *bs = xslot(i);
        const float *xd = reinterpret_cast<const float *>(bs + 256);
        const uint8_t *col = wrow + (uint64_t)i * CB;
        const uint4 esc = tile_ok ? ldg128(col + 3072 + 16 * r) : make_uint4(0, 0, 0, 0);
        const float d = tile_ok ? __half2float(__ldg(reinterpret_cast<const __half *>(col + 3328) + r)) : 0.0f;
        float cd[TC_TOK];
#pragma unroll
        for (int t = 0; t < (int)TC_TOK; t++) cd[t] = __fmul_rn(d, xd[t]);
#pragma unroll
        for (int li = 0; li < 4; li++) {
            const uint32_t L = 2u * th + (li & 1) + (li >> 1) * 4u;
            float vlo[16], vhi[16];
            const uint32_t ta = tbase + ((32u * q) << 16) + b * 256u + 16u * L;
            tc_ld16(ta, vlo);
            tc_ld16(ta + 128u, vhi);
#pragma unroll
            for (int t = 0; t < (int)TC_TOK; t++) {
                const int s = 16 * __float2int_rn(vhi[t]) + __float2int_rn(vlo[t]);
                acc[t][li] = __fmaf_rn(cd[t], __int2float_rn(s), acc[t][li]);
            }
        }
#pragma unroll
        for (int t8 = 0; t8 < 8; t8++) {
            const uint32_t t = 8u * th + t8;
            int sp = 0;
#pragma unroll
            for (int c = 0; c < 16; c++) sp += sbyte(w4(esc, c >> 2), c & 3) * bs[t * 16 + c];
            corr[t8] = __fadd_rn(corr[t8], __fmul_rn(cd[t], __int2float_rn(32 * sp)));
        }
        tc_fence_before();
    };

    load_w(0, 0);
    grid_dependency_wait();
    load_x(0, 0);
    for (uint32_t i = 0; i < a.nb && !failed; i++) {
        const uint32_t b = i & 1u;
        for (uint32_t u = 0; u < 2; u++) {
            if (i > 0) wait_done(u, (i - 1) & 1u);
            store_a(u);
            store_x(i, u);
            if (u == 0) {
                load_w(i, 1);
                load_x(i, 1);
            } else if (i + 1 < a.nb) {
                load_w(i + 1, 0);
                load_x(i + 1, 0);
            }
            fence_proxy_async();
            tc_fence_before();
            if (__syncthreads_or(failed)) {
                failed = true;
                break;
            }
            if (tid == 0) {
                tc_fence_after();
                const uint32_t a0 = smem_u32(stage(u)), b0 = a0 + 2u * TC6_A_BYTES;
#pragma unroll
                for (uint32_t m = 0; m < 4; m++)
#pragma unroll
                    for (uint32_t k2 = 0; k2 < 2; k2++) {
                        const uint32_t koff = (4u * m + 2u * k2) * 128u, L = 4u * u + m;
                        const uint32_t d = tbase + b * 256u + 16u * L;
                        tc_mma(d, tc_desc(a0 + koff, SBO6), tc_desc(b0 + koff, SBO6), k2);
                        tc_mma(d + 128u, tc_desc(a0 + TC6_A_BYTES + koff, SBO6), tc_desc(b0 + koff, SBO6), k2);
                    }
                tc_commit(&mma_done[u]);
            }
        }
        if (!failed && i > 0) epilogue(i - 1);
    }
    if (!failed) {
        wait_done(1, (a.nb - 1) & 1u);
        if (!failed) epilogue(a.nb - 1);
    }
    grid_launch_dependents();
    failed = __syncthreads_or(failed);
    if (!failed) tc_finish(a, stage(0), acc, corr, th, rr, r, T, tile_ok);
    tc_dealloc(tbase, TC6_TMEM_COLS, warp);
}

}  // namespace sg
