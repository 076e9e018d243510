// gemm_batch.cu — the batch kernels of gemm_batch.cuh.
#include "gemm_batch.cuh"
#include "q8k_block.cuh"
#include "tiled_block.cuh"

namespace sg {
using namespace tiled;

namespace {

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One super-block column of one tile (col) against `nv` vectors whose QB data
// for this block start at aq (qs, 256 B apart), ab (bsums, 32 B apart) and ad
// (d): thread (g, r) folds AVX lanes 4g..4g+3 of row r into acc / corr, in the
// order of q4k_dot / q6k_dot followed by the GEMV's single-slot chain step.
template <int DT, int TPW>
__device__ __forceinline__ void gb_block(const uint8_t *col, uint32_t g, uint32_t r, uint32_t nv, const uint8_t *aq,
                                         const uint8_t *ab, const float *ad, float (&acc)[TPW][4],
                                         float (&corr)[TPW]) {
    if constexpr (DT == 0) {
        const uint4 hd = lds128(col + 2048 + 16 * r);
        const float d = h2f_lo(hd.x), dmin = h2f_hi(hd.x);
        const uint32_t sclo = hd.y & 0x3F3F3F3Fu, schi = (hd.w & M4) | ((hd.y >> 2) & B45);
        const uint32_t mnw = g ? (((hd.w >> 4) & M4) | ((hd.z >> 2) & B45)) : (hd.z & 0x3F3F3F3Fu);
        const int sc[8] = {ubyte(sclo, 0), ubyte(sclo, 1), ubyte(sclo, 2), ubyte(sclo, 3),
                           ubyte(schi, 0), ubyte(schi, 1), ubyte(schi, 2), ubyte(schi, 3)};
        uint32_t lo[4][4], hi[4][4];
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
            const uint4 qv = lds128(col + 128 * r + 16 * q4k_chunk(2 * cc + g, r));
#pragma unroll
            for (int m = 0; m < 4; m++) {
                lo[cc][m] = w4(qv, m) & M4;
                hi[cc][m] = w4(qv, m) & 0xF0F0F0F0u;
            }
        }
#pragma unroll
        for (int v = 0; v < TPW; v++) {
            if (v >= (int)nv) break;
            const uint8_t *y = aq + 256u * v + 16u * g;
            uint4 Y[8];
#pragma unroll
            for (int kk = 0; kk < 8; kk++) Y[kk] = lds128(y + 32 * kk);
            const uint4 B = lds128(ab + 32u * v + 16u * g);
            const float xd = ad[v];
            int s[4], sh[4];
#pragma unroll
            for (int m = 0; m < 4; m++) s[m] = sh[m] = 0;
#pragma unroll
            for (int cc = 0; cc < 4; cc++)
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    s[m] += sc[2 * cc] * __dp4a((int)lo[cc][m], (int)w4(Y[2 * cc], m), 0);
                    sh[m] += sc[2 * cc + 1] * dp4a_us(hi[cc][m], (int)w4(Y[2 * cc + 1], m));
                }
            const float cd = __fmul_rn(d, xd);
            int sp = 0;
#pragma unroll
            for (int m = 0; m < 4; m++) sp = __dp2a_lo((int)w4(B, m), (int)__byte_perm(mnw, 0, 0x11 * m), sp);
            sp += __shfl_xor_sync(0xffffffffu, sp, 16);
            const float ct = __fmul_rn(__fmul_rn(dmin, xd), __int2float_rn(sp));
#pragma unroll
            for (int m = 0; m < 4; m++) acc[v][m] = __fmaf_rn(cd, lane_f<0>(s[m] + (sh[m] >> 4)), acc[v][m]);
            corr[v] = __fadd_rn(corr[v], ct);
        }
    } else {
        const uint8_t *qrow = col + 192 * r;
        uint32_t w[8][4];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 L0 = lds128(qrow + 16 * q6k_chunk(4 * h + g, r));
            const uint4 L1 = lds128(qrow + 16 * q6k_chunk(4 * h + 2 + g, r));
            const uint4 H = lds128(qrow + 16 * q6k_chunk(8 + 2 * h + g, r));
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const uint32_t l0 = w4(L0, m), l1 = w4(L1, m), hh = w4(H, m);
                w[4 * h + 0][m] = (l0 & M4) | ((hh << 4) & B45);
                w[4 * h + 1][m] = (l1 & M4) | ((hh << 2) & B45);
                w[4 * h + 2][m] = ((l0 >> 4) & M4) | (hh & B45);
                w[4 * h + 3][m] = ((l1 >> 4) & M4) | ((hh >> 2) & B45);
            }
        }
        const uint4 SC = lds128(col + 3072 + 16 * r);
        const float d = __half2float(*reinterpret_cast<const __half *>(col + 3328 + 2 * r));
        int scv[8];
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int kk = 0; kk < 4; kk++) scv[4 * h + kk] = sbyte(w4(SC, 2 * h + (kk >> 1)), 2 * (kk & 1) + (int)g);
        const uint32_t sw0 = g ? SC.z : SC.x, sw1 = g ? SC.w : SC.y;
#pragma unroll
        for (int v = 0; v < TPW; v++) {
            if (v >= (int)nv) break;
            const uint8_t *y = aq + 256u * v + 16u * g;
            uint4 Y[8];
#pragma unroll
            for (int kk = 0; kk < 8; kk++) Y[kk] = lds128(y + 32 * kk);
            const uint4 B = lds128(ab + 32u * v + 16u * g);
            const float xd = ad[v];
            int s[4];
#pragma unroll
            for (int m = 0; m < 4; m++) s[m] = 0;
#pragma unroll
            for (int kk = 0; kk < 8; kk++)
#pragma unroll
                for (int m = 0; m < 4; m++) s[m] += scv[kk] * __dp4a((int)w[kk][m], (int)w4(Y[kk], m), 0);
            const float cd = __fmul_rn(d, xd);
            int sp = __dp2a_lo((int)B.x, (int)sw0, 0);
            sp = __dp2a_hi((int)B.y, (int)sw0, sp);
            sp = __dp2a_lo((int)B.z, (int)sw1, sp);
            sp = __dp2a_hi((int)B.w, (int)sw1, sp);
            sp += __shfl_xor_sync(0xffffffffu, sp, 16);
            const float ct = __fmul_rn(cd, __int2float_rn(32 * sp));
#pragma unroll
            for (int m = 0; m < 4; m++) acc[v][m] = __fmaf_rn(cd, lane_f<1>(s[m]), acc[v][m]);
            corr[v] = __fadd_rn(corr[v], ct);
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(256) q8k_batch_kernel(const __grid_constant__ QbArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t wid = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= (uint64_t)a.n * a.nb) return;
    const uint32_t t = (uint32_t)(wid / a.nb), i = (uint32_t)(wid % a.nb);
    // token t is vector u of QB group q (gemm_batch.cuh)
    const uint32_t q = t / QB_GROUP, u = t % QB_GROUP, n = qb_group_tokens(a.n, q);
    uint8_t *blk = a.qb + qb_group_offset(q, a.nb) + (uint64_t)i * qb_block_bytes(n);
    q8k_block(a.x + t * a.ldx + 256u * i, reinterpret_cast<int8_t *>(blk + 256u * u),
              reinterpret_cast<int16_t *>(blk + 256u * n + 32u * u), reinterpret_cast<float *>(blk + 288u * n) + u,
              lane);
}

template <int DT, int TPW>
__global__ void __launch_bounds__(64 / TPW * 32, 1) gemm_batch_kernel(const __grid_constant__ GemmBatchArgs a) {
    constexpr uint32_t CB = tiled_col_bytes(DT);
    constexpr uint32_t CONS = gb_consumers(TPW), THREADS = CONS * 32u;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem), *empty = full + GB_MAX_STAGES;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // blockIdx.y: QB group (64 vectors) of the a.ntok: its image, its tokens, its outputs
    const uint32_t ntok = a.ntok > blockIdx.y * QB_GROUP ? qb_group_tokens(a.ntok, blockIdx.y) : 0u;
    const uint8_t *qb = a.qb + qb_group_offset(blockIdx.y, a.nb);
    float *const out = a.out + (uint64_t)blockIdx.y * QB_GROUP * a.ldo;
    const uint32_t wbytes = a.tps * CB, abytes = qb_block_bytes(ntok);
    // A launch this layout does not fit records an error and does nothing
    // (uniform exit, before any barrier).
    if (blockDim.x != THREADS || a.nstages < 2 || a.nstages > GB_MAX_STAGES || ntok == 0 ||
        a.ntok > QB_MAX_TOK || a.nq * a.tps != CONS || a.nq * (uint32_t)TPW < ntok || a.nb == 0 ||
        a.stage_bytes < wbytes + abytes || (a.stage_bytes & 15u) ||
        GB_BAR_BYTES + a.nstages * a.stage_bytes > dynamic_smem_size()) {
        if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    const uint32_t nsteps = (a.ntiles + a.tps - 1) / a.tps;
    const uint32_t my_steps = blockIdx.x < nsteps ? (nsteps - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
    const uint32_t nitems = my_steps * a.nb;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < a.nstages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CONS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    grid_launch_dependents();
    uint8_t *stages = smem + GB_BAR_BYTES;
    const uint64_t tile_bytes = (uint64_t)a.nb * CB;

    // Thread 0 also produces: item k = super-block column k % nb of this CTA's
    // step k / nb.  Weight columns do not depend on the kernel before; the
    // activations do, so the first items' weights are in flight before the
    // dependency wait.
    uint32_t issued = 0;
    bool waited = false;
    auto issue = [&](uint32_t k) {
        const uint32_t s = k % a.nstages;
        const uint32_t step = blockIdx.x + (k / a.nb) * gridDim.x, i = k % a.nb;
        const uint32_t nt = min(a.tps, a.ntiles - step * a.tps);
        uint8_t *st = stages + s * a.stage_bytes;
        mbar_arrive_expect_tx(&full[s], nt * CB + abytes);
        const uint8_t *wt = a.w + (uint64_t)(a.t0 + step * a.tps) * tile_bytes + (uint64_t)i * CB;
        for (uint32_t jj = 0; jj < nt; jj++) bulk_g2s(st + jj * CB, wt + jj * tile_bytes, CB, &full[s]);
        if (!waited) {
            grid_dependency_wait();
            waited = true;
        }
        bulk_g2s(st + wbytes, qb + (uint64_t)i * abytes, abytes, &full[s]);
        issued = k + 1;
    };
    if (threadIdx.x == 0) {
        for (uint32_t k = 0; k < nitems && k < a.nstages; k++) issue(k);
        if (!waited) grid_dependency_wait();
    }

    // Consumers: warp = (tile j of the step, token group q).
    const uint32_t j = warp / a.nq, q = warp % a.nq;
    const uint32_t v0 = (uint32_t)TPW * q, nv = ntok > v0 ? min((uint32_t)TPW, ntok - v0) : 0u;
    const uint32_t g = lane >> 4, r = lane & 15u;
    float acc[TPW][4], corr[TPW];
#pragma unroll
    for (int v = 0; v < TPW; v++) {
        corr[v] = 0.0f;
#pragma unroll
        for (int m = 0; m < 4; m++) acc[v][m] = 0.0f;
    }
    bool failed = false;
    for (uint32_t k = 0; k < nitems; k++) {
        const uint32_t s = k % a.nstages;
        const uint32_t step = blockIdx.x + (k / a.nb) * gridDim.x, i = k % a.nb;
        const bool mine = step * a.tps + j < a.ntiles && nv > 0;
        if (!failed) {
            const bool ok = mbar_wait_bounded(&full[s], (k / a.nstages) & 1u, WAIT_LIMIT_NS);
            if (__any_sync(0xffffffffu, !ok)) {
                if (lane == 0) atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                failed = true;
            }
        }
        if (mine && !failed) {
            const uint8_t *st = stages + s * a.stage_bytes;
            const uint8_t *act = st + wbytes;
            gb_block<DT, TPW>(st + j * CB, g, r, nv, act + 256u * v0, act + 256u * ntok + 32u * v0,
                         reinterpret_cast<const float *>(act + 288u * ntok) + v0, acc, corr);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (warp == 0) {
            bool pf = false;
            if (lane == 0 && !failed && k + a.nstages < nitems) {
                // every warp is done with item k: its stage takes item k + nstages
                if (mbar_wait_bounded(&empty[s], (k / a.nstages) & 1u, WAIT_LIMIT_NS)) {
                    issue(k + a.nstages);
                } else {
                    atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                    pf = true;
                }
            }
            if (__any_sync(0xffffffffu, pf)) failed = true;
        }
        if (i + 1 == a.nb) {
            if (mine && !failed) {
                // 8-lane tree ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), minus the correction
                const uint32_t mt = a.t0 + step * a.tps + j, row = mt * TILE_ROWS + r;
#pragma unroll
                for (int v = 0; v < TPW; v++) {
                    if (v >= (int)nv) break;
                    float x[4];
#pragma unroll
                    for (int m = 0; m < 4; m++) x[m] = __fadd_rn(acc[v][m], __shfl_down_sync(0xffffffffu, acc[v][m], 16));
                    const float yv = __fsub_rn(__fadd_rn(__fadd_rn(x[0], x[2]), __fadd_rn(x[1], x[3])), corr[v]);
                    float *dst = out + (uint64_t)(v0 + v) * a.ldo;
                    if (a.swiglu) {
                        // rows r < 8 gate, r + 8 up of the same outputs (smollm_chat.rs:357-359)
                        const float up = __shfl_down_sync(0xffffffffu, yv, 8);
                        const uint32_t jo = mt * 8 + r;
                        if (g == 0 && r < 8 && 2 * jo < a.r1) dst[jo] = silu_mul(yv, up);
                    } else if (g == 0 && row >= a.r0 && row < a.r1) {
                        dst[row] = yv;
                    }
                }
            }
#pragma unroll
            for (int v = 0; v < TPW; v++) {
                corr[v] = 0.0f;
#pragma unroll
                for (int m = 0; m < 4; m++) acc[v][m] = 0.0f;
            }
        }
    }
    if (threadIdx.x == 0) {
        // no copy may still be landing when the CTA exits: wait (bounded) for
        // the last item issued on every stage
        const uint32_t first = issued > a.nstages ? issued - a.nstages : 0u;
        for (uint32_t kk = first; kk < issued; kk++)
            mbar_wait_bounded(&full[kk % a.nstages], (kk / a.nstages) & 1u, WAIT_LIMIT_NS);
    }
}

template __global__ void gemm_batch_kernel<0, 4>(const __grid_constant__ GemmBatchArgs);
template __global__ void gemm_batch_kernel<1, 4>(const __grid_constant__ GemmBatchArgs);
template __global__ void gemm_batch_kernel<0, 8>(const __grid_constant__ GemmBatchArgs);
template __global__ void gemm_batch_kernel<1, 8>(const __grid_constant__ GemmBatchArgs);

}  // namespace sg
