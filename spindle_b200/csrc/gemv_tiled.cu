// gemv_tiled.cu — kernels over the TILED16 layout (see gemv_tiled.cuh).
#include "q8k_block.cuh"
#include "tiled_block.cuh"
#include "moe_select.cuh"

namespace sg {
using namespace tiled;

// The end of a row-split launch (see TGemvArgs): CTA c of G reads pairs
// [n*c/G, n*(c+1)/G) of this rank's receive buffer (n = nvec * rows), each as
// soon as it carries this call's epoch, into the plain output.  The pairs are
// 8-byte stores, single-copy atomic, so no fence orders data and flag; the
// epoch alternates the buffer's halves, and a rank can be at most one call
// ahead of another (its next call ends only with this rank's rows of that
// call), so a half is never overwritten before it is read.
__device__ __noinline__ void tp_gather(const TGemvArgs &a, uint32_t e) {
    const uint64_t R = a.tp_rows, n = (uint64_t)a.nvec * R;
    const unsigned long long *half = a.my_recv + (uint64_t)(e & 1u) * n;
    const uint64_t lo = n * blockIdx.x / gridDim.x, hi = n * (blockIdx.x + 1) / gridDim.x;
    uint64_t t0 = 0;
    for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        unsigned long long p;
        for (;;) {
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(p) : "l"(half + i) : "memory");
            if ((uint32_t)(p >> 32) == e) break;
            const uint64_t t = globaltimer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > WAIT_LIMIT_NS) {
                atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_PEER);
                p = 0x7fc00000ull;  // NaN
                break;
            }
            __nanosleep(32);
        }
        const uint64_t v = i / R, r = i - v * R;
        a.out[0][v * a.out_stride + r] = __uint_as_float((uint32_t)p);
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.ticket, 1u) == gridDim.x - 1) {
        *a.ticket = 0;  // every CTA of this launch has its ticket
        *a.epoch = e;
    }
}

template <int DT, int NV, int MODE>
__global__ void __launch_bounds__(TGEMV_WARPS * 32, 1) gemv_tiled_kernel(const __grid_constant__ TGemvArgs a) {
    constexpr uint32_t CB = tiled_col_bytes(DT);
    constexpr bool MOE = MODE == IN_MOE_X || MODE == IN_MOE_H;
    extern __shared__ __align__(128) uint8_t smem[];
    // A launch whose shared memory cannot hold this layout records an error
    // and does nothing (uniform exit, before any barrier).
    const uint32_t nwarps = blockDim.x >> 5;
    const uint32_t nact = tiled_nact(MODE, NV, a.nact);
    const bool JOBS = MOE && a.jobs != nullptr;
    const uint32_t job_bytes = JOBS ? tiled_job_bytes(NV) : 0u;
    if (tiled_smem_bytes(nwarps, a.S, a.nstages, a.stage_bytes, a.slot_blocks, NV, a.nb, nact, job_bytes) >
            dynamic_smem_size() ||
        a.bc == 0 || a.stage_bytes < a.bc * CB || a.S == 0 || a.S != (1u << a.s_log2) || a.S > nwarps ||
        (nwarps & (a.S - 1)) || (blockDim.x & 31) ||
        // a group with a second tile needs named barrier 1 + 2G (past 15 for G = 8)
        (a.S > 1 && 2u * (nwarps >> a.s_log2) + 1u > 16u &&
         (MOE ? (a.ntiles + gridDim.x - 1) / gridDim.x > (nwarps >> a.s_log2)
              : a.tiles_q > 1u || (a.tiles_q == 1u && a.tiles_r > 0u))) ||
        a.nstages * nwarps * 8 > ((MOE || a.qx_image) ? MOE_QX_BAR_OFF : TGEMV_BAR_BYTES) ||
        (MODE == IN_Q8K && a.qx_image && a.nvec != 1) ||
        (MOE && a.swiglu && (MODE != IN_MOE_X || (a.nvec != 1 && !JOBS))) ||
        (MOE && !JOBS && NV != 1) ||
        (JOBS && (!a.slots || !a.n_jobs || a.npeers || a.job_ints < 2 + NV || nact % NV || nact > MOE_MAXK * NV)) ||
        (MOE && ((!a.slots && a.max_slots > MOE_MAXK) || a.tiles_per_mat == 0 || nact == 0 ||
                 (uint64_t)a.ntiles * gridDim.x >= (1ull << 32) || a.ntiles < a.max_slots * a.tiles_per_mat)) ||
        (a.npeers && !MOE && (a.npeers > TP_MAX_RANKS || !a.ticket || !a.epoch || !a.out[0] || !a.my_recv)) ||
        (a.npeers && MOE && (MODE != IN_MOE_H || a.npeers > TP_MAX_RANKS || !a.slots || !a.slot_global || !a.epoch)) ||
        (a.slots && (!MOE || !a.n_slots || a.logits || (!JOBS && nact > MOE_MAXK) || (MODE == IN_MOE_X && !a.qx_tokens))) ||
        (MODE == IN_MOE_X && a.logits &&
         (a.n_expert == 0 || a.n_used == 0 || a.n_used > a.n_expert || a.n_used > MOE_MAXK ||
          moe_select_bytes(a.n_expert) > nwarps * a.nstages * a.stage_bytes))) {
        if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t g = lane >> 4, r = lane & 15u;
    // S is a power of two: shifts and masks instead of divisions (a runtime
    // division costs some twenty instructions, paid by every warp)
    const uint32_t S = a.S, SL = a.s_log2, group = warp >> SL, slot = warp & (S - 1u), G = nwarps >> SL;
    const uint32_t astride = act_bytes(a.nb);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * a.nstages;
    uint8_t *act = smem + TGEMV_BAR_BYTES;
    // jobs mode: local job j's slot count at jinfo[j], its slots at jinfo[MOE_MAXK + j * NV ..]
    uint32_t *jinfo = reinterpret_cast<uint32_t *>(act + nact * astride);
    uint8_t *rings = act + nact * astride + job_bytes;
    uint8_t *ring = rings + warp * a.nstages * a.stage_bytes;
    const uint32_t worker_floats = a.slot_blocks * NV * CHAIN_FLOATS;
    float *gscratch = reinterpret_cast<float *>(rings + nwarps * a.nstages * a.stage_bytes) +
                      group * (S - 1) * worker_floats;

    uint32_t ntiles = a.ntiles;
    uint32_t *msel = reinterpret_cast<uint32_t *>(smem + MOE_SEL_OFF);  // [0]: n, [16..32): ids
    const int32_t *sids = reinterpret_cast<const int32_t *>(msel + 16);
    if constexpr (MOE) {
        // The choice comes from the grids before this one: wait for them.
        grid_dependency_wait();
        grid_launch_dependents();
        if (MODE == IN_MOE_X && a.qx_image && threadIdx.x == 0) {
            // x's Q8_K image, ready-made by the router, lands while the choice is made
            uint64_t *qbar = reinterpret_cast<uint64_t *>(smem + MOE_QX_BAR_OFF);
            mbar_init(qbar, 1);
            fence_mbar_init();
            mbar_arrive_expect_tx(qbar, act_bytes(a.nb));
            bulk_g2s(act, a.qx_image, act_bytes(a.nb), qbar);
        }
        if (a.slots) {
            // batched: the slot table (and the jobs) were written by the kernel before
            if (threadIdx.x == 0) msel[0] = min(__ldcg(JOBS ? a.n_jobs : a.n_slots), a.max_slots);
        } else if (MODE == IN_MOE_X && a.logits) {
            // every CTA makes the router's choice itself (identical results);
            // the rings are free until the first weight copy is issued
            float *P = reinterpret_cast<float *>(rings);
            int32_t *K = reinterpret_cast<int32_t *>(P + ((a.n_expert + 3u) & ~3u));
            float *red = reinterpret_cast<float *>(K + ((a.n_expert + 3u) & ~3u));
            moe::Choice *ch = reinterpret_cast<moe::Choice *>(red + 64);
            float *probs = blockIdx.x == 0 ? a.probs : nullptr;
            if (a.n_expert <= 256) {
                // one warp, experts in registers
                if (warp == 0) {
                    if (a.n_expert <= 64)
                        moe::select_warp<2>(a.logits, a.n_expert, a.n_used, a.norm, a.prune, ch, probs, P, lane);
                    else if (a.n_expert <= 128)
                        moe::select_warp<4>(a.logits, a.n_expert, a.n_used, a.norm, a.prune, ch, probs, P, lane);
                    else
                        moe::select_warp<8>(a.logits, a.n_expert, a.n_used, a.norm, a.prune, ch, probs, P, lane);
                }
                __syncthreads();
            } else {
                moe::select(a.logits, a.n_expert, a.n_used, a.norm, a.prune, P, K, red, ch, probs);
            }
            if (threadIdx.x < MOE_MAXK) {
                msel[16 + threadIdx.x] = (uint32_t)ch->id[threadIdx.x];
                if (blockIdx.x == 0) {
                    a.sel_out->id[threadIdx.x] = ch->id[threadIdx.x];
                    a.sel_out->weight[threadIdx.x] = ch->w[threadIdx.x];
                }
            }
            if (threadIdx.x == 0) {
                msel[0] = min(ch->n, a.max_slots);
                if (blockIdx.x == 0) {
                    a.sel_out->pad_[0] = a.sel_out->pad_[1] = a.sel_out->pad_[2] = 0;
                    a.sel_out->n = ch->n;
                }
            }
            fence_proxy_async();  // generic writes to the rings before the copies into them
        } else if (threadIdx.x < 32) {
            const uint32_t n = min(__ldcg(&a.sel->n), a.max_slots);
            const int32_t id = threadIdx.x < n ? __ldcg(&a.sel->id[threadIdx.x]) : 0;
            const bool bad = __any_sync(0xffffffffu, threadIdx.x < n && (id < 0 || (uint32_t)id >= a.n_expert));
            if (threadIdx.x < MOE_MAXK) msel[16 + threadIdx.x] = (uint32_t)id;
            if (threadIdx.x == 0) {
                msel[0] = bad ? 0u : n;
                if (bad) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
            }
        }
        __syncthreads();
        ntiles = msel[0] * a.tiles_per_mat;
    } else {
        // Let the next kernel in the stream launch as soon as SMs free up: it
        // only prefetches its own weights before waiting for this grid to finish.
        grid_launch_dependents();
    }
    const uint32_t b_lo = (a.nb * slot) >> SL, nblk = ((a.nb * (slot + 1)) >> SL) - b_lo;
    const uint32_t bc = a.bc, nchunk = (nblk + bc - 1) / bc;  // stages per tile for this slot
    // This group's tiles: first, first + step, ... (my_tiles of them).  GEMV:
    // groups are numbered CTA-minor so that consecutive tiles land on different
    // SMs.  MoE: each CTA takes a contiguous range, so that it needs the
    // activations of one or two slots only (slots s_lo..s_hi).
    uint32_t first, step, my_tiles, s_lo = 0, s_hi = 0;
    uint32_t cta_units = 0;  // MoE: units s_lo..s_hi of this CTA (0: none), the same in every warp
    if constexpr (MOE) {
        // 32-bit products: the entry check bounds ntiles * gridDim.x below 2^32
        const uint32_t lo = ntiles * blockIdx.x / gridDim.x, hi = ntiles * (blockIdx.x + 1) / gridDim.x;
        first = lo + group;
        step = G;
        my_tiles = first < hi ? (hi - first + G - 1) / G : 0u;
        if (lo < hi) {
            s_lo = lo / a.tiles_per_mat;
            s_hi = (hi - 1) / a.tiles_per_mat;
            cta_units = s_hi - s_lo + 1;
        }
        // activation images per unit: one per slot, NV per job (jobs mode)
        if ((MODE == IN_MOE_H || a.slots) && cta_units * (JOBS ? NV : 1) > nact) {
            if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);  // the host sized nact for this
            my_tiles = 0;
            s_hi = s_lo;
            cta_units = 0;
        }
        if (a.slots) {
            // this CTA's units s_lo..s_hi: expert ids into msel[16..], and for
            // IN_MOE_X each slot's token image into activation image s - s_lo
            // (jobs: image (s - s_lo) * NV + member)
            const uint32_t nloc = cta_units;
            bool bad = false;
            if (JOBS) {
                if (threadIdx.x < nloc) {
                    const int32_t *jb = a.jobs + (uint64_t)(s_lo + threadIdx.x) * a.job_ints;
                    const int32_t e = __ldcg(jb), n = __ldcg(jb + 1);
                    const uint32_t ns = __ldcg(a.n_slots);
                    bad = e < 0 || (uint32_t)e >= a.n_expert || n < 1 || n > NV;
                    for (int v = 0; v < NV; v++) {
                        const int32_t sl = v < n ? __ldcg(jb + 2 + v) : 0;
                        bad = bad || sl < 0 || (uint32_t)sl >= ns;
                        jinfo[MOE_MAXK + threadIdx.x * NV + v] = (uint32_t)sl;
                    }
                    msel[16 + threadIdx.x] = bad ? 0u : (uint32_t)e;
                    jinfo[threadIdx.x] = bad ? 0u : (uint32_t)n;
                }
                __syncthreads();
            } else if (threadIdx.x < nloc) {
                const int32_t e = __ldcg(a.slots + 2 * (s_lo + threadIdx.x));
                bad = e < 0 || (uint32_t)e >= a.n_expert;
                msel[16 + threadIdx.x] = bad ? 0u : (uint32_t)e;
            }
            if (MODE == IN_MOE_X && threadIdx.x == 0) {
                uint64_t *qbar = reinterpret_cast<uint64_t *>(smem + MOE_QX_BAR_OFF);
                mbar_init(qbar, 1);
                fence_mbar_init();
                uint32_t nimg = nloc;
                if (JOBS) {
                    nimg = 0;
                    for (uint32_t j = 0; j < nloc; j++) nimg += jinfo[j];
                }
                mbar_arrive_expect_tx(qbar, nimg * act_bytes(a.nb));
                for (uint32_t j = 0; j < nloc; j++) {
                    const uint32_t nm = JOBS ? jinfo[j] : 1u;
                    for (uint32_t v = 0; v < nm; v++) {
                        const uint32_t sl = JOBS ? jinfo[MOE_MAXK + j * NV + v] : s_lo + j;
                        const int32_t tok = __ldcg(a.slots + 2 * sl + 1);
                        bulk_g2s(act + (j * (JOBS ? NV : 1u) + v) * astride, a.qx_tokens + (uint64_t)tok * astride,
                                 act_bytes(a.nb), qbar);
                    }
                }
            }
            if (__syncthreads_or(bad)) {
                if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
                my_tiles = 0;
                cta_units = 0;
            }
        }
    } else {
        const uint32_t gid = group * gridDim.x + blockIdx.x;
        first = a.t0 + gid;
        step = gridDim.x * G;
        my_tiles = a.tiles_q + (gid < a.tiles_r ? 1u : 0u);  // ceil((ntiles - gid) / step), host-divided
    }
    const uint32_t nitems = my_tiles * nchunk;
    const uint64_t tile_bytes = (uint64_t)a.nb * CB;
    const uint32_t bar_full = 1 + group, bar_free = 1 + G + group, nbar = 32 * S;

    // Item k = chunk k % nchunk (bc super-blocks) of this group's tile k / nchunk.
    // Lane 0 issues the items in order; (ic, itt, itile, ist) follow the next
    // one so that no issue divides.
    auto tile_ptr = [&](uint32_t tt) -> const uint8_t * {
        if constexpr (MOE) {
            const uint32_t s = tt / a.tiles_per_mat;
            return a.w + (uint64_t)sids[a.slots ? s - s_lo : s] * a.mat_stride +
                   (uint64_t)(tt - s * a.tiles_per_mat) * tile_bytes;
        } else {
            return a.w + tt * tile_bytes;
        }
    };
    uint32_t ic = 0, itt = first, ist = 0, iss = 0;
    const uint8_t *itile = nullptr;
    auto issue_next = [&]() {
        if (ic == 0) itile = tile_ptr(itt);
        const uint32_t nbytes = min(bc, nblk - ic * bc) * CB;
        uint64_t *bar = &bars[ist];
        mbar_arrive_expect_tx(bar, nbytes);
        bulk_g2s(ring + ist * a.stage_bytes, itile + (uint64_t)(b_lo + ic * bc) * CB, nbytes, bar);
        iss++;
        if (++ist == a.nstages) ist = 0;
        if (++ic == nchunk) {
            ic = 0;
            itt += step;
        }
    };
    // GEMV: weights do not depend on the previous kernel, so they stream first.
    if (lane == 0) {
        for (uint32_t st = 0; st < a.nstages; st++) mbar_init(&bars[st], 1);
        fence_mbar_init();
        while (iss < nitems && iss < a.nstages) issue_next();
    }
    // The fp32 activations' lines fetched into L2 now, so that their loads
    // after the wait hit L2: a hint only (L2 is where every write lands, so a
    // line the previous grid still writes is simply updated there); the
    // grid's CTAs share the lines out.
    if (MODE == IN_F32 && a.pf_x) {
        const uint32_t lines = a.nb * 8u;  // 128-byte lines per vector
        for (uint32_t v = 0; v < a.nvec; v++)
            for (uint32_t l = blockIdx.x * blockDim.x + threadIdx.x; l < lines; l += gridDim.x * blockDim.x)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(a.x[v] + 32u * l));
    }
    // The activations do: wait for the grid that wrote them, then stage them.
    grid_dependency_wait();
    const uint32_t tp_e = a.npeers ? *a.epoch + 1u : 0u;  // this call's epoch (row split, expert parallelism)
    const uint32_t nb = a.nb;
    bool failed = false;
    if constexpr (MODE == IN_MOE_H) {
        // one warp per (slot, 256-block) of this CTA's slots: the exact Q8_K
        // quantization of h
        const uint32_t upj = JOBS ? NV : 1u, nimg = cta_units * upj;
        for (uint32_t wb = warp; wb < nimg * nb; wb += nwarps) {
            const uint32_t q = wb / nb, b = wb % nb, j = q / upj, v = q - j * upj;
            if (JOBS && v >= jinfo[j]) continue;
            const uint32_t s = JOBS ? jinfo[MOE_MAXK + j * NV + v] : s_lo + q;
            uint8_t *av = act + q * astride;
            q8k_block(a.gu + s * a.gu_stride + 256u * b, reinterpret_cast<int8_t *>(av + 256u * b),
                      reinterpret_cast<int16_t *>(av + 256u * nb + 32u * b),
                      reinterpret_cast<float *>(av + 288u * nb + 4u * b), lane);
        }
    } else if (MODE == IN_MOE_X && (a.qx_image || a.slots)) {
        if (!mbar_wait_bounded(reinterpret_cast<uint64_t *>(smem + MOE_QX_BAR_OFF), 0, WAIT_LIMIT_NS)) {
            // record it, let this warp's weight copies land (bounded), issue no
            // more; the tile loop keeps its barrier protocol so the CTA exits
            if (lane == 0) {
                atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                for (uint32_t p = 0; p < nitems && p < a.nstages; p++)
                    mbar_wait_bounded(&bars[p], 0, WAIT_LIMIT_NS);
            }
            failed = true;
            __syncwarp();
        }
    } else if constexpr (MODE == IN_F32 || MODE == IN_MOE_X) {
        // one warp per (vector, 256-block): the exact Q8_K quantization.  A
        // warp loads up to QB of its blocks at once, so that the whole of x is
        // in flight in one round instead of one L2 round trip per block.
        constexpr int QB = 2;
        for (uint32_t v = 0; v < a.nvec; v++) {
            uint8_t *av = act + v * astride;
            for (uint32_t b0 = warp; b0 < nb; b0 += nwarps * QB) {
                float xv[QB][8];
#pragma unroll
                for (int j = 0; j < QB; j++) {
                    const uint32_t b = b0 + j * nwarps;
                    if (b < nb) {
                        const float4 *xp = reinterpret_cast<const float4 *>(a.x[v] + 256u * b) + 2 * lane;
                        const float4 p0 = xp[0], p1 = xp[1];
                        xv[j][0] = p0.x, xv[j][1] = p0.y, xv[j][2] = p0.z, xv[j][3] = p0.w;
                        xv[j][4] = p1.x, xv[j][5] = p1.y, xv[j][6] = p1.z, xv[j][7] = p1.w;
                    }
                }
#pragma unroll
                for (int j = 0; j < QB; j++) {
                    const uint32_t b = b0 + j * nwarps;
                    if (b < nb)
                        q8k_block_regs(xv[j], reinterpret_cast<int8_t *>(av + 256u * b),
                                       reinterpret_cast<int16_t *>(av + 256u * nb + 32u * b),
                                       reinterpret_cast<float *>(av + 288u * nb + 4u * b), lane);
                }
            }
        }
    } else if (a.qx_image) {
        // one Q8_K vector as a ready image (made by the kernel before): one bulk copy
        if (threadIdx.x == 0) {
            uint64_t *qbar = reinterpret_cast<uint64_t *>(smem + MOE_QX_BAR_OFF);
            mbar_init(qbar, 1);
            fence_mbar_init();
            mbar_arrive_expect_tx(qbar, act_bytes(nb));
            bulk_g2s(act, a.qx_image, act_bytes(nb), qbar);
            if (!mbar_wait_bounded(qbar, 0, WAIT_LIMIT_NS)) {
                atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                failed = true;
            }
        }
        failed = __syncthreads_or(failed);
        if (failed && lane == 0)  // let this warp's weight copies land (bounded) before the tiles are skipped
            for (uint32_t p = 0; p < nitems && p < a.nstages; p++) mbar_wait_bounded(&bars[p], 0, WAIT_LIMIT_NS);
    } else {
        for (uint32_t v = 0; v < a.nvec; v++) {
            uint8_t *av = act + v * astride;
            const uint4 *qs = reinterpret_cast<const uint4 *>(a.xs[v]);
            for (uint32_t j = threadIdx.x; j < nb * 16; j += blockDim.x) reinterpret_cast<uint4 *>(av)[j] = qs[j];
            const uint32_t *bs = reinterpret_cast<const uint32_t *>(a.xb[v]);
            for (uint32_t j = threadIdx.x; j < nb * 8; j += blockDim.x)
                reinterpret_cast<uint32_t *>(av + 256 * nb)[j] = bs[j];
            for (uint32_t j = threadIdx.x; j < nb; j += blockDim.x)
                reinterpret_cast<float *>(av + 288 * nb)[j] = a.xd[v][j];
        }
    }
    __syncthreads();

    uint32_t k = 0, kst = 0, kph = 0;  // item k's ring stage and mbarrier phase
    for (uint32_t ti = 0; ti < my_tiles; ti++) {
        const uint32_t tt = first + ti * step;
        // MoE: slot ms of the choice, tile mt of its matrix
        uint32_t ms = 0, mt = tt;
        if constexpr (MOE) {
            ms = tt / a.tiles_per_mat;
            mt = tt - ms * a.tiles_per_mat;
        }
        const uint8_t *tact =
            (MODE == IN_MOE_H || (MODE == IN_MOE_X && a.slots)) ? act + (ms - s_lo) * (JOBS ? NV : 1u) * astride : act;
        const uint32_t nvu = JOBS ? jinfo[ms - s_lo] : a.nvec;  // this unit's vectors
        float acc[NV][4], corr[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) {
            corr[v] = 0.0f;
#pragma unroll
            for (int m = 0; m < 4; m++) acc[v][m] = 0.0f;
        }
        float *mine = gscratch + (slot ? (slot - 1) * worker_floats : 0u);
        if (slot > 0 && ti > 0) named_sync(bar_free, nbar);  // slot 0 has read the previous tile
        for (uint32_t c = 0; c < nchunk; c++, k++) {
            const uint32_t st = kst, ph = kph;  // = k % nstages, (k / nstages) & 1
            if (++kst == a.nstages) {
                kst = 0;
                kph ^= 1u;
            }
            if (!failed) {
                const bool ok = mbar_wait_bounded(&bars[st], ph, WAIT_LIMIT_NS);
                if (__any_sync(0xffffffffu, !ok)) {
                    // Record the timeout, let copies in flight land (bounded), stop
                    // issuing; keep the barrier protocol so the CTA still exits.
                    if (lane == 0) {
                        atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                        for (uint32_t p = k; p < nitems && p < k + a.nstages; p++)
                            mbar_wait_bounded(&bars[p % a.nstages], (p / a.nstages) & 1u, WAIT_LIMIT_NS);
                    }
                    failed = true;
                    __syncwarp();
                }
            }
            const uint32_t ncols = min(bc, nblk - c * bc);
            for (uint32_t qq = 0; qq < ncols; qq++) {
                const uint32_t q = c * bc + qq, i = b_lo + q;
                const uint8_t *col = ring + st * a.stage_bytes + qq * CB;
                // the block's weights once, then the vectors one at a time, each
                // vector's lane sums consumed by its chain (or handed to slot 0)
                auto step = [&](int v, const int (&s)[4], float cd, float ct) {
                    if (slot == 0) {
#pragma unroll
                        for (int m = 0; m < 4; m++) acc[v][m] = __fmaf_rn(cd, lane_f<DT>(s[m]), acc[v][m]);
                        corr[v] = __fadd_rn(corr[v], ct);
                    } else {
                        float *e = mine + (q * NV + v) * CHAIN_FLOATS;
                        *reinterpret_cast<float4 *>(e + 64 * g + 4 * r) =
                            make_float4(lane_f<DT>(s[0]), lane_f<DT>(s[1]), lane_f<DT>(s[2]), lane_f<DT>(s[3]));
                        if (g == 0) {
                            e[128 + r] = cd;
                            e[144 + r] = ct;
                        }
                    }
                };
                if constexpr (DT == 0) {
                    Q4KWeights wt;
                    q4k_weights(col, g, r, wt);
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        if (v >= (int)nvu) break;
                        int s[4];
                        float cd, ct;
                        q4k_dot(wt, g, i, a.nb, tact + v * astride, s, cd, ct);
                        step(v, s, cd, ct);
                    }
                } else {
                    Q6KWeights wt;
                    q6k_weights(col, g, r, wt);
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        if (v >= (int)nvu) break;
                        int s[4];
                        float cd, ct;
                        q6k_dot(wt, g, i, a.nb, tact + v * astride, s, cd, ct);
                        step(v, s, cd, ct);
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && !failed && k + a.nstages < nitems) {
                fence_proxy_async();
                issue_next();  // item k + nstages, into the stage just consumed
            }
        }
        if (S > 1) {
            if (slot > 0) {
                named_arrive(bar_full, nbar);
            } else {
                named_sync(bar_full, nbar);
                // continue the chain over the other slots' blocks, in block order
                for (uint32_t ws = 1; ws < S; ws++) {
                    const float *src = gscratch + (ws - 1) * worker_floats;
                    const uint32_t n_ws = ((a.nb * (ws + 1)) >> SL) - ((a.nb * ws) >> SL);
                    for (uint32_t q = 0; q < n_ws; q++)
#pragma unroll
                        for (int v = 0; v < NV; v++) {
                            if (v >= (int)nvu) break;
                            const float *e = src + (q * NV + v) * CHAIN_FLOATS;
                            const float4 f = *reinterpret_cast<const float4 *>(e + 64 * g + 4 * r);
                            const float c = e[128 + r];
                            acc[v][0] = __fmaf_rn(c, f.x, acc[v][0]);
                            acc[v][1] = __fmaf_rn(c, f.y, acc[v][1]);
                            acc[v][2] = __fmaf_rn(c, f.z, acc[v][2]);
                            acc[v][3] = __fmaf_rn(c, f.w, acc[v][3]);
                            corr[v] = __fadd_rn(corr[v], e[144 + r]);
                        }
                }
                if (ti + 1 < my_tiles) named_arrive(bar_free, nbar);
            }
        }
        if (slot == 0) {
            // 8-lane tree ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), then minus the correction.
            const uint32_t row = mt * TILE_ROWS + r;
#pragma unroll
            for (int v = 0; v < NV; v++) {
                float x[4];
#pragma unroll
                for (int m = 0; m < 4; m++) x[m] = __fadd_rn(acc[v][m], __shfl_down_sync(0xffffffffu, acc[v][m], 16));
                const float yv = __fsub_rn(__fadd_rn(__fadd_rn(x[0], x[2]), __fadd_rn(x[1], x[3])), corr[v]);
                float *dst = MOE ? a.out[0] + (JOBS ? jinfo[MOE_MAXK + (ms - s_lo) * NV + v] : ms) * a.out_stride
                                 : a.out[v];
                if (MODE == IN_MOE_H && a.npeers) {
                    // this rank's expert output goes to every rank's receive buffer (NVLink peer stores)
                    if (g == 0 && row >= a.r0 && row < a.r1) {
                        const uint64_t o = (uint64_t)(tp_e & 1u) * a.ep_half +
                                           (uint64_t)__ldcg(a.slot_global + ms) * a.out_stride + row;
                        const unsigned long long pr = ((unsigned long long)tp_e << 32) | __float_as_uint(yv);
                        for (uint32_t p = 0; p < a.npeers; p++)
                            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a.peer_recv[p] + o), "l"(pr)
                                         : "memory");
                    }
                } else if (MODE == IN_MOE_X && a.swiglu) {
                    // rows r < 8 are gate rows, rows r + 8 the up rows of the
                    // same outputs: h = silu(gate) * up (smollm_chat.rs:357-359)
                    const float up = __shfl_down_sync(0xffffffffu, yv, 8);
                    const uint32_t j = mt * 8 + r;
                    if (g == 0 && r < 8 && 2 * j < a.r1 && v < (int)nvu) dst[j] = silu_mul(yv, up);
                } else if (g == 0 && v < (int)nvu && row >= a.r0 && row < a.r1) {
                    if (!MOE && a.npeers) {
                        // the row shard goes straight into every rank's receive buffer (NVLink peer stores)
                        const uint64_t o = (uint64_t)(tp_e & 1u) * a.nvec * a.tp_rows +
                                           (uint64_t)v * a.tp_rows + a.row_off + row;
                        const unsigned long long pr = ((unsigned long long)tp_e << 32) | __float_as_uint(yv);
                        for (uint32_t p = 0; p < a.npeers; p++)
                            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a.peer_recv[p] + o), "l"(pr)
                                         : "memory");
                    } else {
                        dst[row] = yv;
                    }
                }
            }
        }
    }
    if constexpr (!MOE) {
        if (a.npeers) tp_gather(a, tp_e);
    }
}

#define SG_TINST1(DT, NV)                                                                          \
    template __global__ void gemv_tiled_kernel<DT, NV, IN_Q8K>(const __grid_constant__ TGemvArgs); \
    template __global__ void gemv_tiled_kernel<DT, NV, IN_F32>(const __grid_constant__ TGemvArgs);
#define SG_TINST(DT)                                                                                        \
    SG_TINST1(DT, 1) SG_TINST1(DT, 2) SG_TINST1(DT, 4) SG_TINST1(DT, 8)                                     \
    template __global__ void gemv_tiled_kernel<DT, 1, IN_MOE_X>(const __grid_constant__ TGemvArgs); \
    template __global__ void gemv_tiled_kernel<DT, 1, IN_MOE_H>(const __grid_constant__ TGemvArgs); \
    template __global__ void gemv_tiled_kernel<DT, 4, IN_MOE_X>(const __grid_constant__ TGemvArgs); \
    template __global__ void gemv_tiled_kernel<DT, 4, IN_MOE_H>(const __grid_constant__ TGemvArgs); \
    template __global__ void gemv_tiled_kernel<DT, 8, IN_MOE_X>(const __grid_constant__ TGemvArgs); \
    template __global__ void gemv_tiled_kernel<DT, 8, IN_MOE_H>(const __grid_constant__ TGemvArgs);
SG_TINST(0)
SG_TINST(1)

// GGUF rows <-> TILED16 (inverse = 1: src is TILED16, dst GGUF rows).
// One thread per (row, super-block); padding rows of dst are left as they are.
__global__ void repack_tiled16_kernel(int dt, const uint8_t *src, uint64_t rows, uint32_t nb, uint8_t *dst,
                                      int inverse, uint64_t rpg, uint64_t dgr, uint64_t off) {
    const uint64_t id = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * nb) return;
    const uint64_t row = id / nb, trow = (row / rpg) * dgr + off + row % rpg;
    const uint32_t i = (uint32_t)(id % nb), r = (uint32_t)(trow % TILE_ROWS);
    const uint32_t bb = dt == 0 ? 144u : 210u, cb = tiled_col_bytes(dt);
    const uint64_t g_off = (row * nb + i) * bb;
    const uint64_t t_off = (trow / TILE_ROWS) * (uint64_t)nb * cb + (uint64_t)i * cb;
    // (offset in the GGUF block, offset in the tile column, length); the quant
    // bytes move in 16-byte chunks to their swizzled slots
    uint32_t seg[16][3];
    int nseg = 0;
    if (dt == 0) {
        seg[nseg][0] = 0, seg[nseg][1] = 2048 + 16 * r, seg[nseg++][2] = 16;
        for (uint32_t c = 0; c < 8; c++) seg[nseg][0] = 16 + 16 * c, seg[nseg][1] = 128 * r + 16 * q4k_chunk(c, r), seg[nseg++][2] = 16;
    } else {
        for (uint32_t c = 0; c < 12; c++) seg[nseg][0] = 16 * c, seg[nseg][1] = 192 * r + 16 * q6k_chunk(c, r), seg[nseg++][2] = 16;
        seg[nseg][0] = 192, seg[nseg][1] = 3072 + 16 * r, seg[nseg++][2] = 16;
        seg[nseg][0] = 208, seg[nseg][1] = 3328 + 2 * r, seg[nseg++][2] = 2;
    }
    for (int sgi = 0; sgi < nseg; sgi++)
        for (uint32_t b = 0; b < seg[sgi][2]; b++) {
            if (inverse)
                dst[g_off + seg[sgi][0] + b] = src[t_off + seg[sgi][1] + b];
            else
                dst[t_off + seg[sgi][1] + b] = src[g_off + seg[sgi][0] + b];
        }
}

}  // namespace sg
