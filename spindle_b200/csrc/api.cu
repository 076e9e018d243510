// api.cu — the C ABI of include/spindle_gpu.h: argument checks, launch plans
// and kernel dispatch.  Host code only; kernels live in the other .cu files.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>
#include <cmath>

#include "gemv_q8k.cuh"
#include "gemv_tiled.cuh"
#include "gemv_list.cuh"
#include "kernels.cuh"
#include "moe.cuh"
#include "decode.cuh"
#include "gemv_float.cuh"
#include "gemm_batch.cuh"
#include "gemm_tc.cuh"

using namespace sg;

namespace {

thread_local char g_err[256] = "";

sg_status cuda_fail(cudaError_t e, const char *what) {
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return SG_ERR_CUDA;
}

#define CK(call)                                       \
    do {                                               \
        cudaError_t e_ = (call);                       \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

std::atomic<int> g_int_enabled{0};  // 0 = undecided, 1 = on, 2 = off

struct DevInfo {
    int sms = 0;
    bool attrs_set = false;
    bool list_attr = false;
};
DevInfo g_dev[64];
std::mutex g_mu;

sg_status dev_info(DevInfo **out) {
    int d;
    CK(cudaGetDevice(&d));
    if (d < 0 || d >= 64) return SG_ERR_INVALID;
    DevInfo &di = g_dev[d];
    if (!di.sms) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!di.sms) CK(cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d));
    }
    *out = &di;
    return SG_OK;
}

inline uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }
inline bool aligned(const void *p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// ---- GEMV kernel table -----------------------------------------------------

typedef void (*gemv_fn)(const GemvArgs);

template <int DT, bool DBG>
gemv_fn pick(int nv, int cpt) {
    switch (cpt) {
    case 1:
        switch (nv) {
        case 1: return gemv_q8k_kernel<DT, 1, 1, DBG>;
        case 2: return gemv_q8k_kernel<DT, 2, 1, DBG>;
        case 3: return gemv_q8k_kernel<DT, 3, 1, DBG>;
        case 4: return gemv_q8k_kernel<DT, 4, 1, DBG>;
        case 5: return gemv_q8k_kernel<DT, 5, 1, DBG>;
        case 6: return gemv_q8k_kernel<DT, 6, 1, DBG>;
        case 7: return gemv_q8k_kernel<DT, 7, 1, DBG>;
        default: return gemv_q8k_kernel<DT, 8, 1, DBG>;
        }
    case 2:
        switch (nv) {
        case 1: return gemv_q8k_kernel<DT, 1, 2, DBG>;
        case 2: return gemv_q8k_kernel<DT, 2, 2, DBG>;
        case 3: return gemv_q8k_kernel<DT, 3, 2, DBG>;
        default: return gemv_q8k_kernel<DT, 4, 2, DBG>;
        }
    case 4: return nv == 1 ? gemv_q8k_kernel<DT, 1, 4, DBG> : gemv_q8k_kernel<DT, 2, 4, DBG>;
    default: return gemv_q8k_kernel<DT, 1, 8, DBG>;
    }
}

gemv_fn pick_gemv(int dt, bool dbg, int nv, int cpt) {
    if (dt == DT_Q4K) return dbg ? pick<DT_Q4K, true>(nv, cpt) : pick<DT_Q4K, false>(nv, cpt);
    return dbg ? pick<DT_Q6K, true>(nv, cpt) : pick<DT_Q6K, false>(nv, cpt);
}

struct Plan {
    int cpt, nv;
    uint32_t R, ntiles, stage_bytes, nstages, sum_stride, grid;
    size_t smem;
    gemv_fn fn;
};

constexpr size_t SMEM_PER_CTA = 110 * 1024;  // two CTAs per SM
constexpr uint32_t STAGE_TARGET = 24 * 1024;
constexpr uint32_t SCRATCH_MAX = 48 * 1024;

sg_status make_plan_uncached(DevInfo *di, int dt, uint32_t nb, uint32_t nrows, uint32_t nvec, bool dbg, Plan *p) {
    sg_status st;
    const uint32_t ncol = nb * 8, bb = dt == DT_Q4K ? 144 : 210, rb = nb * bb;
    int cpt = 1;
    while (ncol > (uint32_t)GEMV_THREADS * cpt) cpt *= 2;
    if (cpt > 8) return SG_ERR_SHAPE;
    const uint32_t nv = nvec < (uint32_t)(8 / cpt) ? nvec : (uint32_t)(8 / cpt);
    const uint32_t P = cpt == 1 ? GEMV_THREADS / ncol : 1;
    const uint32_t stride = 8 * (nb | 1u);
    uint32_t R = STAGE_TARGET / rb;
    R = R < P ? P : R / P * P;
    while (R > P && gemv_scratch_bytes(R, nv, nb, stride) > SCRATCH_MAX) R -= P;
    // Small matrices: split finer so that every SM gets work.
    const uint32_t want_tiles = (uint32_t)di->sms * 2;
    if ((nrows + R - 1) / R < want_tiles) {
        uint32_t r = (nrows + want_tiles - 1) / want_tiles;
        r = (r + P - 1) / P * P;
        if (r < R) R = r;
    }
    if (R == 0) R = 1;
    uint32_t stage = (uint32_t)align_up((uint64_t)R * rb + 48, 128);
    uint32_t nst = 4;
    size_t smem = 128 + (size_t)nst * stage + gemv_scratch_bytes(R, nv, nb, stride);
    while (smem > SMEM_PER_CTA && nst > 2) {
        nst--;
        smem = 128 + (size_t)nst * stage + gemv_scratch_bytes(R, nv, nb, stride);
    }
    if (smem > 220 * 1024) return SG_ERR_SHAPE;
    p->cpt = cpt;
    p->nv = (int)nv;
    p->R = R;
    p->ntiles = (nrows + R - 1) / R;
    p->stage_bytes = stage;
    p->nstages = nst;
    p->sum_stride = stride;
    p->smem = smem;
    p->fn = pick_gemv(dt, dbg, (int)nv, cpt);
    CK(cudaFuncSetAttribute((const void *)p->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    int occ = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, (const void *)p->fn, GEMV_THREADS, smem));
    if (occ < 1) occ = 1;
    const uint32_t cap = (uint32_t)(di->sms * occ);
    p->grid = p->ntiles < cap ? p->ntiles : cap;
    (void)st;
    return SG_OK;
}

// Plans are cached per device and shape: a launch then costs one hash lookup.
struct PlanKey {
    int dev, dt;
    uint32_t nb, nrows, nvec;
    bool dbg;
    bool operator==(const PlanKey &o) const {
        return dev == o.dev && dt == o.dt && nb == o.nb && nrows == o.nrows && nvec == o.nvec && dbg == o.dbg;
    }
};
struct PlanHash {
    size_t operator()(const PlanKey &k) const {
        uint64_t h = (uint64_t)k.dev * 0x9E3779B97F4A7C15ull ^ (uint64_t)k.dt << 1 ^ (uint64_t)k.dbg;
        h = h * 1099511628211ull ^ k.nb;
        h = h * 1099511628211ull ^ k.nrows;
        h = h * 1099511628211ull ^ k.nvec;
        return (size_t)h;
    }
};
std::unordered_map<PlanKey, Plan, PlanHash> g_plans;

sg_status make_plan(int dt, uint32_t nb, uint32_t nrows, uint32_t nvec, bool dbg, Plan *p) {
    int dev;
    CK(cudaGetDevice(&dev));
    const PlanKey key{dev, dt, nb, nrows, nvec, dbg};
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_plans.find(key);
        if (it != g_plans.end()) {
            *p = it->second;
            return SG_OK;
        }
    }
    DevInfo *di;
    sg_status st = dev_info(&di);
    if (st) return st;
    if ((st = make_plan_uncached(di, dt, nb, nrows, nvec, dbg, p))) return st;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_plans.size() > 4096) g_plans.clear();
    g_plans.emplace(key, *p);
    return SG_OK;
}

sg_status check_mat(const uint8_t *d_base, const sg_mat *m, uint64_t r0, uint64_t r1, int *dt) {
    if (!d_base || !m) return SG_ERR_INVALID;
    if (m->dtype != SG_Q4_K && m->dtype != SG_Q6_K) return SG_ERR_DTYPE;
    if (m->cols == 0 || m->cols % 256 || m->cols > SG_MAX_COLS) return SG_ERR_SHAPE;
    if (r0 > r1 || r1 > m->rows || m->rows > 0xFFFFFFFFull) return SG_ERR_INVALID;
    if (m->layout != SG_LAYOUT_GGUF && m->layout != SG_LAYOUT_TILED16) return SG_ERR_INVALID;
    if (!aligned(d_base + m->offset, 16)) return SG_ERR_ALIGN;
    *dt = m->dtype == SG_Q4_K ? DT_Q4K : DT_Q6K;
    return SG_OK;
}

sg_status check_q8k(const sg_q8k &q, uint64_t n) {
    if (!q.d || !q.qs || !q.bsums || q.n != n) return SG_ERR_INVALID;
    if (!aligned(q.d, 4) || !aligned(q.qs, 16) || !aligned(q.bsums, 4)) return SG_ERR_ALIGN;
    return SG_OK;
}

// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel in the stream finishes; it waits for it (griddepcontrol)
// before reading anything that kernel wrote.
template <typename Args>
cudaError_t launch_pdl(const void *fn, dim3 grid, uint32_t block, size_t smem, cudaStream_t stream, Args *args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *params[] = {args};
    return cudaLaunchKernelExC(&cfg, fn, params);
}

// ---- TILED16 GEMV ------------------------------------------------------------

typedef void (*tgemv_fn)(const TGemvArgs);

uint32_t tiled_nv_inst(int nv) { return nv <= 1 ? 1u : nv == 2 ? 2u : nv <= 4 ? 4u : 8u; }

template <int DT, int MODE>
tgemv_fn pick_tiled_t(int nv) {
    return nv == 1 ? gemv_tiled_kernel<DT, 1, MODE> : nv == 2 ? gemv_tiled_kernel<DT, 2, MODE>
           : nv <= 4 ? gemv_tiled_kernel<DT, 4, MODE> : gemv_tiled_kernel<DT, 8, MODE>;
}

tgemv_fn pick_tiled(int dt, int nv, int mode) {
    if (dt == DT_Q4K) {
        switch (mode) {
        case IN_MOE_X: return nv <= 1 ? gemv_tiled_kernel<0, 1, IN_MOE_X> : nv <= 4 ? gemv_tiled_kernel<0, 4, IN_MOE_X>
                                                                             : gemv_tiled_kernel<0, 8, IN_MOE_X>;
        case IN_MOE_H: return nv <= 1 ? gemv_tiled_kernel<0, 1, IN_MOE_H> : nv <= 4 ? gemv_tiled_kernel<0, 4, IN_MOE_H>
                                                                             : gemv_tiled_kernel<0, 8, IN_MOE_H>;
        case IN_F32: return pick_tiled_t<0, IN_F32>(nv);
        default: return pick_tiled_t<0, IN_Q8K>(nv);
        }
    }
    switch (mode) {
    case IN_MOE_X: return nv <= 1 ? gemv_tiled_kernel<1, 1, IN_MOE_X> : nv <= 4 ? gemv_tiled_kernel<1, 4, IN_MOE_X>
                                                                         : gemv_tiled_kernel<1, 8, IN_MOE_X>;
    case IN_MOE_H: return nv <= 1 ? gemv_tiled_kernel<1, 1, IN_MOE_H> : nv <= 4 ? gemv_tiled_kernel<1, 4, IN_MOE_H>
                                                                         : gemv_tiled_kernel<1, 8, IN_MOE_H>;
    case IN_F32: return pick_tiled_t<1, IN_F32>(nv);
    default: return pick_tiled_t<1, IN_Q8K>(nv);
    }
}

int env_int(const char *name, int dflt) {
    const char *e = getenv(name);
    return e && *e ? atoi(e) : dflt;
}

struct TPlan {
    tgemv_fn fn;
    uint32_t S, bc, nstages, stage_bytes, slot_blocks, grid, warps, nact;
    size_t smem;
};

std::unordered_map<uint64_t, TPlan> g_tplans;

// Launch shape of the tiled GEMV: S warps per tile so that the whole GPU has
// work (small row counts split each tile's super-blocks over more warps),
// a 2-stage ring per warp, CTAs of 8 or 16 warps.
// mode: IN_Q8K, IN_F32, IN_MOE_X or IN_MOE_H; max_slots: the MoE slots the
// launch is sized for (ntiles counts all of them), 0 otherwise.
sg_status tiled_plan(int dt, uint32_t nb, uint32_t ntiles, int nv, int mode, uint32_t max_slots, TPlan *p) {
    int dev;
    CK(cudaGetDevice(&dev));
    const uint64_t key = ((uint64_t)dev << 56) ^ ((uint64_t)mode << 53) ^ ((uint64_t)dt << 52) ^
                         ((uint64_t)max_slots << 48) ^ ((uint64_t)nv << 44) ^ ((uint64_t)nb << 32) ^ ntiles;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_tplans.find(key);
        if (it != g_tplans.end()) {
            *p = it->second;
            return SG_OK;
        }
    }
    DevInfo *di;
    sg_status st = dev_info(&di);
    if (st) return st;
    const uint32_t cb = tiled_col_bytes(dt == DT_Q4K ? 0 : 1);
    // the kernel is instantiated for 1, 2, 4 or 8 vectors; its chain scratch is
    // laid out for that count, so size shared memory for it too
    const uint32_t nv_inst = tiled_nv_inst(nv);
    // CTA width: 16 warps (one CTA per SM) or 8 warps (two per SM, so that the
    // next kernel of a chain can become resident and prefetch its weights
    // while this one drains)
    const uint32_t warps = env_int("SG_TILED_WARPS", 16) == 8 ? 8u : 16u;
    const uint32_t warp_slots = (uint32_t)di->sms * 16u;
    // S warps per tile: the critical warp (slot 0 of the busiest group) does
    // ceil(ntiles / groups) tiles, each of ceil(nb / S) full super-blocks plus
    // the cheap chain steps over the other slots' blocks.  Pick the S with the
    // shortest such path.
    uint32_t S = 1;
    // The kernel's S warps of a tile meet at named barriers 1 + group and
    // 1 + G + group (G = warps / S groups), the second only where a group has
    // a second tile; with 16 warps and S = 2 that would be barrier 16, past
    // the hardware's 0..15, so that S is taken only where no group gets a
    // second tile (ntiles <= SMs * G, in the GEMV and the MoE layouts alike).
    auto s_ok = [&](uint32_t s) {
        return !(s > 1 && 2 * (warps / s) + 1 > 16 && (uint64_t)ntiles > (uint64_t)di->sms * (warps / s));
    };
    const int forced = env_int("SG_TILED_S", 0);
    if ((forced == 1 || forced == 2 || forced == 4 || forced == 8 || forced == 16) && (uint32_t)forced <= warps &&
        s_ok((uint32_t)forced)) {
        S = (uint32_t)forced;
    } else {
        double best = 1e30;
        for (uint32_t s = 1; s <= warps && s <= nb; s *= 2) {
            if (!s_ok(s)) continue;
            const uint64_t groups = warp_slots / s;
            const uint64_t tiles = (ntiles + groups - 1) / groups;
            const double per_tile = (double)((nb + s - 1) / s) + 0.06 * (double)(nb - nb / s) + (s > 1 ? 0.5 : 0.0);
            const double cost = (double)tiles * per_tile;
            if (cost < best * 0.98) {
                best = cost;
                S = s;
            }
        }
    }
    uint32_t ns = (uint32_t)env_int("SG_TILED_STAGES", 2), bc = (uint32_t)env_int("SG_TILED_BC", 2);
    if (ns < 2) ns = 2;
    if (ns > 8) ns = 8;
    // the MoE modes keep the router's choice at the top of the barrier area
    // the barriers stay below the ones the MoE modes and image copies keep at the top
    if (ns * warps * 8 > MOE_QX_BAR_OFF) ns = MOE_QX_BAR_OFF / (warps * 8);
    if (bc < 1) bc = 1;
    // MoE: one CTA per SM, each on a contiguous range of tiles; IN_MOE_H stages
    // h for every slot its range touches (at most this many).
    uint32_t moe_nact = 0, moe_grid = 0;
    if (mode >= IN_MOE_X) {
        moe_grid = ntiles < (uint32_t)di->sms ? ntiles : (uint32_t)di->sms;
        if (moe_grid == 0) moe_grid = 1;
        const uint32_t tpm = max_slots ? ntiles / max_slots : 1, tpc = (ntiles + moe_grid - 1) / moe_grid;
        moe_nact = tpm ? (tpc + tpm - 2) / tpm + 1 : 1;
        if (moe_nact > max_slots) moe_nact = max_slots;
        if (moe_nact == 0) moe_nact = 1;
        if (nv_inst > 1) moe_nact *= nv_inst;  // jobs: nv images per unit
    }
    const uint32_t job_bytes = mode >= IN_MOE_X && nv_inst > 1 ? tiled_job_bytes(nv_inst) : 0u;
    const size_t budget = warps == 16 ? 220 * 1024 : 110 * 1024;
    // Several vectors (plain GEMV): the chain scratch grows with the vector
    // count, and a smaller S makes it larger per slot, so every S is tried
    // with the rings shrunk to fit, and the cheapest that fits is taken (the
    // loop below would fall back to S = 1 for long rows: 56 super-blocks on
    // one warp per tile).
    if (mode < IN_MOE_X && nv_inst > 1 && !(forced == 1 || forced == 2 || forced == 4 || forced == 8 || forced == 16)) {
        double best = 1e30;
        uint32_t bestS = 0;
        for (uint32_t s = 1; s <= warps && s <= nb; s *= 2) {
            if (!s_ok(s)) continue;
            const uint32_t sbk = (nb + s - 1) / s;
            bool fits = false;
            for (uint32_t b = bc < sbk ? bc : sbk; b >= 1 && !fits; b--)
                fits = tiled_smem_bytes(warps, s, 2, b * cb, sbk, nv_inst, nb, nv_inst, 0) <= budget;
            if (!fits) continue;
            const uint64_t groups = warp_slots / s;
            const uint64_t tiles = (ntiles + groups - 1) / groups;
            const double cost = (double)tiles * ((double)sbk + 0.06 * (double)(nb - nb / s) + (s > 1 ? 0.5 : 0.0));
            if (cost < best * 0.98) {
                best = cost;
                bestS = s;
            }
        }
        if (bestS) S = bestS;
    }
    // Fit the CTA in shared memory: fewer stages, then smaller stages, then
    // fewer warps per tile (less chain scratch).
    for (;;) {
        p->S = S;
        p->slot_blocks = (nb + S - 1) / S;
        p->bc = bc < p->slot_blocks ? bc : p->slot_blocks;
        p->nstages = ns;
        p->stage_bytes = p->bc * cb;
        p->smem = tiled_smem_bytes(warps, S, ns, p->stage_bytes, p->slot_blocks, nv_inst, nb,
                                   tiled_nact(mode, nv_inst, moe_nact), job_bytes);
        if (p->smem <= budget) break;
        if (ns > 2)
            ns--;
        else if (bc > 1)
            bc--;
        else if (S > 1)
            S = s_ok(S / 2) ? S / 2 : 1;
        else
            return SG_ERR_SHAPE;
    }
    p->fn = pick_tiled(dt, nv, mode);
    CK(cudaFuncSetAttribute((const void *)p->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    int occ = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, (const void *)p->fn, warps * 32, p->smem));
    if (occ < 1) occ = 1;
    p->warps = warps;
    const uint32_t groups = warps / p->S;
    // every SM pulls its share of the weights: launch a full wave even when
    // some groups get no tile (tiles go to CTAs round-robin)
    const uint32_t need = (ntiles + groups - 1) / groups, cap = (uint32_t)(di->sms * occ);
    p->grid = need < (uint32_t)di->sms ? (ntiles < (uint32_t)di->sms ? ntiles : (uint32_t)di->sms) : (need < cap ? need : cap);
    p->nact = moe_nact;
    if (mode >= IN_MOE_X) p->grid = moe_grid;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_tplans.size() > 4096) g_tplans.clear();
    g_tplans.emplace(key, *p);
    return SG_OK;
}

// One of xq (Q8_K inputs) or x (fp32 inputs, vector b at x + b*ldx) is given.
// With image (one vector): x is the Q8_K shared-memory image made by the
// kernel before (act_bytes(nb) bytes), copied in by one bulk copy.
// Row-split tensor parallelism of one launch: where the rows go and the
// arrival counters (see TGemvArgs).
struct TpSpec {
    uint32_t n;
    uint32_t row_off, rows;                     // this shard's first row; rows of the whole matrix
    unsigned long long *recv[TP_MAX_RANKS];     // every rank's receive buffer
    const unsigned long long *my_recv;
    float *out;                                 // this rank's plain output, vector b at out + b * ldo
    uint64_t ldo;
    unsigned *ticket;
    unsigned *epoch;
};

sg_status launch_tiled(const uint8_t *w, int dt, uint32_t nb, const sg_q8k *xq, const float *x, uint64_t ldx,
                       float *const *outs, uint64_t n_vec, uint64_t r0, uint64_t r1, cudaStream_t stream,
                       const uint8_t *image = nullptr, const TpSpec *tp = nullptr) {
    if (image && n_vec != 1) return SG_ERR_INVALID;
    const uint32_t t0 = (uint32_t)(r0 / TILE_ROWS), t1 = (uint32_t)((r1 + TILE_ROWS - 1) / TILE_ROWS);
    const bool qx = x != nullptr;
    for (uint64_t g = 0; g < n_vec;) {
        // as many vectors per launch as the shared-memory plan can stage
        int nv = (int)(n_vec - g < TGEMV_MAXV ? n_vec - g : TGEMV_MAXV);
        TPlan p;
        sg_status st;
        while ((st = tiled_plan(dt, nb, t1 - t0, nv, qx ? IN_F32 : IN_Q8K, 0, &p)) == SG_ERR_SHAPE && nv > 1)
            nv = nv > 4 ? 4 : nv / 2;
        if (st) return st;
        // a row-split call is one launch on every rank (each launch is one arrival round)
        if (tp && (uint64_t)nv < n_vec) return SG_ERR_SHAPE;
        TGemvArgs a;
        memset(&a, 0, sizeof a);
        a.w = w;
        a.nb = nb;
        a.t0 = t0;
        a.ntiles = t1 - t0;
        a.r0 = (uint32_t)r0;
        a.r1 = (uint32_t)r1;
        a.S = p.S;
        a.s_log2 = ilog2u(p.S);
        {
            const uint32_t step = p.grid * (p.warps >> a.s_log2);  // tile groups in the grid
            a.tiles_q = a.ntiles / step;
            a.tiles_r = a.ntiles % step;
        }
        a.bc = p.bc;
        a.nstages = p.nstages;
        a.stage_bytes = p.stage_bytes;
        a.slot_blocks = p.slot_blocks;
        a.nvec = (uint32_t)nv;
        a.qx_image = image;
        a.pf_x = qx && env_int("SG_GEMV_PFX", 1) ? 1u : 0u;
        for (int v = 0; v < nv; v++) {
            if (qx) {
                a.x[v] = x + (g + v) * ldx;
            } else if (!image) {
                a.xd[v] = xq[g + v].d;
                a.xs[v] = xq[g + v].qs;
                a.xb[v] = xq[g + v].bsums;
            }
            if (outs) a.out[v] = outs[g + v];
        }
        if (tp) {  // one launch per call (checked above), so g == 0 here
            a.npeers = tp->n;
            a.row_off = tp->row_off;
            a.tp_rows = tp->rows;
            a.out[0] = tp->out;
            a.out_stride = tp->ldo;
            for (uint32_t q = 0; q < tp->n; q++) a.peer_recv[q] = tp->recv[q];
            a.my_recv = tp->my_recv;
            a.ticket = tp->ticket;
            a.epoch = tp->epoch;
        }
        CK(launch_pdl((const void *)p.fn, p.grid, p.warps * 32, p.smem, stream, &a));
        g += (uint64_t)nv;
    }
    return SG_OK;
}

// ---- batch GEMM (9..128 vectors) ----------------------------------------------

// QB image (gemm_batch.cuh) of n fp32 vectors x + t * ldx of 256 * nb values.
sg_status launch_q8k_batch(const float *x, uint64_t ldx, uint32_t n, uint32_t nb, uint8_t *qb, cudaStream_t s) {
    if (n == 0 || nb == 0) return SG_OK;
    QbArgs a = {x, ldx, n, nb, qb};
    const uint64_t warps = (uint64_t)n * nb;
    CK(launch_pdl((const void *)q8k_batch_kernel, dim3((uint32_t)((warps + 7) / 8)), 256, 0, s, &a));
    return SG_OK;
}

// Rows r0..r1 of a TILED16 matrix for ntok <= 128 vectors given as a QB image:
// vector t, row r at out + t * ldo + r (swiglu: the packed gate/up form, see
// GemmBatchArgs).  One launch; every weight column is read once.
// Q4_K / Q6_K on the tensor cores (gemm_tc.cu): CTAs of 128 rows x 16 tokens.
sg_status launch_gemm_tc(const uint8_t *w, int dt, uint32_t nb, uint64_t r0, uint64_t r1, const uint8_t *qb,
                         uint32_t ntok, float *out, uint64_t ldo, bool swiglu, cudaStream_t s) {
    static std::atomic<uint64_t> attr_done{0};
    int dev;
    CK(cudaGetDevice(&dev));
    if (!(attr_done.load() >> dev & 1)) {
        CK(cudaFuncSetAttribute((const void *)gemm_tc_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TC_SMEM));
        CK(cudaFuncSetAttribute((const void *)gemm_tc_q6k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                TC6_SMEM));
        attr_done.fetch_or(1ull << dev);
    }
    GemmTcArgs a;
    memset(&a, 0, sizeof a);
    a.w = w;
    a.nb = nb;
    a.t0 = (uint32_t)(r0 / TILE_ROWS);
    a.ntiles = (uint32_t)((r1 + TILE_ROWS - 1) / TILE_ROWS) - a.t0;
    a.r0 = (uint32_t)r0;
    a.r1 = (uint32_t)r1;
    a.qb = qb;
    a.ntok = ntok;
    a.out = out;
    a.ldo = ldo;
    a.swiglu = swiglu ? 1u : 0u;
    const dim3 grid((a.ntiles + 7) / 8, (ntok + TC_TOK - 1) / TC_TOK);
    if (dt == DT_Q4K)
        CK(launch_pdl((const void *)gemm_tc_q4k_kernel, grid, TC_THREADS, TC_SMEM, s, &a));
    else
        CK(launch_pdl((const void *)gemm_tc_q6k_kernel, grid, TC_THREADS, TC6_SMEM, s, &a));
    return SG_OK;
}

sg_status launch_gemm_batch(const uint8_t *w, int dt, uint32_t nb, uint64_t r0, uint64_t r1, const uint8_t *qb,
                            uint32_t ntok, float *out, uint64_t ldo, bool swiglu, cudaStream_t s) {
    if (ntok == 0 || r1 <= r0) return SG_OK;
    if (ntok > QB_MAX_TOK) return SG_ERR_SHAPE;
    // tensor cores: Q4_K by default, Q6_K with SG_GEMM_TC=2; SG_GEMM_TC=0 keeps
    // both on the dp4a kernel
    const int tc = env_int("SG_GEMM_TC", 1);
    if ((dt == DT_Q4K && tc >= 1) || (dt == DT_Q6K && tc >= 2))
        return launch_gemm_tc(w, dt, nb, r0, r1, qb, ntok, out, ldo, swiglu, s);

    static std::atomic<uint64_t> attr_done{0};
    int dev;
    CK(cudaGetDevice(&dev));
    if (!(attr_done.load() >> dev & 1)) {
        for (const void *fn : {(const void *)gemm_batch_kernel<0, 4>, (const void *)gemm_batch_kernel<1, 4>,
                               (const void *)gemm_batch_kernel<0, 8>, (const void *)gemm_batch_kernel<1, 8>})
            CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr_done.fetch_or(1ull << dev);
    }
    static const int tpw = env_int("SG_GEMM_TPW", 4) == 8 ? 8 : 4;
    const uint32_t cons = gb_consumers(tpw);
    DevInfo *di;
    sg_status st = dev_info(&di);
    if (st) return st;
    GemmBatchArgs a;
    memset(&a, 0, sizeof a);
    a.w = w;
    a.nb = nb;
    a.t0 = (uint32_t)(r0 / TILE_ROWS);
    a.ntiles = (uint32_t)((r1 + TILE_ROWS - 1) / TILE_ROWS) - a.t0;
    a.r0 = (uint32_t)r0;
    a.r1 = (uint32_t)r1;
    a.qb = qb;
    a.ntok = ntok;
    // the kernel takes one QB group (64 vectors) per CTA row (blockIdx.y): planned for the largest
    const uint32_t gtok = ntok < GB_MAX_TOK ? ntok : GB_MAX_TOK, ngroups = (ntok + QB_GROUP - 1) / QB_GROUP;
    a.nq = 1;
    while (a.nq * (uint32_t)tpw < gtok) a.nq *= 2;
    a.tps = cons / a.nq;
    const uint32_t cb = tiled_col_bytes(dt);
    a.stage_bytes = a.tps * cb + qb_block_bytes(gtok);
    const uint32_t budget = 220u * 1024u - GB_BAR_BYTES;
    a.nstages = budget / a.stage_bytes;
    if (a.nstages > GB_MAX_STAGES) a.nstages = GB_MAX_STAGES;
    if (a.nstages < 2) return SG_ERR_SHAPE;
    a.out = out;
    a.ldo = ldo;
    a.swiglu = swiglu ? 1u : 0u;
    const uint32_t nsteps = (a.ntiles + a.tps - 1) / a.tps;
    const uint32_t grid = nsteps < (uint32_t)di->sms ? nsteps : (uint32_t)di->sms;
    const void *fn = tpw == 4 ? (dt == DT_Q4K ? (const void *)gemm_batch_kernel<0, 4> : (const void *)gemm_batch_kernel<1, 4>)
                              : (dt == DT_Q4K ? (const void *)gemm_batch_kernel<0, 8> : (const void *)gemm_batch_kernel<1, 8>);
    CK(launch_pdl(fn, dim3(grid, ngroups), cons * 32, GB_BAR_BYTES + a.nstages * a.stage_bytes, s, &a));
    return SG_OK;
}

sg_status launch_gemv(const uint8_t *d_base, const sg_mat *m, const sg_q8k *xq, float *const *outs,
                      uint64_t n_vec, uint64_t r0, uint64_t r1, int32_t *dbg, cudaStream_t stream) {
    int dt;
    sg_status st = check_mat(d_base, m, r0, r1, &dt);
    if (st) return st;
    if (r1 == r0 || n_vec == 0) return SG_OK;
    if (!xq || !outs) return SG_ERR_INVALID;
    for (uint64_t b = 0; b < n_vec; b++) {
        if ((st = check_q8k(xq[b], m->cols))) return st;
        if (!outs[b] || !aligned(outs[b], 4)) return SG_ERR_INVALID;
    }
    const uint32_t nb = (uint32_t)(m->cols / 256), bb = dt == DT_Q4K ? 144 : 210;
    const uint64_t rb = (uint64_t)nb * bb;
    if (m->layout == SG_LAYOUT_TILED16) {
        if (dbg) return SG_ERR_INVALID;
        return launch_tiled(d_base + m->offset, dt, nb, xq, nullptr, 0, outs, n_vec, r0, r1, stream);
    }
    for (uint64_t g = 0; g < n_vec; g += GEMV_MAXV) {
        const uint32_t nv = (uint32_t)(n_vec - g < GEMV_MAXV ? n_vec - g : GEMV_MAXV);
        Plan p;
        if ((st = make_plan(dt, nb, (uint32_t)(r1 - r0), nv, dbg != nullptr, &p))) return st;
        GemvArgs a;
        memset(&a, 0, sizeof a);
        a.w = d_base + m->offset;
        a.tma_limit = (m->rows * rb) & ~15ull;
        a.nb = nb;
        a.rb = (uint32_t)rb;
        a.r0 = (uint32_t)r0;
        a.nrows = (uint32_t)(r1 - r0);
        a.R = p.R;
        a.ntiles = p.ntiles;
        a.stage_bytes = p.stage_bytes;
        a.nstages = p.nstages;
        a.sum_stride = p.sum_stride;
        a.nvec = nv;
        for (uint32_t v = 0; v < nv; v++) {
            a.xd[v] = xq[g + v].d;
            a.xs[v] = xq[g + v].qs;
            a.xb[v] = xq[g + v].bsums;
            a.out[v] = outs[g + v];
        }
        a.dbg_sums = dbg;
        p.fn<<<p.grid, GEMV_THREADS, p.smem, stream>>>(a);
        CK(cudaGetLastError());
    }
    return SG_OK;
}

// ---- MoE layer ---------------------------------------------------------------

inline bool kquant(int32_t dt) { return dt == SG_Q4_K || dt == SG_Q6_K; }
inline bool cols_ok(uint64_t c) { return c && c % 256 == 0 && c <= SG_MAX_COLS; }

uint64_t tiled_bytes(int32_t dt, uint64_t rows, uint64_t cols) {
    uint64_t b = 0;
    return sg_tiled16_bytes(dt, rows, cols, &b) == SG_OK ? b : 0;
}

sg_status check_moe(const sg_moe *m) {
    if (!m || !m->router || !m->gate_up || !m->down) return SG_ERR_INVALID;
    if (!kquant(m->gate_up_dtype) || !kquant(m->down_dtype)) return SG_ERR_DTYPE;
    if (!cols_ok(m->dim) || !cols_ok(m->n_ff)) return SG_ERR_SHAPE;
    if (m->n_expert == 0 || m->n_expert > ROUTER_MAX_EXPERTS || m->n_used == 0 || m->n_used > m->n_expert)
        return SG_ERR_INVALID;
    if (m->n_used > SG_MOE_MAX_USED) return SG_ERR_SHAPE;
    if (m->gate_up_stride < tiled_bytes(m->gate_up_dtype, 2 * m->n_ff, m->dim) ||
        m->down_stride < tiled_bytes(m->down_dtype, m->dim, m->n_ff))
        return SG_ERR_INVALID;
    if (!aligned(m->router, 16) || !aligned(m->gate_up, 16) || !aligned(m->down, 16) || m->gate_up_stride % 16 ||
        m->down_stride % 16)
        return SG_ERR_ALIGN;
    if (m->shared_gate_up) {
        if (!m->shared_down) return SG_ERR_INVALID;
        if (!kquant(m->shared_gate_up_dtype) || !kquant(m->shared_down_dtype)) return SG_ERR_DTYPE;
        if (!cols_ok(m->shared_n_ff)) return SG_ERR_SHAPE;
        if (!aligned(m->shared_gate_up, 16) || !aligned(m->shared_down, 16) || !aligned(m->shared_gate, 16))
            return SG_ERR_ALIGN;
    }
    return SG_OK;
}

// Scratch of sg_moe_forward, each piece 256-byte aligned.
struct MoeScratch {
    uint64_t sel, shsel, scale, logits, qx, h, y, hsh, ysh, total;
};

MoeScratch moe_scratch(const sg_moe *m) {
    MoeScratch L;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const bool sh = m->shared_gate_up != nullptr;
    L.sel = take(sizeof(sg_moe_choice));
    L.shsel = take(sizeof(sg_moe_choice));
    L.scale = take(4);
    L.logits = take(m->n_expert * 4);
    L.qx = take(act_bytes((uint32_t)(m->dim / 256)));
    L.h = take(m->n_used * m->n_ff * 4);
    L.y = take(m->n_used * m->dim * 4);
    L.hsh = take(sh ? m->shared_n_ff * 4 : 0);
    L.ysh = take(sh ? m->dim * 4 : 0);
    L.total = off;
    return L;
}

// Scratch of the batched layer (moe_forward_batch) for n_tok tokens.
struct MoeBatchScratch {
    uint64_t choices, slot_base, slots, n_slots, slots_sh, n_slots_sh, shsel, scale, logits, qx, h, y, hsh, ysh;
    uint64_t slots_local, slot_global, n_local, ticket, jobs, n_jobs, total;
};

// Jobs of the batched layer (the slots of an expert grouped, up to job_max
// per job): at most one per slot and at most n_slots / job_max + n_expert.
uint64_t moe_max_jobs(uint64_t n_slots, uint64_t n_expert, uint64_t job_max) {
    const uint64_t b = n_slots / job_max + n_expert;
    return b < n_slots ? b : n_slots;
}

MoeBatchScratch moe_batch_scratch(const sg_moe *m, uint64_t n_tok) {
    MoeBatchScratch L;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const bool sh = m->shared_gate_up != nullptr;
    const uint64_t slots = n_tok * m->n_used;
    L.choices = take(n_tok * sizeof(sg_moe_choice));
    L.slot_base = take(n_tok * 4);
    L.slots = take(slots * 8);
    L.n_slots = take(4);
    L.slots_sh = take(sh ? n_tok * 8 : 0);
    L.n_slots_sh = take(4);
    L.shsel = take(sizeof(sg_moe_choice));
    L.scale = take(n_tok * 4);
    L.logits = take(n_tok * m->n_expert * 4);
    L.qx = take(n_tok * act_bytes((uint32_t)(m->dim / 256)));
    L.h = take(slots * m->n_ff * 4);
    L.y = take(slots * m->dim * 4);
    L.hsh = take(sh ? n_tok * m->shared_n_ff * 4 : 0);
    L.ysh = take(sh ? n_tok * m->dim * 4 : 0);
    L.slots_local = take(slots * 8);  // expert parallelism: this rank's slots
    L.slot_global = take(slots * 4);
    L.n_local = take(4);
    L.ticket = take(4);  // the select kernel's last-CTA count (zeroed by the router kernel)
    L.jobs = take(moe_max_jobs(slots, m->n_expert, 4) * MOE_JOB_INTS * 4);  // sized for the smallest jobs
    L.n_jobs = take(4);
    L.total = off;
    return L;
}

// The expert choice of a grouped launch: made from the router's logits in the
// kernel (IN_MOE_X with logits), or read from `sel`.
struct MoeRoute {
    const float *logits;
    sg_moe_choice *sel_out;
    float *probs;
    uint32_t n_used;
    int32_t norm;
    float prune;
};

// One grouped launch of the tiled GEMV over the chosen experts (IN_MOE_X or IN_MOE_H).
// Batched form: the slots come from a device table of (expert, token) pairs.
struct MoeSlots {
    const int32_t *slots;
    const uint32_t *n_slots;
    const uint8_t *qx_tokens;  // IN_MOE_X: the tokens' Q8_K images
    // jobs mode (TGemvArgs::jobs): the select kernel's expert jobs, each unit
    // job_nv vectors; max_slots then counts jobs
    const int32_t *jobs;
    const uint32_t *n_jobs;
    uint32_t job_nv;
    // IN_MOE_H with expert parallelism: slot outputs to every rank (see TGemvArgs)
    uint32_t npeers;
    const uint32_t *slot_global;
    unsigned long long *recv[TP_MAX_RANKS];
    uint64_t ep_half;
    unsigned *epoch;
};

sg_status launch_moe_group(int32_t dtype, int mode, const uint8_t *w, uint64_t mat_stride, uint64_t rows,
                           uint64_t cols, uint32_t max_slots, uint32_t n_expert, const sg_moe_choice *sel,
                           const MoeRoute *route, const float *x, const uint8_t *qx, const float *h,
                           uint64_t h_stride, float *out, uint64_t out_stride, cudaStream_t stream,
                           const MoeSlots *slots = nullptr) {
    const int dt = dtype == SG_Q4_K ? DT_Q4K : DT_Q6K;
    const uint32_t nb = (uint32_t)(cols / 256), tiles = (uint32_t)((rows + TILE_ROWS - 1) / TILE_ROWS);
    const bool jobs = slots && slots->jobs;
    if (jobs && ((slots->job_nv != 4 && slots->job_nv != 8) || slots->job_nv + 2 > MOE_JOB_INTS || slots->npeers))
        return SG_ERR_INVALID;
    TPlan p;
    sg_status st = tiled_plan(dt, nb, max_slots * tiles, jobs ? (int)slots->job_nv : 1, mode, max_slots, &p);
    if (st) return st;
    if (route && moe_select_bytes(n_expert) > p.warps * p.nstages * p.stage_bytes) return SG_ERR_SHAPE;
    TGemvArgs a;
    memset(&a, 0, sizeof a);
    a.w = w;
    a.nb = nb;
    a.ntiles = max_slots * tiles;
    a.r1 = (uint32_t)rows;
    a.S = p.S;
    a.s_log2 = ilog2u(p.S);
    a.bc = p.bc;
    a.nstages = p.nstages;
    a.stage_bytes = p.stage_bytes;
    a.slot_blocks = p.slot_blocks;
    a.nvec = 1;
    a.x[0] = x;
    a.qx_image = qx;
    a.swiglu = mode == IN_MOE_X;  // the packed gate/up tiles interleave 8 gate and 8 up rows
    a.out[0] = out;
    a.sel = sel;
    if (route) {
        a.logits = route->logits;
        a.sel_out = route->sel_out;
        a.probs = route->probs;
        a.n_used = route->n_used;
        a.norm = route->norm;
        a.prune = route->prune;
    }
    a.nact = p.nact;
    a.mat_stride = mat_stride;
    a.out_stride = out_stride;
    a.tiles_per_mat = tiles;
    a.max_slots = max_slots;
    a.n_expert = n_expert;
    a.gu = h;
    a.gu_stride = h_stride;
    if (slots) {
        if (p.nact > MOE_MAXK * (jobs ? tiled_nv_inst((int)slots->job_nv) : 1u)) return SG_ERR_SHAPE;
        if (jobs) {
            a.jobs = slots->jobs;
            a.n_jobs = slots->n_jobs;
            a.job_ints = MOE_JOB_INTS;
        }
        a.slots = slots->slots;
        a.n_slots = slots->n_slots;
        a.qx_tokens = slots->qx_tokens;
        a.sel = nullptr;
        a.qx_image = nullptr;
        if (slots->npeers) {
            a.npeers = slots->npeers;
            a.slot_global = slots->slot_global;
            for (uint32_t q = 0; q < slots->npeers; q++) a.peer_recv[q] = slots->recv[q];
            a.ep_half = slots->ep_half;
            a.epoch = slots->epoch;
        }
    }
    CK(launch_pdl((const void *)p.fn, p.grid, p.warps * 32, p.smem, stream, &a));
    return SG_OK;
}

// Router logits over the whole GPU (a few rows per CTA), plus one CTA for the
// shared expert's gate and one-slot choice when the layer has a shared expert.
sg_status launch_router(const sg_moe *m, const float *x, float *logits, uint8_t *qx, sg_moe_choice *shsel, float *scale,
                        cudaStream_t stream, uint32_t n_tok = 1, uint64_t ldx = 0, unsigned *zero_word = nullptr) {
    static std::atomic<uint64_t> attr_done{0};  // bit d: the smem attribute is set on device d
    int dev;
    CK(cudaGetDevice(&dev));
    if (!(attr_done.load() >> dev & 1)) {
        CK(cudaFuncSetAttribute((const void *)moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                227 * 1024));
        attr_done.fetch_or(1ull << dev);
    }
    DevInfo *di;
    sg_status st = dev_info(&di);
    if (st) return st;
    RouterArgs a;
    memset(&a, 0, sizeof a);
    a.w = m->router;
    a.x = x;
    a.dim = (uint32_t)m->dim;
    a.n_expert = (uint32_t)m->n_expert;
    // about one CTA per SM; fewer rows per CTA when they do not fit in 200 KB
    uint32_t rpc = (a.n_expert + di->sms - 1) / di->sms;
    if (rpc > ROUTER_MAX_ROWS) rpc = ROUTER_MAX_ROWS;
    // a large batch: tiles of 8 experts x 8 tokens, one CTA each (every CTA
    // stages its rows and its tokens' x once); a small one: rows spread over
    // the SMs, all tokens staged together
    uint32_t tc = n_tok < 32 ? (n_tok ? n_tok : 1u) : 8u;
    if (n_tok >= 32) rpc = 8;
    while (tc > 1 && router_smem_bytes(a.dim, rpc, tc) > 160 * 1024) tc--;
    while (rpc > 1 && router_smem_bytes(a.dim, rpc, tc) > 200 * 1024) rpc--;
    const uint32_t smem = router_smem_bytes(a.dim, rpc, tc);
    if (smem > 227 * 1024) return SG_ERR_SHAPE;
    a.rows_per_cta = rpc;
    a.row_ctas = (a.n_expert + rpc - 1) / rpc;
    a.logits = logits;
    a.qx = qx;
    const bool sh = m->shared_gate_up != nullptr;
    a.shared_sel = sh ? shsel : nullptr;
    a.shared_gate = sh ? m->shared_gate : nullptr;
    a.shared_scale = sh ? scale : nullptr;
    a.n_tok = n_tok;
    a.ldx = n_tok > 1 ? ldx : m->dim;
    a.zero_word = zero_word;
    a.tok_chunk = tc;
    // 8 threads per (row, token): one warp for a lone token, up to 256 threads for a batch
    uint32_t threads = (8 * rpc * tc + 31) / 32 * 32;
    if (threads > ROUTER_MAX_THREADS) threads = ROUTER_MAX_THREADS;
    CK(launch_pdl((const void *)moe_router_kernel, dim3(a.row_ctas + (sh ? 1 : 0), (n_tok + tc - 1) / tc), threads, smem,
                  stream, &a));
    return SG_OK;
}

sg_status pack_experts(int32_t dtype, const uint8_t *src, uint64_t n_expert, uint64_t rows, uint64_t cols,
                       uint64_t dst_rows, uint64_t off, uint8_t *dst, cudaStream_t stream) {
    const uint64_t n = n_expert * rows * (cols / 256);
    if (!n) return SG_OK;
    repack_tiled16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
        dtype == SG_Q4_K ? 0 : 1, src, n_expert * rows, (uint32_t)(cols / 256), dst, 0, rows, dst_rows, off);
    CK(cudaGetLastError());
    return SG_OK;
}

// ---- float path --------------------------------------------------------------

typedef void (*fgemv_fn)(const FGemvArgs);

template <int DT, bool M>
fgemv_fn pick_float_t(uint64_t nv) {
    return nv == 1 ? gemv_float_kernel<DT, 1, M> : nv == 2 ? gemv_float_kernel<DT, 2, M>
           : nv <= 4 ? gemv_float_kernel<DT, 4, M> : gemv_float_kernel<DT, 8, M>;
}

fgemv_fn pick_float(int32_t dt, bool multi, uint64_t nv) {
    switch (dt) {
    case SG_F32: return multi ? pick_float_t<FDT_F32, true>(nv) : pick_float_t<FDT_F32, false>(nv);
    case SG_F16: return pick_float_t<FDT_F16, false>(nv);
    case SG_Q8_0: return multi ? pick_float_t<FDT_Q8_0, true>(nv) : pick_float_t<FDT_Q8_0, false>(nv);
    case SG_Q4_K: return multi ? pick_float_t<FDT_Q4_K, true>(nv) : pick_float_t<FDT_Q4_K, false>(nv);
    default: return multi ? pick_float_t<FDT_Q6_K, true>(nv) : pick_float_t<FDT_Q6_K, false>(nv);
    }
}

// has_multi_kernel (quant_multi.rs:220-227)
bool float_has_multi(int32_t dt, uint64_t n) {
    switch (dt) {
    case SG_Q4_K: case SG_Q6_K: return n % 256 == 0;
    case SG_Q8_0: return n % 32 == 0;
    case SG_F32: return n % 8 == 0;
    default: return false;
    }
}

// matvec_rows_avx2 per vector (allow_multi false) or matmul_rows_avx2
// (quant_multi.rs:232-273: rows_multi for several vectors when the format has
// a shared-decode kernel).
sg_status float_matvec(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                       uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, bool allow_multi, cudaStream_t stream) {
    if (!d_base || !m) return SG_ERR_INVALID;
    const int32_t dt = m->dtype;
    if (dt != SG_F32 && dt != SG_F16 && dt != SG_Q8_0 && dt != SG_Q4_K && dt != SG_Q6_K) return SG_ERR_DTYPE;
    uint64_t rb;
    sg_status st = sg_row_bytes(dt, m->cols, &rb);
    if (st) return st;
    if (m->cols == 0 || m->cols > SG_MAX_COLS) return SG_ERR_SHAPE;
    if (m->layout != SG_LAYOUT_GGUF) return SG_ERR_INVALID;
    if (r0 > r1 || r1 > m->rows || m->rows > 0xFFFFFFFFull) return SG_ERR_INVALID;
    if (r1 == r0 || n_vec == 0) return SG_OK;
    if (!d_x || !d_out || (n_vec > 1 && (ldx < m->cols || ldo < m->rows))) return SG_ERR_INVALID;
    const uint8_t *w = d_base + m->offset;
    const uint64_t walign = dt == SG_Q4_K ? 16 : dt == SG_F32 ? 4 : 2;
    if (!aligned(w, walign) || !aligned(d_x, 4) || !aligned(d_out, 4)) return SG_ERR_ALIGN;
    const bool multi = allow_multi && n_vec > 1 && float_has_multi(dt, m->cols);
    uint64_t group = FGEMV_MAXV;
    if (dt == SG_Q4_K && !multi) {  // the per-vector sub-block sums live in 48 KB of shared memory
        const uint64_t per = fgemv_smem_bytes(FDT_Q4_K, false, 1, (uint32_t)m->cols);
        if (per > 48 * 1024) return SG_ERR_SHAPE;
        group = 48 * 1024 / per < group ? 48 * 1024 / per : group;
    }
    for (uint64_t g = 0; g < n_vec; g += group) {
        const uint64_t nv = n_vec - g < group ? n_vec - g : group;
        FGemvArgs a;
        memset(&a, 0, sizeof a);
        a.w = w;
        a.row_bytes = rb;
        a.n = (uint32_t)m->cols;
        a.r0 = (uint32_t)r0;
        a.r1 = (uint32_t)r1;
        a.nvec = (uint32_t)nv;
        a.x = d_x + g * ldx;
        a.ldx = ldx;
        a.out = d_out + g * ldo;
        a.ldo = ldo;
        const uint32_t grid = (uint32_t)((r1 - r0 + FGEMV_ROWS - 1) / FGEMV_ROWS);
        a.stage_x = nv == 1 && m->cols % 4 == 0 && m->cols <= FGEMV_STAGE_X_MAX && aligned(a.x, 16) ? 1u : 0u;
        const uint32_t smem = fgemv_smem_bytes(dt, multi, (uint32_t)nv, (uint32_t)m->cols, a.stage_x != 0);
        const void *fn = (const void *)pick_float(dt, multi, nv);
        if (smem) CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
        CK(launch_pdl(fn, grid, FGEMV_THREADS, smem, stream, &a));
    }
    return SG_OK;
}

}  // namespace

// ---- C ABI -----------------------------------------------------------------

extern "C" {

const char *sg_status_string(sg_status s) {
    switch (s) {
    case SG_OK: return "ok";
    case SG_ERR_INVALID: return "invalid argument";
    case SG_ERR_DTYPE: return "unsupported dtype";
    case SG_ERR_SHAPE: return "unsupported shape";
    case SG_ERR_ALIGN: return "misaligned device pointer";
    case SG_ERR_CUDA: return "CUDA error";
    case SG_ERR_NCCL: return "NCCL error";
    case SG_ERR_TIMEOUT: return "device wait timed out";
    case SG_ERR_NOMEM: return "out of memory";
    case SG_ERR_NOALLOC_LIMIT: return "request above the static scratch limit";
    default: return "unknown status";
    }
}

const char *sg_last_error_string(void) { return g_err; }

sg_status sg_row_bytes(int32_t dtype, uint64_t cols, uint64_t *out) {
    if (!out) return SG_ERR_INVALID;
    uint64_t blk, bytes;
    switch (dtype) {
    case SG_F32: blk = 1; bytes = 4; break;
    case SG_F16: blk = 1; bytes = 2; break;
    case SG_Q8_0: blk = 32; bytes = 34; break;
    case SG_Q4_K: blk = 256; bytes = 144; break;
    case SG_Q6_K: blk = 256; bytes = 210; break;
    default: return SG_ERR_DTYPE;
    }
    if (cols % blk) return SG_ERR_SHAPE;
    *out = cols / blk * bytes;
    return SG_OK;
}

int32_t sg_int_kernels_enabled(void) {
    int v = g_int_enabled.load(std::memory_order_relaxed);
    if (v == 0) {
        const char *e = getenv("SPINDLE_FLOAT_KERNELS");  // quant_q8k.rs:46
        v = (!e || !*e || strcmp(e, "0") == 0) ? 1 : 2;
        g_int_enabled.store(v, std::memory_order_relaxed);
    }
    return v == 1;
}

void sg_set_int_kernels(int32_t on) { g_int_enabled.store(on ? 1 : 2, std::memory_order_relaxed); }

int32_t sg_supports(const sg_mat *m) {
    return m && sg_int_kernels_enabled() && (m->dtype == SG_Q4_K || m->dtype == SG_Q6_K) && m->cols > 0 &&
           m->cols % 256 == 0;
}

uint64_t sg_q8k_bytes(uint64_t n) {
    const uint64_t nb = n / 256;
    return align_up(nb * 4, 16) + align_up(n, 16) + align_up(nb * 32, 16);
}

sg_status sg_q8k_view(void *d_buf, uint64_t n, sg_q8k *out) {
    if (!d_buf || !out || n % 256) return SG_ERR_INVALID;
    if (!aligned(d_buf, 16)) return SG_ERR_ALIGN;
    const uint64_t nb = n / 256;
    uint8_t *p = (uint8_t *)d_buf;
    out->d = (float *)p;
    out->qs = (int8_t *)(p + align_up(nb * 4, 16));
    out->bsums = (int16_t *)(p + align_up(nb * 4, 16) + align_up(n, 16));
    out->n = n;
    return SG_OK;
}

sg_status sg_alloc(uint64_t bytes, void **d_out) {
    if (!d_out) return SG_ERR_INVALID;
    cudaError_t e = cudaMalloc(d_out, align_up(bytes ? bytes : 1, 256));
    if (e == cudaErrorMemoryAllocation) return SG_ERR_NOMEM;
    CK(e);
    return SG_OK;
}

sg_status sg_free(void *d_ptr) {
    CK(cudaFree(d_ptr));
    return SG_OK;
}

sg_status sg_upload(const void *h_src, uint64_t bytes, void **d_out) {
    if (!h_src || !d_out) return SG_ERR_INVALID;
    sg_status st = sg_alloc(bytes, d_out);
    if (st) return st;
    CK(cudaMemcpy(*d_out, h_src, bytes, cudaMemcpyHostToDevice));
    return SG_OK;
}

sg_status sg_memcpy_h2d(void *d_dst, const void *h_src, uint64_t bytes, void *stream) {
    CK(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    return SG_OK;
}

sg_status sg_memcpy_d2h(void *h_dst, const void *d_src, uint64_t bytes, void *stream) {
    CK(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    return SG_OK;
}

sg_status sg_stream_sync(void *stream) {
    CK(cudaStreamSynchronize((cudaStream_t)stream));
    return SG_OK;
}

sg_status sg_device_status(void) {
    unsigned v = 0, zero = 0;
    CK(cudaMemcpyFromSymbol(&v, g_dev_status, sizeof v));
    if (v) CK(cudaMemcpyToSymbol(g_dev_status, &zero, sizeof zero));
    return v == DEV_OK ? SG_OK : v == DEV_BAD_LAUNCH ? SG_ERR_INVALID : SG_ERR_TIMEOUT;  // TMA or peer wait
}

sg_status sg_matmul_rows(const uint8_t *d_base, const sg_mat *m, const sg_q8k *xq, float *const *outs,
                         uint64_t n_vec, uint64_t r0, uint64_t r1, void *stream) {
    return launch_gemv(d_base, m, xq, outs, n_vec, r0, r1, nullptr, (cudaStream_t)stream);
}

sg_status sg_block_sums(const uint8_t *d_base, const sg_mat *m, const sg_q8k *xq, int32_t *d_out, uint64_t r0,
                        uint64_t r1, void *stream) {
    if (!d_out || !xq) return SG_ERR_INVALID;
    if (!aligned(d_out, 4)) return SG_ERR_ALIGN;
    // The kernel also writes the fp32 outputs; park them in the export buffer's
    // slack is not possible, so use a scratch row buffer the caller cannot see.
    float *tmp = nullptr;
    CK(cudaMallocAsync((void **)&tmp, (r1 > r0 ? r1 : 1) * sizeof(float), (cudaStream_t)stream));
    float *outs[1] = {tmp - r0};
    sg_status st = launch_gemv(d_base, m, xq, outs, 1, r0, r1, d_out, (cudaStream_t)stream);
    cudaError_t e = cudaFreeAsync(tmp, (cudaStream_t)stream);
    if (st) return st;
    CK(e);
    return SG_OK;
}

sg_status sg_q8k_quantize(const float *d_x, uint64_t n, uint64_t n_vec, uint64_t ldx, const sg_q8k *outs,
                          void *stream) {
    if (n_vec == 0) return SG_OK;
    if (!d_x || !outs || n == 0 || n % 256 || (n_vec > 1 && ldx < n)) return SG_ERR_INVALID;
    if (!aligned(d_x, 16) || (n_vec > 1 && ldx % 4)) return SG_ERR_ALIGN;
    for (uint64_t b = 0; b < n_vec; b++) {
        sg_status st = check_q8k(outs[b], n);
        if (st) return st;
        if (!aligned(outs[b].qs, 8)) return SG_ERR_ALIGN;
    }
    const uint64_t nb = n / 256;
    for (uint64_t g = 0; g < n_vec; g += Q8K_MAXV) {
        Q8kArgs a;
        memset(&a, 0, sizeof a);
        const uint32_t nv = (uint32_t)(n_vec - g < Q8K_MAXV ? n_vec - g : Q8K_MAXV);
        a.x = d_x + g * ldx;
        a.ldx = ldx;
        a.nb = (uint32_t)nb;
        a.nvec = nv;
        for (uint32_t v = 0; v < nv; v++) a.outs[v] = outs[g + v];
        const uint64_t warps = nb * nv;
        CK(launch_pdl((const void *)q8k_quantize_kernel, (uint32_t)((warps + 7) / 8), 256, 0, (cudaStream_t)stream,
                      &a));
    }
    return SG_OK;
}

sg_status sg_quantize_weights(int32_t dtype, const float *d_w, uint64_t rows, uint64_t cols, uint8_t *d_out,
                              void *stream) {
    if (!d_w || !d_out) return SG_ERR_INVALID;
    if (dtype != SG_Q4_K && dtype != SG_Q6_K) return SG_ERR_DTYPE;
    if (cols == 0 || cols % 256) return SG_ERR_SHAPE;
    const uint64_t nblocks = rows * (cols / 256);
    if (!nblocks) return SG_OK;
    const unsigned grid = (unsigned)((nblocks + 127) / 128);
    if (dtype == SG_Q4_K)
        quantize_q4k_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(d_w, nblocks, d_out);
    else
        quantize_q6k_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(d_w, nblocks, d_out);
    CK(cudaGetLastError());
    return SG_OK;
}

sg_status sg_tiled16_bytes(int32_t dtype, uint64_t rows, uint64_t cols, uint64_t *out) {
    if (!out) return SG_ERR_INVALID;
    if (dtype != SG_Q4_K && dtype != SG_Q6_K) return SG_ERR_DTYPE;
    if (cols == 0 || cols % 256) return SG_ERR_SHAPE;
    const uint64_t tiles = (rows + TILE_ROWS - 1) / TILE_ROWS;
    *out = tiles * (cols / 256) * tiled_col_bytes(dtype == SG_Q4_K ? 0 : 1);
    return SG_OK;
}

static sg_status repack(int32_t dtype, const uint8_t *src, uint64_t rows, uint64_t cols, uint8_t *dst, int inverse,
                        void *stream) {
    uint64_t bytes;
    sg_status st = sg_tiled16_bytes(dtype, rows, cols, &bytes);
    if (st) return st;
    if (!src || !dst) return SG_ERR_INVALID;
    if (!inverse) CK(cudaMemsetAsync(dst, 0, bytes, (cudaStream_t)stream));  // zero padding rows
    const uint64_t n = rows * (cols / 256);
    if (n) {
        repack_tiled16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
            dtype == SG_Q4_K ? 0 : 1, src, rows, (uint32_t)(cols / 256), dst, inverse, rows, 0, 0);
        CK(cudaGetLastError());
    }
    return SG_OK;
}

sg_status sg_repack_tiled16(int32_t dtype, const uint8_t *d_gguf, uint64_t rows, uint64_t cols, uint8_t *d_tiled,
                            void *stream) {
    return repack(dtype, d_gguf, rows, cols, d_tiled, 0, stream);
}

sg_status sg_unpack_tiled16(int32_t dtype, const uint8_t *d_tiled, uint64_t rows, uint64_t cols, uint8_t *d_gguf,
                            void *stream) {
    return repack(dtype, d_tiled, rows, cols, d_gguf, 1, stream);
}

sg_status sg_matvec(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                    uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, void *stream) {
    int dt;
    sg_status st = check_mat(d_base, m, r0, r1, &dt);
    if (st) return st;
    if (m->layout != SG_LAYOUT_TILED16) return SG_ERR_INVALID;
    if (r1 == r0 || n_vec == 0) return SG_OK;
    if (!d_x || !d_out || (n_vec > 1 && (ldx < m->cols || ldo < m->rows))) return SG_ERR_INVALID;
    if (!aligned(d_x, 16) || (n_vec > 1 && ldx % 4) || !aligned(d_out, 4)) return SG_ERR_ALIGN;
    float *outs[TGEMV_MAXV];
    for (uint64_t g = 0; g < n_vec; g += TGEMV_MAXV) {
        const uint64_t nv = n_vec - g < TGEMV_MAXV ? n_vec - g : TGEMV_MAXV;
        for (uint64_t v = 0; v < nv; v++) outs[v] = d_out + (g + v) * ldo;
        st = launch_tiled(d_base + m->offset, dt, (uint32_t)(m->cols / 256), nullptr, d_x + g * ldx, ldx, outs, nv, r0,
                          r1, (cudaStream_t)stream);
        if (st) return st;
    }
    return SG_OK;
}

// ---- a list of GEMVs in one launch --------------------------------------------

// Launch plan of gemv_list_kernel, one 16-warp CTA per SM: per matrix the S of
// tiled_plan's cost model (S = 2 with 16 warps only where no group gets a
// second tile: that case would need a 17th named barrier); one ring geometry
// for the whole list (stages of two columns of the widest type, then smaller
// until the CTA fits); each matrix's remainder tiles start at the CTA after
// the last one that took the previous matrix's.
sg_status list_plan(GlArgs *a, size_t *smem, uint32_t *grid) {
    DevInfo *di;
    sg_status st = dev_info(&di);
    if (st) return st;
    const uint32_t warps = 16, G = (uint32_t)di->sms;
    const uint32_t warp_slots = G * warps;
    const int forced = env_int("SG_LIST_S", 0);  // a fixed S where it is valid (tuning)
    uint32_t act_max = 0, cb_max = 0, chain = 0;
    for (uint32_t j = 0; j < a->n; j++) {
        GlMat &m = a->m[j];
        const uint32_t nb = m.nb, cb = tiled_col_bytes(m.dt ? 1 : 0);
        uint32_t S = 1;
        double best = 1e30;
        for (uint32_t s = 1; s <= warps && s <= nb; s *= 2) {
            const uint64_t groups = warp_slots / s;
            const uint64_t tiles = (m.ntiles + groups - 1) / groups;
            if (s > 1 && 2 * (warps / s) + 1 > 16 && tiles > 1) continue;
            if (forced > 0 && s == (uint32_t)forced) {
                S = s;
                break;
            }
            const double per_tile = (double)((nb + s - 1) / s) + 0.06 * (double)(nb - nb / s) + (s > 1 ? 0.5 : 0.0);
            const double cost = (double)tiles * per_tile;
            if (cost < best * 0.98) {
                best = cost;
                S = s;
            }
        }
        m.S = S;
        m.s_log2 = ilog2u(S);
        m.slot_blocks = (nb + S - 1) / S;
        const uint32_t step = G * (warps / S);
        m.tiles_q = m.ntiles / step;
        m.tiles_r = m.ntiles % step;
        if (act_bytes(nb) > act_max) act_max = act_bytes(nb);
        if (cb > cb_max) cb_max = cb;
        const uint32_t c = list_chain_floats(warps, S, m.slot_blocks);
        if (c > chain) chain = c;
    }
    uint32_t ns = (uint32_t)std::min(std::max(env_int("SG_LIST_STAGES", 2), 2), 4);
    uint32_t sb = (uint32_t)env_int("SG_LIST_STAGE_BYTES", 0);
    if (sb < cb_max || sb % 16) sb = 2 * cb_max;
    const size_t budget = 220 * 1024;
    for (;;) {
        *smem = list_smem_bytes(warps, ns, sb, act_max, chain);
        if (*smem <= budget) break;
        if (ns > 2)
            ns--;
        else if (sb > 2 * 2304u && 2 * 2304u >= cb_max)
            sb = 2 * 2304u;  // Q4_K two columns a stage, Q6_K one
        else if (sb > cb_max)
            sb = cb_max;
        else
            return SG_ERR_SHAPE;
    }
    const bool rot = env_int("SG_LIST_ROT", 1) != 0;
    uint32_t cur = 0;
    for (uint32_t j = 0; j < a->n; j++) {
        GlMat &m = a->m[j];
        const uint32_t bc = sb / tiled_col_bytes(m.dt ? 1 : 0);
        m.bc = bc < m.slot_blocks ? bc : m.slot_blocks;
        m.rot = rot ? (G - cur) % G : 0u;
        cur = (cur + m.tiles_r % G) % G;
    }
    a->nstages = ns;
    a->stage_bytes = sb;
    a->act_bytes = act_max;
    a->chain_floats = chain;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!di->list_attr) {
            CK(cudaFuncSetAttribute((const void *)gemv_list_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    227 * 1024));
            di->list_attr = true;
        }
    }
    *grid = G;
    return SG_OK;
}

static_assert(GL_MAX == SG_LIST_MAX, "gemv_list_kernel's list length is the header's");

// One of d_x (fp32 vectors) or d_img (Q8_K images) is given.
sg_status matvec_list_impl(const uint8_t *const *d_base, const sg_mat *mats, const float *const *d_x,
                           const uint8_t *const *d_img, float *const *d_out, uint64_t n, void *stream) {
    if (n == 0) return SG_OK;
    if (!d_base || !mats || (!d_x && !d_img) || !d_out || n > SG_LIST_MAX) return SG_ERR_INVALID;
    GlArgs a;
    memset(&a, 0, sizeof a);
    uint32_t k = 0;
    for (uint64_t j = 0; j < n; j++) {
        const sg_mat *m = &mats[j];
        int dt;
        sg_status st = check_mat(d_base[j], m, 0, m->rows, &dt);
        if (st) return st;
        if (m->layout != SG_LAYOUT_TILED16 || m->rows > 0xFFFFFFF0ull) return SG_ERR_INVALID;
        if (m->rows == 0) continue;
        const void *in = d_x ? (const void *)d_x[j] : (const void *)d_img[j];
        if (!in || !d_out[j]) return SG_ERR_INVALID;
        if (!aligned(in, 16) || !aligned(d_out[j], 4)) return SG_ERR_ALIGN;
        GlMat &g = a.m[k++];
        g.w = d_base[j] + m->offset;
        g.x = d_x ? d_x[j] : nullptr;
        g.img = d_x ? nullptr : d_img[j];
        g.out = d_out[j];
        g.dt = dt == DT_Q4K ? 0u : 1u;
        g.nb = (uint32_t)(m->cols / 256);
        g.rows = (uint32_t)m->rows;
        g.ntiles = (uint32_t)((m->rows + TILE_ROWS - 1) / TILE_ROWS);
    }
    if (k == 0) return SG_OK;
    a.n = k;
    size_t smem;
    uint32_t grid;
    sg_status st = list_plan(&a, &smem, &grid);
    if (st) return st;
    CK(launch_pdl((const void *)gemv_list_kernel, grid, 16 * 32, smem, (cudaStream_t)stream, &a));
    return SG_OK;
}

sg_status sg_matvec_list(const uint8_t *const *d_base, const sg_mat *mats, const float *const *d_x,
                         float *const *d_out, uint64_t n, void *stream) {
    return d_x ? matvec_list_impl(d_base, mats, d_x, nullptr, d_out, n, stream) : SG_ERR_INVALID;
}

sg_status sg_matvec_list_q8k(const uint8_t *const *d_base, const sg_mat *mats, const uint8_t *const *d_img,
                             float *const *d_out, uint64_t n, void *stream) {
    return d_img ? matvec_list_impl(d_base, mats, nullptr, d_img, d_out, n, stream) : SG_ERR_INVALID;
}

uint64_t sg_q8k_image_bytes(uint64_t cols) {
    if (cols == 0 || cols % 256 || cols > SG_MAX_COLS) return 0;
    return act_bytes((uint32_t)(cols / 256));
}

sg_status sg_q8k_images(const float *const *d_x, const uint64_t *cols, uint8_t *const *d_img, uint64_t n,
                        void *stream) {
    if (n == 0) return SG_OK;
    if (!d_x || !cols || !d_img || n > SG_LIST_MAX) return SG_ERR_INVALID;
    QImgArgs a;
    memset(&a, 0, sizeof a);
    a.n = (uint32_t)n;
    for (uint64_t j = 0; j < n; j++) {
        if (cols[j] == 0 || cols[j] % 256 || cols[j] > SG_MAX_COLS) return SG_ERR_SHAPE;
        if (!d_x[j] || !d_img[j]) return SG_ERR_INVALID;
        if (!aligned(d_x[j], 16) || !aligned(d_img[j], 16)) return SG_ERR_ALIGN;
        a.x[j] = d_x[j];
        a.img[j] = d_img[j];
        a.nb[j] = (uint32_t)(cols[j] / 256);
        a.blk0[j + 1] = a.blk0[j] + a.nb[j];
    }
    const uint32_t warps = a.blk0[n];
    CK(launch_pdl((const void *)q8k_images_kernel, dim3((warps + 7) / 8), 256, 0, (cudaStream_t)stream, &a));
    return SG_OK;
}

uint64_t sg_matmul_batch_scratch_bytes(const sg_mat *m, uint64_t n_vec) {
    if (!m || m->cols % 256 || n_vec == 0 || n_vec > SG_BATCH_MAX_VEC) return 0;
    return qb_image_bytes((uint32_t)n_vec, (uint32_t)(m->cols / 256));
}

sg_status sg_matmul_batch(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                          uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, void *d_scratch,
                          uint64_t scratch_bytes, void *stream) {
    int dt;
    sg_status st = check_mat(d_base, m, r0, r1, &dt);
    if (st) return st;
    if (m->layout != SG_LAYOUT_TILED16 || n_vec > SG_BATCH_MAX_VEC) return SG_ERR_INVALID;
    if (r1 == r0 || n_vec == 0) return SG_OK;
    if (!d_x || !d_out || !d_scratch || (n_vec > 1 && (ldx < m->cols || ldo < m->rows)) ||
        scratch_bytes < sg_matmul_batch_scratch_bytes(m, n_vec))
        return SG_ERR_INVALID;
    if (!aligned(d_x, 16) || ldx % 4 || !aligned(d_out, 4) || !aligned(d_scratch, 16)) return SG_ERR_ALIGN;
    const uint32_t nb = (uint32_t)(m->cols / 256);
    cudaStream_t s = (cudaStream_t)stream;
    if ((st = launch_q8k_batch(d_x, ldx, (uint32_t)n_vec, nb, (uint8_t *)d_scratch, s))) return st;
    return launch_gemm_batch(d_base + m->offset, dt, nb, r0, r1, (const uint8_t *)d_scratch, (uint32_t)n_vec, d_out,
                             n_vec > 1 ? ldo : m->rows, false, s);
}

sg_status sg_matvec_rows_float(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                               uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, void *stream) {
    return float_matvec(d_base, m, d_x, ldx, d_out, ldo, n_vec, r0, r1, false, (cudaStream_t)stream);
}

sg_status sg_matmul_rows_float(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                               uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, void *stream) {
    return float_matvec(d_base, m, d_x, ldx, d_out, ldo, n_vec, r0, r1, true, (cudaStream_t)stream);
}

uint64_t sg_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

sg_status sg_ipc_get_handle(void *d_ptr, void *handle_out) {
    if (!d_ptr || !handle_out) return SG_ERR_INVALID;
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, d_ptr));
    memcpy(handle_out, &h, sizeof h);
    return SG_OK;
}

sg_status sg_ipc_open(const void *handle, void **d_out) {
    if (!handle || !d_out) return SG_ERR_INVALID;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    CK(cudaIpcOpenMemHandle(d_out, h, cudaIpcMemLazyEnablePeerAccess));
    return SG_OK;
}

sg_status sg_ipc_close(void *d_ptr) {
    if (!d_ptr) return SG_ERR_INVALID;
    CK(cudaIpcCloseMemHandle(d_ptr));
    return SG_OK;
}

uint64_t sg_tp_comm_bytes(void) { return SG_TP_COMM_BYTES; }

sg_status sg_tp_comm_init(void *d_comm, void *stream) {
    if (!d_comm) return SG_ERR_INVALID;
    if (!aligned(d_comm, 256)) return SG_ERR_ALIGN;
    CK(cudaMemsetAsync(d_comm, 0, SG_TP_COMM_BYTES, (cudaStream_t)stream));
    return SG_OK;
}

uint64_t sg_tp_recv_bytes(uint64_t n_vec, uint64_t rows) { return 2ull * 8ull * n_vec * rows; }

sg_status sg_matvec_tp(const uint8_t *d_shard, const sg_mat *m, const float *d_x, uint64_t ldx, uint64_t n_vec,
                       uint64_t row0, uint64_t rows, float *d_out, uint64_t ldo, const sg_tp_group *grp,
                       void *stream) {
    int dt;
    sg_status st = check_mat(d_shard, m, 0, m ? m->rows : 0, &dt);
    if (st) return st;
    if (m->layout != SG_LAYOUT_TILED16 || !grp || !grp->n_ranks || grp->n_ranks > SG_TP_MAX_RANKS ||
        grp->rank >= grp->n_ranks || !grp->comm)
        return SG_ERR_INVALID;
    if (m->rows == 0 || n_vec == 0 || n_vec > TGEMV_MAXV) return SG_ERR_INVALID;  // every rank must arrive
    if (!d_x || !d_out || (n_vec > 1 && ldx < m->cols) || row0 + m->rows > rows || rows > 0xFFFFFFFFull ||
        (n_vec > 1 && ldo < rows))
        return SG_ERR_INVALID;
    if (!aligned(d_x, 16) || (n_vec > 1 && ldx % 4) || !aligned(d_out, 4) || !aligned(grp->comm, 256))
        return SG_ERR_ALIGN;
    TpSpec tp;
    memset(&tp, 0, sizeof tp);
    tp.n = grp->n_ranks;
    tp.row_off = (uint32_t)row0;
    tp.rows = (uint32_t)rows;
    for (uint32_t q = 0; q < grp->n_ranks; q++) {
        if (!grp->recv[q]) return SG_ERR_INVALID;
        if (!aligned(grp->recv[q], 8)) return SG_ERR_ALIGN;
        tp.recv[q] = (unsigned long long *)grp->recv[q];
    }
    tp.my_recv = tp.recv[grp->rank];
    tp.out = d_out;
    tp.ldo = n_vec > 1 ? ldo : rows;
    tp.ticket = (unsigned *)((uint8_t *)grp->comm + 64);
    tp.epoch = (unsigned *)((uint8_t *)grp->comm + 128);
    return launch_tiled(d_shard + m->offset, dt, (uint32_t)(m->cols / 256), nullptr, d_x, ldx, nullptr, n_vec, 0,
                        m->rows, (cudaStream_t)stream, nullptr, &tp);
}

uint64_t sg_matvec_scratch_bytes(uint64_t cols, uint64_t n_vec) {
    const uint64_t qb = sg_q8k_bytes(cols);
    return qb && n_vec > UINT64_MAX / qb ? UINT64_MAX : n_vec * qb;  // saturates instead of wrapping
}

sg_status sg_matvec_scratch(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx, float *d_out,
                            uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1, void *d_scratch,
                            uint64_t scratch_bytes, void *stream) {
    int dt;
    sg_status st = check_mat(d_base, m, r0, r1, &dt);
    if (st) return st;
    if (r1 == r0 || n_vec == 0) return SG_OK;
    if (!d_x || !d_out || !d_scratch || (n_vec > 1 && (ldx < m->cols || ldo < m->rows))) return SG_ERR_INVALID;
    const uint64_t qb = sg_q8k_bytes(m->cols);  // > 0: check_mat rejected cols == 0
    if (n_vec > scratch_bytes / qb) return SG_ERR_INVALID;  // a division, so a huge n_vec cannot wrap past it
    if (!aligned(d_scratch, 16)) return SG_ERR_ALIGN;
    for (uint64_t g = 0; g < n_vec; g += Q8K_MAXV) {
        const uint64_t nv = n_vec - g < Q8K_MAXV ? n_vec - g : Q8K_MAXV;
        sg_q8k q[Q8K_MAXV];
        float *outs[Q8K_MAXV];
        for (uint64_t v = 0; v < nv; v++) {
            if ((st = sg_q8k_view((uint8_t *)d_scratch + (g + v) * qb, m->cols, &q[v]))) return st;
            outs[v] = d_out + (g + v) * ldo;
        }
        if ((st = sg_q8k_quantize(d_x + g * ldx, m->cols, nv, ldx, q, stream))) return st;
        if ((st = launch_gemv(d_base, m, q, outs, nv, r0, r1, nullptr, (cudaStream_t)stream))) return st;
    }
    return SG_OK;
}

sg_status sg_moe_pack_gate_up(int32_t dtype, const uint8_t *d_gate_exps, const uint8_t *d_up_exps,
                              uint64_t n_expert, uint64_t n_ff, uint64_t dim, uint8_t *d_out, void *stream) {
    if (!d_gate_exps || !d_up_exps || !d_out || !n_expert || !n_ff) return SG_ERR_INVALID;
    if (!kquant(dtype)) return SG_ERR_DTYPE;
    if (!cols_ok(dim)) return SG_ERR_SHAPE;
    if (n_ff % 8) return SG_ERR_SHAPE;
    // gate row i of an expert -> packed row 16 * (i / 8) + i % 8, up row i ->
    // the same + 8 (every row of every tile is written: no padding)
    sg_status st = pack_experts(dtype, d_gate_exps, n_expert * n_ff / 8, 8, dim, 16, 0, d_out, (cudaStream_t)stream);
    if (st) return st;
    return pack_experts(dtype, d_up_exps, n_expert * n_ff / 8, 8, dim, 16, 8, d_out, (cudaStream_t)stream);
}

sg_status sg_moe_pack_down(int32_t dtype, const uint8_t *d_down_exps, uint64_t n_expert, uint64_t dim,
                           uint64_t n_ff, uint8_t *d_out, void *stream) {
    if (!d_down_exps || !d_out || !n_expert || !dim) return SG_ERR_INVALID;
    if (!kquant(dtype)) return SG_ERR_DTYPE;
    if (!cols_ok(n_ff)) return SG_ERR_SHAPE;
    const uint64_t stride = tiled_bytes(dtype, dim, n_ff);
    CK(cudaMemsetAsync(d_out, 0, stride * n_expert, (cudaStream_t)stream));
    return pack_experts(dtype, d_down_exps, n_expert, dim, n_ff, align_up(dim, TILE_ROWS), 0, d_out,
                        (cudaStream_t)stream);
}

uint64_t sg_moe_scratch_bytes(const sg_moe *m) { return check_moe(m) ? 0 : moe_scratch(m).total; }

}  // extern "C"

namespace {

// moe_forward; with `defer` set, the combine is not launched: its arguments
// are returned there for the kernel that consumes the layer's output.
sg_status moe_forward_impl(const sg_moe *m, const float *d_x, float *d_out, void *d_scratch, uint64_t scratch_bytes,
                           sg_moe_choice *d_choice, float *d_probs, void *stream, CombineArgs *defer) {
    sg_status st = check_moe(m);
    if (st) return st;
    if (!d_x || !d_out || !d_scratch) return SG_ERR_INVALID;
    if (!aligned(d_x, 16) || !aligned(d_out, 4) || !aligned(d_scratch, 256) || !aligned(d_choice, 16) ||
        !aligned(d_probs, 4))
        return SG_ERR_ALIGN;
    const MoeScratch L = moe_scratch(m);
    if (scratch_bytes < L.total) return SG_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *sc = (uint8_t *)d_scratch;
    sg_moe_choice *sel = d_choice ? d_choice : (sg_moe_choice *)(sc + L.sel);
    sg_moe_choice *shsel = (sg_moe_choice *)(sc + L.shsel);
    float *scale = (float *)(sc + L.scale), *y = (float *)(sc + L.y);
    float *logits = (float *)(sc + L.logits), *h = (float *)(sc + L.h);
    float *hsh = (float *)(sc + L.hsh), *ysh = (float *)(sc + L.ysh);
    uint8_t *qx = sc + L.qx;
    const bool sh = m->shared_gate_up != nullptr;
    const uint32_t k = (uint32_t)m->n_used, ne = (uint32_t)m->n_expert;
    // Each kernel waits for the one before it (programmatic dependent launch):
    // router -> [shared gate/up] -> gate/up (makes the choice, publishes it in
    // sel) -> down -> [shared down] -> combine.
    if ((st = launch_router(m, d_x, logits, qx, shsel, scale, s))) return st;
    if (sh && (st = launch_moe_group(m->shared_gate_up_dtype, IN_MOE_X, m->shared_gate_up, 0, 2 * m->shared_n_ff,
                                     m->dim, 1, 1, shsel, nullptr, d_x, qx, nullptr, 0, hsh, 0, s)))
        return st;
    const MoeRoute route = {logits, sel, d_probs, k, m->norm, m->moe_prune};
    if ((st = launch_moe_group(m->gate_up_dtype, IN_MOE_X, m->gate_up, m->gate_up_stride, 2 * m->n_ff, m->dim, k,
                               ne, sel, &route, d_x, qx, nullptr, 0, h, m->n_ff, s)))
        return st;
    if ((st = launch_moe_group(m->down_dtype, IN_MOE_H, m->down, m->down_stride, m->dim, m->n_ff, k, ne, sel,
                               nullptr, nullptr, nullptr, h, m->n_ff, y, m->dim, s)))
        return st;
    if (sh && (st = launch_moe_group(m->shared_down_dtype, IN_MOE_H, m->shared_down, 0, m->dim, m->shared_n_ff, 1, 1,
                                     shsel, nullptr, nullptr, nullptr, hsh, m->shared_n_ff, ysh, 0, s)))
        return st;
    CombineArgs c;
    c.sel = sel;
    c.y = y;
    c.ysh = sh ? ysh : nullptr;
    c.shared_scale = scale;
    c.out = d_out;
    c.dim = (uint32_t)m->dim;
    c.max_slots = k;
    if (defer) {
        *defer = c;
        return SG_OK;
    }
    CK(launch_pdl((const void *)moe_combine_kernel, (uint32_t)((m->dim + 255) / 256), 256, 0, s, &c));
    return SG_OK;
}

}  // namespace

extern "C" {

sg_status sg_moe_forward(const sg_moe *m, const float *d_x, float *d_out, void *d_scratch, uint64_t scratch_bytes,
                         sg_moe_choice *d_choice, float *d_probs, void *stream) {
    return moe_forward_impl(m, d_x, d_out, d_scratch, scratch_bytes, d_choice, d_probs, stream, nullptr);
}

uint64_t sg_moe_batch_scratch_bytes(const sg_moe *m, uint64_t n_tok) {
    if (check_moe(m) || n_tok == 0 || n_tok > SG_MOE_MAX_BATCH) return 0;
    return moe_batch_scratch(m, n_tok).total;
}

}  // extern "C"

namespace {

// moe_forward_batch, on one GPU (ep null) or with this rank's experts only
// (expert parallelism: slot outputs exchanged through the ranks' receive buffers).
sg_status moe_batch_impl(const sg_moe *m, const sg_moe_ep *ep, const float *d_x, uint64_t ldx, uint64_t n_tok,
                         float *d_out, uint64_t ldo, void *d_scratch, uint64_t scratch_bytes, sg_moe_choice *d_choices,
                         void *stream) {
    sg_status st = check_moe(m);
    if (st) return st;
    if (n_tok == 0) return SG_OK;
    if (n_tok > SG_MOE_MAX_BATCH || m->n_expert > 256) return SG_ERR_SHAPE;
    if (!d_x || !d_out || !d_scratch || (n_tok > 1 && (ldx < m->dim || ldo < m->dim))) return SG_ERR_INVALID;
    if (!aligned(d_x, 16) || (n_tok > 1 && ldx % 4) || !aligned(d_out, 4) || !aligned(d_scratch, 256) ||
        !aligned(d_choices, 16))
        return SG_ERR_ALIGN;
    if (ep) {
        if (!ep->n_ranks || ep->n_ranks > SG_TP_MAX_RANKS || ep->rank >= ep->n_ranks || !ep->comm ||
            ep->expert_lo > ep->expert_hi || ep->expert_hi > m->n_expert || n_tok * m->n_used > ep->recv_slots)
            return SG_ERR_INVALID;
        for (uint32_t q = 0; q < ep->n_ranks; q++)
            if (!ep->recv[q] || !aligned(ep->recv[q], 8)) return SG_ERR_INVALID;
        if (!aligned(ep->comm, 256)) return SG_ERR_ALIGN;
    }
    const MoeBatchScratch L = moe_batch_scratch(m, n_tok);
    if (scratch_bytes < L.total) return SG_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *sc = (uint8_t *)d_scratch;
    sg_moe_choice *choices = d_choices ? d_choices : (sg_moe_choice *)(sc + L.choices);
    uint32_t *slot_base = (uint32_t *)(sc + L.slot_base), *n_slots = (uint32_t *)(sc + L.n_slots);
    int32_t *slots = (int32_t *)(sc + L.slots), *slots_sh = (int32_t *)(sc + L.slots_sh);
    uint32_t *n_slots_sh = (uint32_t *)(sc + L.n_slots_sh);
    float *scale = (float *)(sc + L.scale), *logits = (float *)(sc + L.logits);
    float *h = (float *)(sc + L.h), *y = (float *)(sc + L.y), *hsh = (float *)(sc + L.hsh), *ysh = (float *)(sc + L.ysh);
    uint8_t *qx = sc + L.qx;
    const bool sh = m->shared_gate_up != nullptr;
    const uint32_t k = (uint32_t)m->n_used, ne = (uint32_t)m->n_expert, nt = (uint32_t)n_tok;
    int32_t *slots_local = (int32_t *)(sc + L.slots_local);
    uint32_t *slot_global = (uint32_t *)(sc + L.slot_global), *n_local = (uint32_t *)(sc + L.n_local);
    // router (every token) -> choices and slot table -> gate/up over all slots
    // (this rank's, with expert parallelism) -> down -> [shared gate/up, down
    // over one slot per token] -> combine
    unsigned *sel_ticket = (unsigned *)(sc + L.ticket);
    // from this many tokens on, the expert passes run over jobs (each expert's
    // weights decoded once for up to job_nv of its slots); SG_MOE_JOB_NV=0: per slot
    const int job_nv = env_int("SG_MOE_JOB_NV", 4);
    const bool use_jobs = !ep && (job_nv == 4 || job_nv == 8) && nt >= (uint32_t)env_int("SG_MOE_JOBS_MIN", 16);
    int32_t *jobs = (int32_t *)(sc + L.jobs);
    uint32_t *n_jobs = (uint32_t *)(sc + L.n_jobs);
    if ((st = launch_router(m, d_x, logits, qx, (sg_moe_choice *)(sc + L.shsel), scale, s, nt, ldx, sel_ticket)))
        return st;
    {
        static std::atomic<uint64_t> attr_done{0};
        int dev;
        CK(cudaGetDevice(&dev));
        if (!(attr_done.load() >> dev & 1)) {
            CK(cudaFuncSetAttribute((const void *)moe_select_batch_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));  // + its static words
            attr_done.fetch_or(1ull << dev);
        }
        SelectBatchArgs sa = {logits, nt, ne, k, m->norm, m->moe_prune, choices, slot_base, slots, n_slots,
                              sh ? slots_sh : nullptr, sh ? n_slots_sh : nullptr,
                              ep ? slots_local : nullptr, slot_global, n_local,
                              ep ? (uint32_t)ep->expert_lo : 0u, ep ? (uint32_t)ep->expert_hi : 0u, sel_ticket,
                              use_jobs ? jobs : nullptr, n_jobs, (uint32_t)job_nv,
                              (uint32_t)moe_max_jobs((uint64_t)nt * k, ne, 4)};
        const uint32_t sel_grid = (nt + SELECT_BATCH_THREADS / 32 - 1) / (SELECT_BATCH_THREADS / 32);
        CK(launch_pdl((const void *)moe_select_batch_kernel, sel_grid, SELECT_BATCH_THREADS, select_batch_smem(nt), s,
                      &sa));
    }
    const uint32_t ne_run = ep ? (uint32_t)(ep->expert_hi - ep->expert_lo) : ne;
    MoeSlots ms;
    memset(&ms, 0, sizeof ms);
    ms.slots = ep ? slots_local : slots;
    ms.n_slots = ep ? n_local : n_slots;
    ms.qx_tokens = qx;
    MoeSlots md = ms;
    unsigned *ep_epoch = ep ? (unsigned *)((uint8_t *)ep->comm + 128) : nullptr;
    if (ep) {
        md.npeers = ep->n_ranks;
        md.slot_global = slot_global;
        for (uint32_t q = 0; q < ep->n_ranks; q++) md.recv[q] = (unsigned long long *)ep->recv[q];
        md.ep_half = ep->recv_slots * m->dim;
        md.epoch = ep_epoch;
    }
    uint32_t units = nt * k;  // launch units: slots, or jobs
    if (use_jobs) {
        ms.jobs = md.jobs = jobs;
        ms.n_jobs = md.n_jobs = n_jobs;
        ms.job_nv = md.job_nv = (uint32_t)job_nv;
        units = (uint32_t)moe_max_jobs((uint64_t)nt * k, ne, (uint64_t)job_nv);
    }
    if (!ep || ne_run > 0) {
        if ((st = launch_moe_group(m->gate_up_dtype, IN_MOE_X, m->gate_up, m->gate_up_stride, 2 * m->n_ff, m->dim,
                                   units, ne_run ? ne_run : 1, nullptr, nullptr, nullptr, nullptr, nullptr, 0, h,
                                   m->n_ff, s, &ms)) ||
            (st = launch_moe_group(m->down_dtype, IN_MOE_H, m->down, m->down_stride, m->dim, m->n_ff, units,
                                   ne_run ? ne_run : 1, nullptr, nullptr, nullptr, nullptr, h, m->n_ff, y, m->dim, s,
                                   &md)))
            return st;
    }
    if (sh) {
        const MoeSlots mss = {slots_sh, n_slots_sh, qx};
        if ((st = launch_moe_group(m->shared_gate_up_dtype, IN_MOE_X, m->shared_gate_up, 0, 2 * m->shared_n_ff,
                                   m->dim, nt, 1, nullptr, nullptr, nullptr, nullptr, nullptr, 0, hsh,
                                   m->shared_n_ff, s, &mss)) ||
            (st = launch_moe_group(m->shared_down_dtype, IN_MOE_H, m->shared_down, 0, m->dim, m->shared_n_ff, nt, 1,
                                   nullptr, nullptr, nullptr, nullptr, hsh, m->shared_n_ff, ysh, m->dim, s, &mss)))
            return st;
    }
    CombineBatchArgs c;
    memset(&c, 0, sizeof c);
    c.choices = choices;
    c.slot_base = slot_base;
    c.y = y;
    c.ysh = sh ? ysh : nullptr;
    c.shared_scale = scale;
    c.out = d_out;
    c.ldo = n_tok > 1 ? ldo : m->dim;
    c.dim = (uint32_t)m->dim;
    c.n_used = k;
    if (ep) {
        c.recv = (const unsigned long long *)ep->recv[ep->rank];
        c.half = ep->recv_slots * m->dim;
        c.ticket = (unsigned *)((uint8_t *)ep->comm + 64);
        c.epoch = ep_epoch;
    }
    CK(launch_pdl((const void *)moe_combine_batch_kernel, dim3((uint32_t)((m->dim + 255) / 256), nt), 256, 0, s, &c));
    return SG_OK;
}

}  // namespace

extern "C" {

sg_status sg_moe_forward_batch(const sg_moe *m, const float *d_x, uint64_t ldx, uint64_t n_tok, float *d_out,
                               uint64_t ldo, void *d_scratch, uint64_t scratch_bytes, sg_moe_choice *d_choices,
                               void *stream) {
    return moe_batch_impl(m, nullptr, d_x, ldx, n_tok, d_out, ldo, d_scratch, scratch_bytes, d_choices, stream);
}

uint64_t sg_moe_ep_recv_bytes(const sg_moe *m, uint64_t n_tok_max) {
    if (check_moe(m) || n_tok_max == 0 || n_tok_max > SG_MOE_MAX_BATCH) return 0;
    return 2ull * 8ull * n_tok_max * m->n_used * m->dim;
}

sg_status sg_moe_forward_batch_ep(const sg_moe *m, const sg_moe_ep *ep, const float *d_x, uint64_t ldx,
                                  uint64_t n_tok, float *d_out, uint64_t ldo, void *d_scratch, uint64_t scratch_bytes,
                                  sg_moe_choice *d_choices, void *stream) {
    if (!ep) return SG_ERR_INVALID;
    return moe_batch_impl(m, ep, d_x, ldx, n_tok, d_out, ldo, d_scratch, scratch_bytes, d_choices, stream);
}

}  // extern "C"

// ---- decoder step (forward_slice) ------------------------------------------

namespace {

bool kq(int32_t dt) { return dt == SG_Q4_K || dt == SG_Q6_K; }

sg_status check_model(const sg_model *m) {
    if (!m || !m->embed || !m->lm_head || !m->output_norm || !m->layers) return SG_ERR_INVALID;
    if (!m->n_heads || !m->n_kv_heads || m->n_heads % m->n_kv_heads || !m->n_layers || !m->vocab || !m->max_seq)
        return SG_ERR_INVALID;
    if (m->dim % 256 || m->dim == 0 || m->dim > 8192 || m->head_dim % 64 || m->head_dim == 0 || m->head_dim > 256 ||
        (m->n_heads * m->head_dim) % 256 || attn_smem_bytes(m->head_dim, m->max_seq, 2) > 227 * 1024)
        return SG_ERR_SHAPE;
    if (m->embed_dtype != SG_F32 && m->embed_dtype != SG_F16 && !kq(m->embed_dtype)) return SG_ERR_DTYPE;
    if (!kq(m->lm_head_dtype)) return SG_ERR_DTYPE;
    for (uint32_t l = 0; l < m->n_layers; l++) {
        const sg_layer &y = m->layers[l];
        if (!y.attn_norm || !y.ffn_norm || !y.wq || !y.wk || !y.wv || !y.wo) return SG_ERR_INVALID;
        if (!kq(y.wq_dtype) || !kq(y.wk_dtype) || !kq(y.wv_dtype) || !kq(y.wo_dtype)) return SG_ERR_DTYPE;
        if (y.is_moe) {
            sg_status st = check_moe(&y.moe);
            if (st) return st;
            if (y.moe.dim != m->dim) return SG_ERR_SHAPE;
        } else {
            if (!y.ffn_gate_up || !y.ffn_down) return SG_ERR_INVALID;
            if (!kq(y.ffn_gate_up_dtype) || !kq(y.ffn_down_dtype)) return SG_ERR_DTYPE;
            if (!cols_ok(y.n_ff)) return SG_ERR_SHAPE;
        }
    }
    return SG_OK;
}

struct ModelScratch {
    uint64_t x, xn, qx, q, k, v, att, proj, logits, h, freqs, sel1, amax, moe, moe_bytes, total;
};

ModelScratch model_scratch(const sg_model *m) {
    ModelScratch L;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const uint64_t q_dim = (uint64_t)m->n_heads * m->head_dim, kv_dim = (uint64_t)m->n_kv_heads * m->head_dim;
    uint64_t n_ff = 0, moe = 0;
    for (uint32_t l = 0; l < m->n_layers; l++) {
        const sg_layer &y = m->layers[l];
        if (y.is_moe) {
            const uint64_t b = moe_scratch(&y.moe).total;
            moe = b > moe ? b : moe;
        } else if (y.n_ff > n_ff) {
            n_ff = y.n_ff;
        }
    }
    L.x = take(m->dim * 4);
    L.xn = take(m->dim * 4);
    L.qx = take(act_bytes(m->dim / 256));
    L.q = take((q_dim + kv_dim) * 4);  // q then k: one GEMV fills both when wk follows wq
    L.k = L.q + q_dim * 4;
    L.v = take(kv_dim * 4);
    L.att = take(q_dim * 4);
    L.proj = take(m->dim * 4);
    L.logits = take((uint64_t)m->vocab * 4);
    L.h = take(n_ff * 4);
    L.freqs = take(m->head_dim / 2 * 4);
    L.sel1 = take(sizeof(sg_moe_choice));
    L.amax = take(ARGMAX_CTAS * 8 + 8);  // the argmax's partial maxima, then its ticket count
    L.moe = take(moe);
    L.moe_bytes = moe;
    L.total = off;
    return L;
}

sg_status launch_norm(float *x, const float *add, float rs, const float *w, float eps, uint32_t n, float *xn,
                      uint8_t *qx, cudaStream_t s, uint32_t ntok = 1) {
    NormArgs a = {x, add, rs, w, eps, n, xn, qx};
    CK(launch_pdl((const void *)rmsnorm_kernel, ntok, NORM_THREADS, n * 4, s, &a));
    return SG_OK;
}

// Scratch of sg_forward_batch for up to n_max tokens per call.
struct ModelBatchScratch {
    uint64_t x, xn, qx, qkv, att, proj, logits, h, freqs, amax, slots, n_slots, moe, moe_bytes, qb, total;
};

ModelBatchScratch model_batch_scratch(const sg_model *m, uint64_t n) {
    ModelBatchScratch L;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const uint64_t q_dim = (uint64_t)m->n_heads * m->head_dim, kv_dim = (uint64_t)m->n_kv_heads * m->head_dim;
    uint64_t n_ff = 0, moe = 0;
    for (uint32_t l = 0; l < m->n_layers; l++) {
        const sg_layer &y = m->layers[l];
        if (y.is_moe) {
            const uint64_t b = sg_moe_batch_scratch_bytes(&y.moe, n);
            moe = b > moe ? b : moe;
        } else if (y.n_ff > n_ff) {
            n_ff = y.n_ff;
        }
    }
    L.x = take(n * m->dim * 4);
    L.xn = take(n * m->dim * 4);
    L.qx = take(n * act_bytes(m->dim / 256));
    L.qkv = take(n * (q_dim + 2 * kv_dim) * 4);
    L.att = take(n * q_dim * 4);
    L.proj = take(n * m->dim * 4);
    L.logits = take(n * (uint64_t)m->vocab * 4);
    L.h = take(n * n_ff * 4);
    L.freqs = take(m->head_dim / 2 * 4);
    L.amax = take(n * (ARGMAX_CTAS * 8 + 4));  // partial maxima, then the ticket counts
    L.slots = take(n * 8);                       // dense FFN: slot t = (0, t)
    L.n_slots = take(4);
    L.moe = take(moe);
    L.moe_bytes = moe;
    // QB image of the widest input of a batch GEMM (dim, q_dim or a dense n_ff)
    uint64_t widest = m->dim > q_dim ? m->dim : q_dim;
    if (n_ff > widest) widest = n_ff;
    L.qb = take(qb_image_bytes((uint32_t)n, (uint32_t)(widest / 256)));
    L.total = off;
    return L;
}

// Rows of a TILED16 matrix for n fp32 vectors (cols apart), outs[t] per vector.
sg_status gemv_rows(const uint8_t *w, int32_t dtype, uint64_t rows, uint64_t cols, const float *x,
                    std::vector<float *> &outs, uint32_t n, cudaStream_t s) {
    return launch_tiled(w, dtype == SG_Q4_K ? DT_Q4K : DT_Q6K, (uint32_t)(cols / 256), nullptr, x, cols, outs.data(), n,
                        0, rows, s);
}

sg_status gemv_image(const uint8_t *w, int32_t dtype, uint64_t rows, uint64_t cols, const uint8_t *image, float *out,
                     cudaStream_t s) {
    float *outs[1] = {out};
    return launch_tiled(w, dtype == SG_Q4_K ? DT_Q4K : DT_Q6K, (uint32_t)(cols / 256), nullptr, nullptr, 0, outs, 1,
                        0, rows, s, image);
}

}  // namespace

extern "C" {

uint64_t sg_model_scratch_bytes(const sg_model *m) { return check_model(m) ? 0 : model_scratch(m).total; }

uint64_t sg_model_ep_scratch_bytes(const sg_model *m) {
    if (check_model(m)) return 0;
    uint64_t moe = 0;
    for (uint32_t l = 0; l < m->n_layers; l++)
        if (m->layers[l].is_moe) {
            const uint64_t b = moe_batch_scratch(&m->layers[l].moe, 1).total;
            moe = b > moe ? b : moe;
        }
    return align_up(model_scratch(m).total, 256) + moe;
}

uint64_t sg_model_kv_bytes(const sg_model *m) {
    if (check_model(m)) return 0;
    return 2ull * m->n_layers * m->max_seq * m->n_kv_heads * m->head_dim * 2;
}

sg_status sg_model_prepare(const sg_model *m, void *d_scratch, uint64_t scratch_bytes, void *stream) {
    sg_status st = check_model(m);
    if (st) return st;
    const ModelScratch L = model_scratch(m);
    if (!d_scratch || scratch_bytes < L.total) return SG_ERR_INVALID;
    if (!aligned(d_scratch, 256)) return SG_ERR_ALIGN;
    // Rope::new (smollm_chat.rs:1403-1406): 1 / theta^(2i / head_dim), the host's powf
    std::vector<float> f(m->head_dim / 2);
    for (uint32_t i = 0; i < m->head_dim / 2; i++) {
        const float e = (2.0f * (float)i) / (float)m->head_dim;
        f[i] = 1.0f / powf(m->rope_theta, e);
    }
    sg_moe_choice one;
    memset(&one, 0, sizeof one);
    one.n = 1;
    one.weight[0] = 1.0f;
    uint8_t *sc = (uint8_t *)d_scratch;
    CK(cudaMemcpyAsync(sc + L.freqs, f.data(), f.size() * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    CK(cudaMemcpyAsync(sc + L.sel1, &one, sizeof one, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    CK(cudaMemsetAsync(sc + L.amax + ARGMAX_CTAS * 8, 0, 8, (cudaStream_t)stream));
    CK(cudaStreamSynchronize((cudaStream_t)stream));  // the host sources go out of scope
    return SG_OK;
}

uint64_t sg_model_batch_scratch_bytes(const sg_model *m, uint64_t n_max) {
    if (check_model(m) || n_max == 0 || n_max > SG_MOE_MAX_BATCH) return 0;
    for (uint32_t l = 0; l < m->n_layers; l++)
        if (m->layers[l].is_moe && m->layers[l].moe.n_expert > 256) return 0;
    return model_batch_scratch(m, n_max).total;
}

sg_status sg_model_batch_prepare(const sg_model *m, uint64_t n_max, void *d_scratch, uint64_t scratch_bytes,
                                 void *stream) {
    sg_status st = check_model(m);
    if (st) return st;
    if (n_max == 0 || n_max > SG_MOE_MAX_BATCH) return SG_ERR_SHAPE;
    const ModelBatchScratch L = model_batch_scratch(m, n_max);
    if (!d_scratch || scratch_bytes < L.total) return SG_ERR_INVALID;
    if (!aligned(d_scratch, 256)) return SG_ERR_ALIGN;
    std::vector<float> f(m->head_dim / 2);
    for (uint32_t i = 0; i < m->head_dim / 2; i++) {
        const float e = (2.0f * (float)i) / (float)m->head_dim;
        f[i] = 1.0f / powf(m->rope_theta, e);
    }
    std::vector<int32_t> slots(2 * n_max);
    for (uint64_t t = 0; t < n_max; t++) {
        slots[2 * t] = 0;
        slots[2 * t + 1] = (int32_t)t;
    }
    uint8_t *sc = (uint8_t *)d_scratch;
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemcpyAsync(sc + L.freqs, f.data(), f.size() * 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(sc + L.slots, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemsetAsync(sc + L.amax + n_max * ARGMAX_CTAS * 8, 0, n_max * 4, s));
    CK(cudaStreamSynchronize(s));  // the host sources go out of scope
    return SG_OK;
}

sg_status sg_forward_batch(const sg_model *m, const int32_t *d_tokens, uint64_t n, const int32_t *d_pos, void *d_kv,
                           void *d_scratch, uint64_t scratch_bytes, uint64_t n_max, float *d_logits, uint64_t ldl,
                           int64_t *d_greedy, void *stream) {
    return sg_forward_batch_range(m, 0, m ? m->n_layers : 0, d_tokens, nullptr, n, d_pos, d_kv, d_scratch,
                                  scratch_bytes, n_max, nullptr, d_logits, ldl, d_greedy, stream);
}

sg_status sg_forward_batch_range(const sg_model *m, uint32_t l0, uint32_t l1, const int32_t *d_tokens,
                                 const float *d_hidden_in, uint64_t n, const int32_t *d_pos, void *d_kv,
                                 void *d_scratch, uint64_t scratch_bytes, uint64_t n_max, float *d_hidden_out,
                                 float *d_logits, uint64_t ldl, int64_t *d_greedy, void *stream) {
    sg_status st = check_model(m);
    if (st) return st;
    if (l0 >= l1 || l1 > m->n_layers) return SG_ERR_INVALID;
    if (n == 0) return SG_OK;
    // l0 > 0 without d_hidden_in: continue from the state a call ending at l0
    // left in this scratch (l1 < n_layers without d_hidden_out leaves it)
    const bool resume = l0 > 0 && !d_hidden_in;
    if ((l0 == 0 && !d_tokens) || !d_pos || !d_kv || !d_scratch || n > n_max || n_max > SG_MOE_MAX_BATCH)
        return SG_ERR_INVALID;
    if (!aligned(d_hidden_in, 16) || !aligned(d_hidden_out, 16)) return SG_ERR_ALIGN;
    if (d_logits && n > 1 && ldl < m->vocab) return SG_ERR_INVALID;
    if (!aligned(d_scratch, 256) || !aligned(d_kv, 16) || !aligned(d_tokens, 4) || !aligned(d_pos, 4) ||
        !aligned(d_logits, 4) || !aligned(d_greedy, 8))
        return SG_ERR_ALIGN;
    const ModelBatchScratch L = model_batch_scratch(m, n_max);
    if (scratch_bytes < L.total) return SG_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *sc = (uint8_t *)d_scratch;
    const uint32_t dim = m->dim, hd = m->head_dim, q_dim = m->n_heads * hd, kv_dim = m->n_kv_heads * hd;
    const uint32_t nt = (uint32_t)n, qkv_stride = q_dim + 2 * kv_dim;
    float *x = (float *)(sc + L.x), *xn = (float *)(sc + L.xn), *qkv = (float *)(sc + L.qkv);
    float *att = (float *)(sc + L.att), *proj = (float *)(sc + L.proj), *h = (float *)(sc + L.h);
    float *logits = d_logits ? d_logits : (float *)(sc + L.logits);
    const uint64_t lstride = d_logits && n > 1 ? ldl : m->vocab;
    uint8_t *qx = sc + L.qx;
    const float *freqs = (const float *)(sc + L.freqs);
    const uint64_t cache = (uint64_t)m->max_seq * kv_dim;
    uint16_t *kc = (uint16_t *)d_kv, *vc = kc + (uint64_t)m->n_layers * cache;
    const float scale = m->attn_scale != 0.0f ? m->attn_scale : 1.0f / sqrtf((float)hd);
    {
        static std::atomic<uint64_t> attr_done{0};
        int dev;
        CK(cudaGetDevice(&dev));
        if (!(attr_done.load() >> dev & 1)) {
            for (const void *fn : {(const void *)attention_kernel<64, 64>, (const void *)attention_kernel<128, 64>,
                                   (const void *)attention_kernel<256, 64>, (const void *)attention_kernel<64, 128>,
                                   (const void *)attention_kernel<128, 128>, (const void *)attention_kernel<256, 128>,
                                   (const void *)attention_batch_kernel<64>, (const void *)attention_batch_kernel<128>,
                                   (const void *)attention_batch_kernel<256>})
                CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
            attr_done.fetch_or(1ull << dev);
        }
    }
    std::vector<float *> oq(nt), ok_(nt), ov(nt), oo(nt), ol(nt);
    for (uint32_t t = 0; t < nt; t++) {
        oq[t] = qkv + (uint64_t)t * qkv_stride;
        ok_[t] = oq[t] + q_dim;
        ov[t] = ok_[t] + kv_dim;
        oo[t] = proj + (uint64_t)t * dim;
        ol[t] = logits + (uint64_t)t * lstride;
    }
    uint32_t *n_slots = (uint32_t *)(sc + L.n_slots);
    uint8_t *qb = sc + L.qb;
    const bool batch_gemm = nt >= (uint32_t)env_int("SG_BATCH_GEMM_MIN", 9);
    // attention chunks: 64 positions (half the shared memory, more CTAs per
    // SM) when the launch has several waves of CTAs; 128 otherwise
    DevInfo *attn_di;
    if ((st = dev_info(&attn_di))) return st;
    const uint32_t attn_chunk = (uint64_t)nt * m->n_heads >= 8ull * (uint64_t)attn_di->sms ? 64u : 128u;
    // from SG_ATTN_BATCH_MIN tokens on (default 16), the attention with shared K/V rows
    const uint32_t grp = m->n_kv_heads ? m->n_heads / m->n_kv_heads : 0u;
    const bool attn_shared = nt >= (uint32_t)env_int("SG_ATTN_BATCH_MIN", 16) && grp && ATTN_PAIRS % grp == 0 &&
                             m->n_heads % m->n_kv_heads == 0 && (hd == 64 || hd == 128 || hd == 256);
    const void *attn_batch_fn = hd == 64    ? (const void *)attention_batch_kernel<64>
                                : hd == 128 ? (const void *)attention_batch_kernel<128>
                                            : (const void *)attention_batch_kernel<256>;
    const void *attn_fn = attn_chunk == 64
                              ? (hd == 64    ? (const void *)attention_kernel<64, 64>
                                 : hd == 128 ? (const void *)attention_kernel<128, 64>
                                             : (const void *)attention_kernel<256, 64>)
                              : (hd == 64    ? (const void *)attention_kernel<64, 128>
                                 : hd == 128 ? (const void *)attention_kernel<128, 128>
                                             : (const void *)attention_kernel<256, 128>);
    if (l0 == 0) {
        EmbedArgs ea = {m->embed, m->embed_dtype, dim, m->vocab, m->embedding_scale, nullptr, x, d_tokens, n_slots};
        CK(launch_pdl((const void *)embed_kernel, dim3((dim + 255) / 256, nt), 256, 0, s, &ea));
    } else if (!resume) {
        // a later pipeline stage: the raw residual of the stage before
        CK(cudaMemcpyAsync(x, d_hidden_in, (uint64_t)nt * dim * 4, cudaMemcpyDeviceToDevice, s));
        CK(cudaMemsetAsync(n_slots, 0, 4, s));
        CK(cudaMemsetAsync(n_slots, (int)nt, 1, s));  // nt <= 128: the low byte
    }
    for (uint32_t l = l0; l < l1; l++) {
        const sg_layer &y = m->layers[l];
        if ((st = launch_norm(x, l > l0 || resume ? proj : nullptr, m->residual_scale, y.attn_norm, m->rms_eps, dim, xn,
                              nullptr, s, nt)))
            return st;
        uint64_t wq_bytes = 0;
        const bool qk_one = y.wk_dtype == y.wq_dtype && !sg_tiled16_bytes(y.wq_dtype, q_dim, dim, &wq_bytes) &&
                            y.wk == y.wq + wq_bytes;
        // many tokens: one quantize per input and one batch GEMM per matrix;
        // few: the GEMV with up to 8 vectors per launch
        auto gemv = [&](const uint8_t *w, int32_t dt, uint32_t rows, uint32_t cols, const float *xin,
                        std::vector<float *> &outs) {
            if (batch_gemm)
                return launch_gemm_batch(w, dt == SG_Q4_K ? DT_Q4K : DT_Q6K, cols / 256, 0, rows, qb, nt, outs[0],
                                         outs.size() > 1 ? (uint64_t)(outs[1] - outs[0]) : rows, false, s);
            return launch_tiled(w, dt == SG_Q4_K ? DT_Q4K : DT_Q6K, cols / 256, nullptr, xin, cols, outs.data(), nt, 0,
                                rows, s);
        };
        if (batch_gemm && (st = launch_q8k_batch(xn, dim, nt, dim / 256, qb, s))) return st;
        if (qk_one) {
            if ((st = gemv(y.wq, y.wq_dtype, q_dim + kv_dim, dim, xn, oq))) return st;
        } else if ((st = gemv(y.wq, y.wq_dtype, q_dim, dim, xn, oq)) || (st = gemv(y.wk, y.wk_dtype, kv_dim, dim, xn, ok_))) {
            return st;
        }
        if ((st = gemv(y.wv, y.wv_dtype, kv_dim, dim, xn, ov))) return st;
        RopeBatchArgs ra = {qkv, qkv + q_dim, qkv + q_dim + kv_dim, qkv_stride, y.q_norm, y.k_norm, m->rms_eps, freqs,
                            hd, m->n_heads, m->n_kv_heads, m->rope_neox, d_pos, kc + l * cache, vc + l * cache,
                            m->max_seq};
        CK(launch_pdl((const void *)rope_kv_batch_kernel, dim3(m->n_heads + m->n_kv_heads, nt), 32, 0, s, &ra));
        AttnArgs aa = {qkv, nullptr, nullptr, nullptr, nullptr, m->rms_eps, freqs, hd, m->n_heads, m->n_kv_heads,
                       m->max_seq, m->rope_neox, scale, d_pos, kc + l * cache, vc + l * cache, att, 1, qkv_stride,
                       2, attn_chunk, nt};  // two buffers: many CTAs, two or more of them per SM
        if (attn_shared) {
            // one CTA per (KV head, block of tokens): each K/V row staged once for the block's pairs
            const uint32_t tb = ATTN_PAIRS / (m->n_heads / m->n_kv_heads);
            CK(launch_pdl(attn_batch_fn, dim3(m->n_kv_heads, (nt + tb - 1) / tb), attn_batch_threads(hd),
                          attn_batch_smem(hd), s, &aa));
        } else {
            CK(launch_pdl(attn_fn, dim3(m->n_heads, nt), attn_threads(hd),
                          attn_smem_bytes(hd, m->max_seq, 2, attn_chunk), s, &aa));
        }
        if (batch_gemm && (st = launch_q8k_batch(att, q_dim, nt, q_dim / 256, qb, s))) return st;
        if ((st = gemv(y.wo, y.wo_dtype, dim, q_dim, att, oo))) return st;
        if ((st = launch_norm(x, proj, m->residual_scale, y.ffn_norm, m->rms_eps, dim, xn, qx, s, nt))) return st;
        if (y.is_moe) {
            if ((st = sg_moe_forward_batch(&y.moe, xn, dim, n, proj, dim, sc + L.moe, L.moe_bytes, nullptr, stream)))
                return st;
        } else if (batch_gemm) {
            // dense FFN: gate/up with SiLU*up in the epilogue, then down
            if ((st = launch_q8k_batch(xn, dim, nt, dim / 256, qb, s)) ||
                (st = launch_gemm_batch(y.ffn_gate_up, y.ffn_gate_up_dtype == SG_Q4_K ? DT_Q4K : DT_Q6K, dim / 256, 0,
                                        2 * (uint64_t)y.n_ff, qb, nt, h, y.n_ff, true, s)) ||
                (st = launch_q8k_batch(h, y.n_ff, nt, y.n_ff / 256, qb, s)) ||
                (st = launch_gemm_batch(y.ffn_down, y.ffn_down_dtype == SG_Q4_K ? DT_Q4K : DT_Q6K, y.n_ff / 256, 0,
                                        dim, qb, nt, proj, dim, false, s)))
                return st;
        } else {
            const MoeSlots ms = {(const int32_t *)(sc + L.slots), n_slots, qx};
            if ((st = launch_moe_group(y.ffn_gate_up_dtype, IN_MOE_X, y.ffn_gate_up, 0, 2 * y.n_ff, dim, nt, 1,
                                       nullptr, nullptr, nullptr, nullptr, nullptr, 0, h, y.n_ff, s, &ms)) ||
                (st = launch_moe_group(y.ffn_down_dtype, IN_MOE_H, y.ffn_down, 0, dim, y.n_ff, nt, 1, nullptr, nullptr,
                                       nullptr, nullptr, h, y.n_ff, proj, dim, s, &ms)))
                return st;
        }
    }
    if (l1 < m->n_layers && !d_hidden_out) return SG_OK;  // the state stays in the scratch (x, proj)
    if (l1 < m->n_layers) {
        // a middle stage returns the raw residual (smollm_chat.rs:3546-3551)
        const uint64_t tot = (uint64_t)nt * dim;
        void *args[] = {&x, &proj, (void *)&m->residual_scale, &d_hidden_out, (void *)&tot};
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((uint32_t)((tot + 255) / 256));
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        CK(cudaLaunchKernelExC(&cfg, (const void *)residual_kernel, args));
        return SG_OK;
    }
    // the last stage: output-normed hidden states (what forward_batch_slice
    // returns), then the head only when logits or greedy tokens are asked for
    // (a prompt fed by feed(), smollm_chat.rs:3042-3106, keeps hidden states only)
    float *xo = d_hidden_out ? d_hidden_out : xn;
    if ((st = launch_norm(x, proj, m->residual_scale, m->output_norm, m->rms_eps, dim, xo, nullptr, s, nt))) return st;
    if (!d_logits && !d_greedy) return SG_OK;
    if (batch_gemm) {
        if ((st = launch_q8k_batch(xo, dim, nt, dim / 256, qb, s)) ||
            (st = launch_gemm_batch(m->lm_head, m->lm_head_dtype == SG_Q4_K ? DT_Q4K : DT_Q6K, dim / 256, 0, m->vocab,
                                    qb, nt, logits, lstride, false, s)))
            return st;
    } else if ((st = gemv_rows(m->lm_head, m->lm_head_dtype, m->vocab, dim, xo, ol, nt, s))) {
        return st;
    }
    ArgmaxArgs ga = {logits, m->vocab, nullptr, d_greedy, (unsigned long long *)(sc + L.amax),
                     (unsigned *)(sc + L.amax + n_max * ARGMAX_CTAS * 8), 1, lstride};
    if (d_greedy) CK(launch_pdl((const void *)argmax_kernel, dim3(ARGMAX_CTAS, nt), ARGMAX_THREADS, 0, s, &ga));
    return SG_OK;
}

sg_status sg_kv_shift(const sg_model *m, void *d_kv, const void *d_scratch, uint32_t l0, uint32_t l1,
                      uint32_t n_keep, uint32_t n_discard, uint32_t cur_pos, void *stream) {
    sg_status st = check_model(m);
    if (st) return st;
    if (!d_kv || !d_scratch || l0 > l1 || l1 > m->n_layers || cur_pos > m->max_seq) return SG_ERR_INVALID;
    if (!aligned(d_kv, 16) || !aligned(d_scratch, 256)) return SG_ERR_ALIGN;
    // shift_kv (smollm_chat.rs:2942-2972): nothing to drop past the pinned positions
    const uint32_t n_ctx = cur_pos > n_keep ? cur_pos - n_keep : 0u;
    if (n_discard > n_ctx) n_discard = n_ctx;
    if (n_discard == 0 || l0 == l1) return SG_OK;
    const uint32_t n_move = n_ctx - n_discard, kv_dim = m->n_kv_heads * m->head_dim;
    const ModelScratch L = model_scratch(m);
    uint16_t *kc = (uint16_t *)d_kv, *vc = kc + (uint64_t)m->n_layers * m->max_seq * kv_dim;
    for (uint32_t i0 = 0; i0 < n_move; i0 += n_discard) {  // waves of n_discard rows (see kv_shift_kernel)
        const uint32_t i1 = n_move - i0 < n_discard ? n_move : i0 + n_discard;
        KvShiftArgs a = {kc, vc, (const float *)((const uint8_t *)d_scratch + L.freqs), l0, l1, m->max_seq, kv_dim,
                         m->head_dim, (uint32_t)(m->rope_neox != 0), n_keep, n_discard, i0, i1};
        const uint64_t work = (uint64_t)(l1 - l0) * (i1 - i0) * (kv_dim / 2);
        const uint64_t blocks = (work + 255) / 256;
        kv_shift_kernel<<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, (cudaStream_t)stream>>>(a);
        CK(cudaGetLastError());
    }
    return SG_OK;
}

uint64_t sg_pipe_recv_bytes(uint64_t n_max) { return 2ull * 8ull * n_max; }

sg_status sg_pipe_send(const float *d_src, uint64_t n, uint64_t n_max, void *d_peer_recv, void *d_comm, void *stream) {
    if (!d_src || !d_peer_recv || !d_comm || n > n_max) return SG_ERR_INVALID;
    if (!aligned(d_peer_recv, 8) || !aligned(d_comm, 256)) return SG_ERR_ALIGN;
    if (n == 0) return SG_OK;
    PipeArgs a = {d_src, nullptr, (unsigned long long *)d_peer_recv, n, n_max, (unsigned *)((uint8_t *)d_comm + 128),
                  (unsigned *)((uint8_t *)d_comm + 64), (unsigned *)((uint8_t *)d_comm + 192)};
    const uint32_t grid = (uint32_t)((n + 255) / 256 < 148 ? (n + 255) / 256 : 148);
    CK(launch_pdl((const void *)pipe_send_kernel, grid, 256, 0, (cudaStream_t)stream, &a));
    return SG_OK;
}

sg_status sg_pipe_recv(float *d_dst, uint64_t n, uint64_t n_max, void *d_recv, void *d_comm, void *d_peer_comm,
                       void *stream) {
    if (!d_dst || !d_recv || !d_comm || !d_peer_comm || n > n_max) return SG_ERR_INVALID;
    if (!aligned(d_recv, 8) || !aligned(d_comm, 256) || !aligned(d_peer_comm, 256)) return SG_ERR_ALIGN;
    if (n == 0) return SG_OK;
    PipeArgs a = {nullptr, d_dst, (unsigned long long *)d_recv, n, n_max, (unsigned *)((uint8_t *)d_comm + 128),
                  (unsigned *)((uint8_t *)d_comm + 64), (unsigned *)((uint8_t *)d_peer_comm + 192)};
    const uint32_t grid = (uint32_t)((n + 255) / 256 < 148 ? (n + 255) / 256 : 148);
    CK(launch_pdl((const void *)pipe_recv_kernel, grid, 256, 0, (cudaStream_t)stream, &a));
    return SG_OK;
}

// sg_forward and sg_forward_ep: eps (host, [n_layers]) runs every MoE layer
// on this rank's experts, its slot outputs exchanged with the other ranks
// (moe_forward_batch for one token, expert-parallel), in scratch past the
// one-GPU step's.
static sg_status forward_one(const sg_model *m, const sg_moe_ep *eps, int32_t *d_state, void *d_kv, void *d_scratch,
                             uint64_t scratch_bytes, float *d_hidden, float *d_logits, int64_t *d_token,
                             void *stream) {
    sg_status st = check_model(m);
    if (st) return st;
    if (!d_state || !d_kv || !d_scratch) return SG_ERR_INVALID;
    if (!aligned(d_scratch, 256) || !aligned(d_kv, 16) || !aligned(d_state, 4) || !aligned(d_hidden, 4) ||
        !aligned(d_logits, 4) || !aligned(d_token, 8))
        return SG_ERR_ALIGN;
    const ModelScratch L = model_scratch(m);
    if (scratch_bytes < (eps ? sg_model_ep_scratch_bytes(m) : L.total)) return SG_ERR_INVALID;
    const uint64_t ep_off = align_up(L.total, 256), ep_bytes = scratch_bytes - (eps ? ep_off : 0);
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *sc = (uint8_t *)d_scratch;
    float *x = (float *)(sc + L.x), *xn = (float *)(sc + L.xn), *q = (float *)(sc + L.q), *k = (float *)(sc + L.k);
    float *v = (float *)(sc + L.v), *att = (float *)(sc + L.att), *proj = (float *)(sc + L.proj);
    float *logits = d_logits ? d_logits : (float *)(sc + L.logits), *h = (float *)(sc + L.h);
    const float *freqs = (const float *)(sc + L.freqs);
    const sg_moe_choice *sel1 = (const sg_moe_choice *)(sc + L.sel1);
    uint8_t *qx = sc + L.qx;
    const uint32_t dim = m->dim, hd = m->head_dim, q_dim = m->n_heads * hd, kv_dim = m->n_kv_heads * hd;
    const uint64_t cache = (uint64_t)m->max_seq * kv_dim;  // f16 elements per layer
    uint16_t *kc = (uint16_t *)d_kv, *vc = kc + (uint64_t)m->n_layers * cache;
    const float scale = m->attn_scale != 0.0f ? m->attn_scale : 1.0f / sqrtf((float)hd);
    static std::atomic<uint64_t> attr_done{0};
    int dev;
    CK(cudaGetDevice(&dev));
    if (!(attr_done.load() >> dev & 1)) {
        for (const void *fn : {(const void *)attention_kernel<64, ATTN_CHUNK>, (const void *)attention_kernel<128, ATTN_CHUNK>,
                               (const void *)attention_kernel<256, ATTN_CHUNK>})
            CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr_done.fetch_or(1ull << dev);
    }
    const void *attn_fn = hd == 64    ? (const void *)attention_kernel<64, ATTN_CHUNK>
                          : hd == 128 ? (const void *)attention_kernel<128, ATTN_CHUNK>
                                      : (const void *)attention_kernel<256, ATTN_CHUNK>;

    EmbedArgs ea = {m->embed, m->embed_dtype, dim, m->vocab, m->embedding_scale, d_state, x};
    CK(launch_pdl((const void *)embed_kernel, (dim + 255) / 256, 256, 0, s, &ea));
    // an MoE layer's combine runs inside the norm that consumes its output
    CombineArgs comb{};
    bool deferred = false;
    auto norm_after_ffn = [&](const float *w) {
        NormArgs a = {x, deferred ? nullptr : proj, m->residual_scale, w, m->rms_eps, dim, xn, qx};
        if (deferred) {
            a.csel = comb.sel;
            a.cy = comb.y;
            a.cysh = comb.ysh;
            a.cscale = comb.shared_scale;
            a.cmax_slots = comb.max_slots;
        }
        deferred = false;
        return launch_pdl((const void *)rmsnorm_kernel, 1, NORM_THREADS, dim * 4, s, &a);
    };
    for (uint32_t l = 0; l < m->n_layers; l++) {
        const sg_layer &y = m->layers[l];
        // attention: norm (+ the previous layer's FFN residual), Q/K/V, head norms, RoPE, KV, attention
        if (l) {
            CK(norm_after_ffn(y.attn_norm));
        } else if ((st = launch_norm(x, nullptr, m->residual_scale, y.attn_norm, m->rms_eps, dim, xn, qx, s))) {
            return st;
        }
        // wk stored right after wq in the same format: one launch computes q and k (k follows q in scratch)
        uint64_t wq_bytes = 0;
        const bool qk_one = y.wk_dtype == y.wq_dtype && !sg_tiled16_bytes(y.wq_dtype, q_dim, dim, &wq_bytes) &&
                            y.wk == y.wq + wq_bytes;
        if (qk_one) {
            if ((st = gemv_image(y.wq, y.wq_dtype, q_dim + kv_dim, dim, qx, q, s))) return st;
        } else if ((st = gemv_image(y.wq, y.wq_dtype, q_dim, dim, qx, q, s)) ||
                   (st = gemv_image(y.wk, y.wk_dtype, kv_dim, dim, qx, k, s))) {
            return st;
        }
        if ((st = gemv_image(y.wv, y.wv_dtype, kv_dim, dim, qx, v, s))) return st;
        // one CTA per head: as many chunk buffers as fit, so that every K and V
        // chunk of a short context is in flight before the dependency wait
        const uint32_t nbuf = attn_smem_bytes(hd, m->max_seq, ATTN_MAX_BUF) <= 227 * 1024 ? ATTN_MAX_BUF : 2u;
        AttnArgs aa = {q, k, v, y.q_norm, y.k_norm, m->rms_eps, freqs, hd, m->n_heads, m->n_kv_heads, m->max_seq,
                       m->rope_neox, scale, d_state, kc + l * cache, vc + l * cache, att, 0, 0, nbuf, ATTN_CHUNK};
        CK(launch_pdl(attn_fn, m->n_heads, attn_threads(hd), attn_smem_bytes(hd, m->max_seq, nbuf), s, &aa));
        {
            float *outs[1] = {proj};
            if ((st = launch_tiled(y.wo, y.wo_dtype == SG_Q4_K ? DT_Q4K : DT_Q6K, q_dim / 256, nullptr, att, q_dim,
                                   outs, 1, 0, dim, s)))
                return st;
        }
        // feed-forward: norm (+ attention residual), then the dense SwiGLU or the MoE layer
        if ((st = launch_norm(x, proj, m->residual_scale, y.ffn_norm, m->rms_eps, dim, xn, qx, s))) return st;
        if (y.is_moe && eps) {
            // this rank's experts; every rank's combine writes the whole layer output
            if ((st = moe_batch_impl(&y.moe, &eps[l], xn, dim, 1, proj, dim, sc + ep_off, ep_bytes, nullptr, stream)))
                return st;
        } else if (y.is_moe) {
            if ((st = moe_forward_impl(&y.moe, xn, proj, sc + L.moe, L.moe_bytes, nullptr, nullptr, stream, &comb)))
                return st;
            deferred = true;
        } else {
            if ((st = launch_moe_group(y.ffn_gate_up_dtype, IN_MOE_X, y.ffn_gate_up, 0, 2 * y.n_ff, dim, 1, 1, sel1,
                                       nullptr, xn, qx, nullptr, 0, h, 0, s)) ||
                (st = launch_moe_group(y.ffn_down_dtype, IN_MOE_H, y.ffn_down, 0, dim, y.n_ff, 1, 1, sel1, nullptr,
                                       nullptr, nullptr, h, 0, proj, 0, s)))
                return st;
        }
    }
    // output norm (+ the last FFN residual), LM head, greedy token
    CK(norm_after_ffn(m->output_norm));
    if (d_hidden) CK(cudaMemcpyAsync(d_hidden, xn, dim * 4, cudaMemcpyDeviceToDevice, s));
    if ((st = gemv_image(m->lm_head, m->lm_head_dtype, m->vocab, dim, qx, logits, s))) return st;
    ArgmaxArgs ga = {logits, m->vocab, d_state, d_token, (unsigned long long *)(sc + L.amax),
                     (unsigned *)(sc + L.amax + ARGMAX_CTAS * 8)};
    CK(launch_pdl((const void *)argmax_kernel, ARGMAX_CTAS, ARGMAX_THREADS, 0, s, &ga));
    return SG_OK;
}

sg_status sg_forward(const sg_model *m, int32_t *d_state, void *d_kv, void *d_scratch, uint64_t scratch_bytes,
                     float *d_hidden, float *d_logits, int64_t *d_token, void *stream) {
    return forward_one(m, nullptr, d_state, d_kv, d_scratch, scratch_bytes, d_hidden, d_logits, d_token, stream);
}

sg_status sg_forward_ep(const sg_model *m, const sg_moe_ep *eps, int32_t *d_state, void *d_kv, void *d_scratch,
                        uint64_t scratch_bytes, float *d_hidden, float *d_logits, int64_t *d_token, void *stream) {
    if (!eps) return SG_ERR_INVALID;
    return forward_one(m, eps, d_state, d_kv, d_scratch, scratch_bytes, d_hidden, d_logits, d_token, stream);
}

}  // extern "C"
