// gemv_list.cu — a list of independent GEMVs in one launch (see gemv_list.cuh).
#include "gemv_list.cuh"
#include "q8k_block.cuh"
#include "tiled_block.cuh"

namespace sg {
using namespace tiled;

namespace {

// One warp's part of matrix m: its tile group, its slot's super-blocks, its tiles.
struct GlGeo {
    uint32_t S, group, slot, G;
    uint32_t b_lo, nblk, bc, nchunk;
    uint32_t first, step, my_tiles;
};

__device__ __forceinline__ GlGeo gl_geo(const GlMat &m, uint32_t warp, uint32_t nwarps) {
    GlGeo o;
    const uint32_t SL = m.s_log2;
    o.S = m.S;
    o.group = warp >> SL;
    o.slot = warp & (m.S - 1u);
    o.G = nwarps >> SL;
    o.b_lo = (m.nb * o.slot) >> SL;
    o.nblk = ((m.nb * (o.slot + 1u)) >> SL) - o.b_lo;
    o.bc = m.bc;
    o.nchunk = (o.nblk + o.bc - 1u) / o.bc;
    // groups numbered CTA-minor, so that consecutive tiles land on different
    // SMs; then rotated, so that the remainder tiles move on from matrix to matrix
    const uint32_t total = gridDim.x * o.G;
    uint32_t gid = o.group * gridDim.x + blockIdx.x + m.rot;
    if (gid >= total) gid -= total;
    o.first = gid;
    o.step = total;
    o.my_tiles = m.tiles_q + (gid < m.tiles_r ? 1u : 0u);
    return o;
}

// The ring's producer (lane 0 of each warp): the warp's items in the order
// the warp consumes them, matrix after matrix; item = chunk c (bc super-blocks
// of the warp's slot) of the warp's tile t of matrix j.
struct GlProducer {
    uint32_t j, t, c, st, issued;
    GlGeo geo;

    __device__ __forceinline__ void seek(const GlArgs &a, uint32_t warp, uint32_t nwarps) {
        while (j < a.n && t >= geo.my_tiles) {
            if (++j < a.n) {
                geo = gl_geo(a.m[j], warp, nwarps);
                t = c = 0;
            }
        }
    }
    __device__ __forceinline__ void init(const GlArgs &a, uint32_t warp, uint32_t nwarps) {
        j = t = c = st = issued = 0;
        geo = gl_geo(a.m[0], warp, nwarps);
        seek(a, warp, nwarps);
    }
    __device__ __forceinline__ bool issue(const GlArgs &a, uint8_t *ring, uint64_t *bars, uint32_t warp,
                                          uint32_t nwarps) {
        if (j >= a.n) return false;
        const GlMat &m = a.m[j];
        const uint32_t cb = tiled_col_bytes(m.dt ? 1 : 0);
        const uint32_t tt = geo.first + t * geo.step;
        const uint32_t nblocks = min(geo.bc, geo.nblk - c * geo.bc);
        const uint8_t *src = m.w + ((uint64_t)tt * m.nb + geo.b_lo + c * geo.bc) * cb;
        mbar_arrive_expect_tx(&bars[st], nblocks * cb);
        bulk_g2s(ring + st * a.stage_bytes, src, nblocks * cb, &bars[st]);
        issued++;
        if (++st == a.nstages) st = 0;
        if (++c == geo.nchunk) {
            c = 0;
            ++t;
            seek(a, warp, nwarps);
        }
        return true;
    }
};

// The state a warp carries from tile to tile.
struct GlWarp {
    uint32_t k, kst, kph;  // items consumed; the ring stage and mbarrier phase of the next
    bool failed;           // a copy timed out: no more waits or copies
};

// The warp's tiles of matrix m (gemv_tiled_kernel's tile loop for one vector).
template <int DT>
__device__ __forceinline__ void gl_tiles(const GlArgs &a, const GlMat &m, const GlGeo &geo, const uint8_t *av,
                                         uint8_t *ring, uint64_t *bars, float *chain, uint32_t warp, uint32_t nwarps,
                                         uint32_t lane, GlWarp &ws, GlProducer &prod) {
    constexpr uint32_t CB = tiled_col_bytes(DT);
    const uint32_t g = lane >> 4, r = lane & 15u;
    const uint32_t S = geo.S, slot = geo.slot;
    const uint32_t worker_floats = m.slot_blocks * CHAIN_FLOATS;
    float *gscratch = chain + geo.group * (S - 1u) * worker_floats;
    float *mine = gscratch + (slot ? (slot - 1u) * worker_floats : 0u);
    // named barriers 1..2G (the host keeps 2G + 1 <= 16 wherever a group has a
    // second tile, the only case that uses bar_free)
    const uint32_t bar_full = 1u + geo.group, bar_free = 1u + geo.G + geo.group, nbar = 32u * S;
    for (uint32_t ti = 0; ti < geo.my_tiles; ti++) {
        const uint32_t tt = geo.first + ti * geo.step;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, corr = 0.0f;
        if (slot > 0 && ti > 0) named_sync(bar_free, nbar);  // slot 0 has read the previous tile
        for (uint32_t c = 0; c < geo.nchunk; c++, ws.k++) {
            const uint32_t st = ws.kst, ph = ws.kph;
            if (++ws.kst == a.nstages) {
                ws.kst = 0;
                ws.kph ^= 1u;
            }
            if (!ws.failed) {
                const bool ok = mbar_wait_bounded(&bars[st], ph, WAIT_LIMIT_NS);
                if (__any_sync(0xffffffffu, !ok)) {
                    // record it, let the copies in flight land (bounded), issue
                    // no more; keep the barrier protocol so the CTA still exits
                    if (lane == 0) {
                        atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                        for (uint32_t p = ws.k; p < prod.issued; p++)
                            mbar_wait_bounded(&bars[p % a.nstages], (p / a.nstages) & 1u, WAIT_LIMIT_NS);
                    }
                    ws.failed = true;
                    __syncwarp();
                }
            }
            const uint32_t ncols = min(geo.bc, geo.nblk - c * geo.bc);
            for (uint32_t qq = 0; qq < ncols; qq++) {
                const uint32_t q = c * geo.bc + qq, i = geo.b_lo + q;
                const uint8_t *col = ring + st * a.stage_bytes + qq * CB;
                int s[4];
                float cd, ct;
                if constexpr (DT == 0) {
                    Q4KWeights wt;
                    q4k_weights(col, g, r, wt);
                    q4k_dot(wt, g, i, m.nb, av, s, cd, ct);
                } else {
                    Q6KWeights wt;
                    q6k_weights(col, g, r, wt);
                    q6k_dot(wt, g, i, m.nb, av, s, cd, ct);
                }
                if (slot == 0) {
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[j] = __fmaf_rn(cd, lane_f<DT>(s[j]), acc[j]);
                    corr = __fadd_rn(corr, ct);
                } else {
                    float *e = mine + q * CHAIN_FLOATS;
                    *reinterpret_cast<float4 *>(e + 64 * g + 4 * r) =
                        make_float4(lane_f<DT>(s[0]), lane_f<DT>(s[1]), lane_f<DT>(s[2]), lane_f<DT>(s[3]));
                    if (g == 0) {
                        e[128 + r] = cd;
                        e[144 + r] = ct;
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && !ws.failed) {
                fence_proxy_async();  // this stage's reads before the copy that refills it
                prod.issue(a, ring, bars, warp, nwarps);
            }
        }
        if (S > 1) {
            if (slot > 0) {
                named_arrive(bar_full, nbar);
            } else {
                named_sync(bar_full, nbar);
                // continue the chain over the other slots' blocks, in block order
                for (uint32_t wsl = 1; wsl < S; wsl++) {
                    const float *src = gscratch + (wsl - 1u) * worker_floats;
                    const uint32_t n_ws = ((m.nb * (wsl + 1u)) >> m.s_log2) - ((m.nb * wsl) >> m.s_log2);
                    for (uint32_t q = 0; q < n_ws; q++) {
                        const float *e = src + q * CHAIN_FLOATS;
                        const float4 f = *reinterpret_cast<const float4 *>(e + 64 * g + 4 * r);
                        const float cd = e[128 + r];
                        acc[0] = __fmaf_rn(cd, f.x, acc[0]);
                        acc[1] = __fmaf_rn(cd, f.y, acc[1]);
                        acc[2] = __fmaf_rn(cd, f.z, acc[2]);
                        acc[3] = __fmaf_rn(cd, f.w, acc[3]);
                        corr = __fadd_rn(corr, e[144 + r]);
                    }
                }
                if (ti + 1 < geo.my_tiles) named_arrive(bar_free, nbar);
            }
        }
        if (slot == 0) {
            // 8-lane tree ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), then minus the correction
            float x[4];
#pragma unroll
            for (int j = 0; j < 4; j++) x[j] = __fadd_rn(acc[j], __shfl_down_sync(0xffffffffu, acc[j], 16));
            const float yv = __fsub_rn(__fadd_rn(__fadd_rn(x[0], x[2]), __fadd_rn(x[1], x[3])), corr);
            const uint32_t row = tt * TILE_ROWS + r;
            if (g == 0 && row < m.rows) m.out[row] = yv;
        }
    }
}

// One warp quantizes 256-blocks b0, b0 + stride, ... of x (nb blocks) into the
// image at av, two blocks' loads in flight at once.
__device__ __forceinline__ void gl_quantize(const float *x, uint32_t nb, uint8_t *av, uint32_t b0, uint32_t stride,
                                            uint32_t lane) {
    constexpr int QB = 2;
    for (uint32_t bb = b0; bb < nb; bb += stride * QB) {
        float xv[QB][8];
#pragma unroll
        for (int q = 0; q < QB; q++) {
            const uint32_t b = bb + q * stride;
            if (b < nb) {
                const float4 *xp = reinterpret_cast<const float4 *>(x + 256u * b) + 2 * lane;
                const float4 p0 = xp[0], p1 = xp[1];
                xv[q][0] = p0.x, xv[q][1] = p0.y, xv[q][2] = p0.z, xv[q][3] = p0.w;
                xv[q][4] = p1.x, xv[q][5] = p1.y, xv[q][6] = p1.z, xv[q][7] = p1.w;
            }
        }
#pragma unroll
        for (int q = 0; q < QB; q++) {
            const uint32_t b = bb + q * stride;
            if (b < nb)
                q8k_block_regs(xv[q], reinterpret_cast<int8_t *>(av + 256u * b),
                               reinterpret_cast<int16_t *>(av + 256u * nb + 32u * b),
                               reinterpret_cast<float *>(av + 288u * nb + 4u * b), lane);
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(TGEMV_WARPS * 32, 1) gemv_list_kernel(const __grid_constant__ GlArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nwarps = blockDim.x >> 5;
    // A launch whose arguments or shared memory do not fit this layout records
    // an error and does nothing (uniform exit, before any barrier).
    bool bad = a.n == 0 || a.n > GL_MAX || (blockDim.x & 31u) || nwarps == 0 || nwarps > TGEMV_WARPS ||
               a.nstages == 0 || a.nstages * nwarps * 8u > GL_IMG_BAR_OFF || (a.act_bytes & 15u) ||
               (a.stage_bytes & 15u) ||
               list_smem_bytes(nwarps, a.nstages, a.stage_bytes, a.act_bytes, a.chain_floats) > dynamic_smem_size();
    for (uint32_t j = 0; j < a.n && !bad; j++) {
        const GlMat &m = a.m[j];
        const uint32_t cb = tiled_col_bytes(m.dt ? 1 : 0);
        bad = m.dt > 1u || m.nb == 0 || act_bytes(m.nb) > a.act_bytes || m.S == 0 || m.s_log2 > 4u ||
              m.S != (1u << m.s_log2) || m.S > nwarps || (nwarps & (m.S - 1u)) || m.S > m.nb || m.bc == 0 ||
              m.bc * cb > a.stage_bytes || m.slot_blocks * m.S < m.nb ||
              list_chain_floats(nwarps, m.S, m.slot_blocks) > a.chain_floats ||
              (m.S > 1u && 2u * (nwarps >> m.s_log2) + 1u > 16u &&
               (m.tiles_q > 1u || (m.tiles_q == 1u && m.tiles_r > 0u))) ||
              m.rot >= gridDim.x * (nwarps >> m.s_log2) || (uint64_t)m.ntiles * TILE_ROWS < m.rows || !m.w ||
              !m.out || ((uintptr_t)m.w & 15u) ||
              (m.img ? ((uintptr_t)m.img & 15u) != 0 : (!m.x || ((uintptr_t)m.x & 15u)));
    }
    if (bad) {
        if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    // the next kernel may launch as soon as SMs free up
    grid_launch_dependents();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * a.nstages;
    uint64_t *ibar = reinterpret_cast<uint64_t *>(smem + GL_IMG_BAR_OFF);  // activation buffer b's image copy
    uint8_t *act = smem + TGEMV_BAR_BYTES;
    uint8_t *rings = act + 2u * a.act_bytes;
    uint8_t *ring = rings + warp * a.nstages * a.stage_bytes;
    float *chain = reinterpret_cast<float *>(rings + nwarps * a.nstages * a.stage_bytes);

    // Weights depend on nothing: every warp's ring fills before the wait.
    GlProducer prod;
    prod.init(a, warp, nwarps);
    if (threadIdx.x == 0) {
        mbar_init(&ibar[0], 1);
        mbar_init(&ibar[1], 1);
    }
    if (lane == 0) {
        for (uint32_t st = 0; st < a.nstages; st++) mbar_init(&bars[st], 1);
        fence_mbar_init();
        for (uint32_t st = 0; st < a.nstages; st++)
            if (!prod.issue(a, ring, bars, warp, nwarps)) break;
    }
    // x_0's lines into L2 (a hint; the grid's CTAs share the lines out)
    if (!a.m[0].img) {
        const uint32_t lines = a.m[0].nb * 8u;
        for (uint32_t l = blockIdx.x * blockDim.x + threadIdx.x; l < lines; l += gridDim.x * blockDim.x)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a.m[0].x + 32u * l));
    }
    grid_dependency_wait();  // the inputs may come from the grid before
    // x_j goes into buffer j & 1; an image by one bulk copy (x_0's now,
    // x_{j+1}'s once matrix j starts, when every warp is done with the buffer)
    auto copy_image = [&](uint32_t j) {
        const uint32_t bytes = act_bytes(a.m[j].nb);
        mbar_arrive_expect_tx(&ibar[j & 1u], bytes);
        bulk_g2s(act + (j & 1u) * a.act_bytes, a.m[j].img, bytes, &ibar[j & 1u]);
    };
    if (threadIdx.x == 0 && a.m[0].img) copy_image(0);
    __syncthreads();  // the buffers' mbarriers are initialized before anyone waits on them

    GlWarp ws = {0u, 0u, 0u, false};
    uint32_t iph = 0;  // bit b: buffer b's image-copy phase
    for (uint32_t j = 0; j < a.n; j++) {
        const GlMat &m = a.m[j];
        uint8_t *av = act + (j & 1u) * a.act_bytes;
        if (m.img) {
            const uint32_t b = j & 1u, ph = (iph >> b) & 1u;
            if (!mbar_wait_bounded(&ibar[b], ph, WAIT_LIMIT_NS)) {
                // record it and let the copy land (bounded) before anything touches the buffer
                if (lane == 0) atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                mbar_wait_bounded(&ibar[b], ph, WAIT_LIMIT_NS);
            }
            iph ^= 1u << b;
        } else {
            gl_quantize(m.x, m.nb, av, warp, nwarps, lane);
        }
        // x_j staged; every warp is done with matrix j - 1 (its chain scratch,
        // and the activation buffer matrix j + 1 will use: its generic reads
        // and writes ordered before the image copy into it)
        fence_proxy_async();
        __syncthreads();
        if (j + 1 < a.n && a.m[j + 1].img) {
            if (threadIdx.x == 0) copy_image(j + 1);
        } else if (j + 1 < a.n) {
            const uint32_t lines = a.m[j + 1].nb * 8u;
            for (uint32_t l = blockIdx.x * blockDim.x + threadIdx.x; l < lines; l += gridDim.x * blockDim.x)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(a.m[j + 1].x + 32u * l));
        }
        const GlGeo geo = gl_geo(m, warp, nwarps);
        if (m.dt == 0)
            gl_tiles<0>(a, m, geo, av, ring, bars, chain, warp, nwarps, lane, ws, prod);
        else
            gl_tiles<1>(a, m, geo, av, ring, bars, chain, warp, nwarps, lane, ws, prod);
    }
}

__global__ void __launch_bounds__(256) q8k_images_kernel(const __grid_constant__ QImgArgs a) {
    // the next kernel (the GEMV reading the images) may launch now and stream
    // its weights; then wait for the kernel that wrote x
    grid_launch_dependents();
    grid_dependency_wait();
    const uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
    if (a.n == 0 || a.n > GL_MAX || w >= a.blk0[a.n]) return;
    uint32_t j = 0;
    while (j + 1 < a.n && w >= a.blk0[j + 1]) j++;
    const uint32_t nb = a.nb[j], b = w - a.blk0[j];
    uint8_t *img = a.img[j];
    q8k_block(a.x[j] + 256u * b, reinterpret_cast<int8_t *>(img + 256u * b),
              reinterpret_cast<int16_t *>(img + 256u * nb + 32u * b), reinterpret_cast<float *>(img + 288u * nb + 4u * b),
              lane);
    // the padding after d[nb] is zero, so that an image is the same bytes every time
    const uint32_t pad = (act_bytes(nb) - 292u * nb) / 4u;
    if (b == nb - 1u && lane < pad) reinterpret_cast<uint32_t *>(img + 292u * nb)[lane] = 0u;
}

}  // namespace sg
