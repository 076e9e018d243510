// gemv_tiled.cu — kernels over the TILED16 layout (see gemv_tiled.cuh).
#include "gemv_tiled.cuh"

namespace sg {

namespace {

constexpr uint32_t M4 = 0x0F0F0F0Fu, B45 = 0x30303030u;

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint4 ldg128(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ uint32_t w4(const uint4 &v, int m) { return m == 0 ? v.x : m == 1 ? v.y : m == 2 ? v.z : v.w; }
__device__ __forceinline__ int sbyte(uint32_t w, int b) { return (int)(int8_t)(w >> (8 * b)); }
__device__ __forceinline__ int ubyte(uint32_t w, int b) { return (int)((w >> (8 * b)) & 0xFFu); }
__device__ __forceinline__ int lo16(uint32_t w) { return (int)(int16_t)(w & 0xFFFFu); }
__device__ __forceinline__ int hi16(uint32_t w) { return (int)(int16_t)(w >> 16); }
__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace

template <int DT, int NV>
__global__ void __launch_bounds__(TGEMV_WARPS * 32) gemv_tiled_kernel(const __grid_constant__ TGemvArgs a) {
    constexpr uint32_t CB = tiled_col_bytes(DT);
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * a.nstages;
    uint8_t *ring = smem + 256 + warp * a.nstages * a.stage_bytes;
    const uint32_t g = lane >> 4, r = lane & 15u;
    const uint32_t nchunks = (a.nb + a.bc - 1) / a.bc;
    const uint32_t gw = blockIdx.x * TGEMV_WARPS + warp, W = gridDim.x * TGEMV_WARPS;
    const uint32_t my_tiles = gw < a.ntiles ? (a.ntiles - gw + W - 1) / W : 0u;
    const uint32_t nitems = my_tiles * nchunks;
    const uint64_t tile_bytes = (uint64_t)a.nb * CB;

    auto issue = [&](uint32_t k) {
        const uint32_t tt = a.t0 + gw + (k / nchunks) * W, c = k % nchunks;
        const uint32_t ncols = min(a.bc, a.nb - c * a.bc);
        uint64_t *bar = &bars[k % a.nstages];
        mbar_arrive_expect_tx(bar, ncols * CB);
        bulk_g2s(ring + (k % a.nstages) * a.stage_bytes, a.w + tt * tile_bytes + (uint64_t)c * a.bc * CB,
                 ncols * CB, bar);
    };
    if (lane == 0) {
        for (uint32_t s = 0; s < a.nstages; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (lane == 0)
        for (uint32_t k = 0; k < nitems && k < a.nstages; k++) issue(k);

    uint32_t k = 0;
    for (uint32_t ti = 0; ti < my_tiles; ti++) {
        const uint32_t tt = a.t0 + gw + ti * W;
        float acc[NV][4], corr[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) {
            corr[v] = 0.0f;
#pragma unroll
            for (int m = 0; m < 4; m++) acc[v][m] = 0.0f;
        }
        for (uint32_t c = 0; c < nchunks; c++, k++) {
            const uint32_t st = k % a.nstages;
            const bool ok = mbar_wait_bounded(&bars[st], (k / a.nstages) & 1u, WAIT_LIMIT_NS);
            if (__any_sync(0xffffffffu, !ok)) {
                if (lane == 0) {
                    atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                    for (uint32_t q = k; q < nitems && q < k + a.nstages; q++)
                        mbar_wait_bounded(&bars[q % a.nstages], (q / a.nstages) & 1u, WAIT_LIMIT_NS);
                }
                __syncwarp();
                return;
            }
            const uint8_t *stage = ring + st * a.stage_bytes;
            const uint32_t ncols = min(a.bc, a.nb - c * a.bc);
            for (uint32_t q = 0; q < ncols; q++) {
                const uint32_t i = c * a.bc + q;
                const uint8_t *col = stage + q * CB;
                if constexpr (DT == 0) {
                    // ---- Q4_K: head = d, dmin, 12 scale bytes; qs row = 128 B
                    const uint4 hd = lds128(col + 2048 + 16 * r);
                    const float d = h2f_lo(hd.x), dmin = h2f_hi(hd.x);
                    const uint32_t sclo = hd.y & 0x3F3F3F3Fu, schi = (hd.w & M4) | ((hd.y >> 2) & B45);
                    const uint32_t mnw = g ? (((hd.w >> 4) & M4) | ((hd.z >> 2) & B45)) : (hd.z & 0x3F3F3F3Fu);
                    const int sc[8] = {ubyte(sclo, 0), ubyte(sclo, 1), ubyte(sclo, 2), ubyte(sclo, 3),
                                       ubyte(schi, 0), ubyte(schi, 1), ubyte(schi, 2), ubyte(schi, 3)};
                    uint32_t lo[4][4], hi[4][4];
#pragma unroll
                    for (int cc = 0; cc < 4; cc++) {
                        const uint4 qv = lds128(col + 128 * r + 32 * cc + 16 * g);
#pragma unroll
                        for (int m = 0; m < 4; m++) {
                            lo[cc][m] = w4(qv, m) & M4;
                            hi[cc][m] = (w4(qv, m) >> 4) & M4;
                        }
                    }
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        if (v >= (int)a.nvec) break;
                        const int8_t *y = a.xs[v] + 256u * i + 16u * g;
                        uint4 Y[8];
#pragma unroll
                        for (int kk = 0; kk < 8; kk++) Y[kk] = ldg128(y + 32 * kk);
                        const uint4 B = ldg128(a.xb[v] + 16u * i + 8u * g);
                        const float xd = __ldg(a.xd[v] + i);
                        int s[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int cc = 0; cc < 4; cc++)
#pragma unroll
                            for (int m = 0; m < 4; m++) {
                                s[m] += sc[2 * cc] * __dp4a((int)lo[cc][m], (int)w4(Y[2 * cc], m), 0);
                                s[m] += sc[2 * cc + 1] * __dp4a((int)hi[cc][m], (int)w4(Y[2 * cc + 1], m), 0);
                            }
                        const float cd = __fmul_rn(d, xd);
#pragma unroll
                        for (int m = 0; m < 4; m++) acc[v][m] = __fmaf_rn(cd, __int2float_rn(s[m]), acc[v][m]);
                        int sp = 0;
#pragma unroll
                        for (int m = 0; m < 4; m++) sp += ubyte(mnw, m) * (lo16(w4(B, m)) + hi16(w4(B, m)));
                        sp += __shfl_xor_sync(0xffffffffu, sp, 16);
                        corr[v] = __fadd_rn(corr[v], __fmul_rn(__fmul_rn(dmin, xd), __int2float_rn(sp)));
                    }
                } else {
                    // ---- Q6_K: qlqh row = ql[128] qh[64]; scales row = 16 B; d = 2 B
                    const uint8_t *qrow = col + 192 * r;
                    uint32_t w[8][4];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint4 L0 = lds128(qrow + 64 * h + 16 * g);
                        const uint4 L1 = lds128(qrow + 64 * h + 32 + 16 * g);
                        const uint4 H = lds128(qrow + 128 + 32 * h + 16 * g);
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
                    // chunk 4h+k of lanes 4g..4g+3 uses scale 8h + 2k + g
                    int scv[8];
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            scv[4 * h + kk] = sbyte(w4(SC, 2 * h + (kk >> 1)), 2 * (kk & 1) + (int)g);
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        if (v >= (int)a.nvec) break;
                        const int8_t *y = a.xs[v] + 256u * i + 16u * g;
                        uint4 Y[8];
#pragma unroll
                        for (int kk = 0; kk < 8; kk++) Y[kk] = ldg128(y + 32 * kk);
                        const uint4 Ba = ldg128(a.xb[v] + 16u * i), Bb = ldg128(a.xb[v] + 16u * i + 8u);
                        const float xd = __ldg(a.xd[v] + i);
                        int s[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int kk = 0; kk < 8; kk++)
#pragma unroll
                            for (int m = 0; m < 4; m++) s[m] += scv[kk] * __dp4a((int)w[kk][m], (int)w4(Y[kk], m), 0);
                        const float cd = __fmul_rn(d, xd);
#pragma unroll
                        for (int m = 0; m < 4; m++) acc[v][m] = __fmaf_rn(cd, __int2float_rn(s[m]), acc[v][m]);
                        // groups of parity g: sum_j sc[2j+g] * bsums[2j+g]
                        int sp = 0;
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const uint32_t bw = j < 4 ? w4(Ba, j) : w4(Bb, j - 4);
                            sp += scv[j] * (g ? hi16(bw) : lo16(bw));
                        }
                        sp += __shfl_xor_sync(0xffffffffu, sp, 16);
                        corr[v] = __fadd_rn(corr[v], __fmul_rn(cd, __int2float_rn(32 * sp)));
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && k + a.nstages < nitems) {
                fence_proxy_async();
                issue(k + a.nstages);
            }
        }
        // 8-lane tree ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), then minus the correction.
        const uint32_t row = tt * TILE_ROWS + r;
#pragma unroll
        for (int v = 0; v < NV; v++) {
            float x[4];
#pragma unroll
            for (int m = 0; m < 4; m++) x[m] = __fadd_rn(acc[v][m], __shfl_down_sync(0xffffffffu, acc[v][m], 16));
            if (g == 0 && v < (int)a.nvec && row >= a.r0 && row < a.r1)
                a.out[v][row] = __fsub_rn(__fadd_rn(__fadd_rn(x[0], x[2]), __fadd_rn(x[1], x[3])), corr[v]);
        }
    }
}

#define SG_TINST(DT)                                                                                         \
    template __global__ void gemv_tiled_kernel<DT, 1>(const __grid_constant__ TGemvArgs);                   \
    template __global__ void gemv_tiled_kernel<DT, 2>(const __grid_constant__ TGemvArgs);                   \
    template __global__ void gemv_tiled_kernel<DT, 4>(const __grid_constant__ TGemvArgs);                   \
    template __global__ void gemv_tiled_kernel<DT, 8>(const __grid_constant__ TGemvArgs);
SG_TINST(0)
SG_TINST(1)

// GGUF rows <-> TILED16 (inverse = 1: src is TILED16, dst GGUF rows).
// One thread per (row, super-block); padding rows of dst are left as they are.
__global__ void repack_tiled16_kernel(int dt, const uint8_t *src, uint64_t rows, uint32_t nb, uint8_t *dst,
                                      int inverse) {
    const uint64_t id = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * nb) return;
    const uint64_t row = id / nb;
    const uint32_t i = (uint32_t)(id % nb), r = (uint32_t)(row % TILE_ROWS);
    const uint32_t bb = dt == 0 ? 144u : 210u, cb = tiled_col_bytes(dt);
    const uint64_t g_off = (row * nb + i) * bb;
    const uint64_t t_off = (row / TILE_ROWS) * (uint64_t)nb * cb + (uint64_t)i * cb;
    // (offset in the GGUF block, offset in the tile column, length)
    uint32_t seg[3][3];
    int nseg;
    if (dt == 0) {
        seg[0][0] = 0, seg[0][1] = 2048 + 16 * r, seg[0][2] = 16;
        seg[1][0] = 16, seg[1][1] = 128 * r, seg[1][2] = 128;
        nseg = 2;
    } else {
        seg[0][0] = 0, seg[0][1] = 192 * r, seg[0][2] = 192;
        seg[1][0] = 192, seg[1][1] = 3072 + 16 * r, seg[1][2] = 16;
        seg[2][0] = 208, seg[2][1] = 3328 + 2 * r, seg[2][2] = 2;
        nseg = 3;
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
