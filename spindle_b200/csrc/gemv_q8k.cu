// gemv_q8k.cu — kernel body of the Q4_K / Q6_K x Q8_K GEMV (see gemv_q8k.cuh).
#include "gemv_q8k.cuh"

namespace sg {

__device__ unsigned g_dev_status = 0;

namespace {

constexpr uint32_t M4 = 0x0F0F0F0Fu, M2 = 0x03030303u;

__device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

__device__ __forceinline__ int sbyte(uint32_t w, int b) { return (int)(int8_t)(w >> (8 * b)); }
__device__ __forceinline__ int ubyte(uint32_t w, int b) { return (int)((w >> (8 * b)) & 0xFFu); }

// Sum over the 8 consecutive lanes of one super-block (xor partners stay
// inside the group, so the group's mask suffices).
__device__ __forceinline__ int group8_sum(int v, unsigned mask) {
    v += __shfl_xor_sync(mask, v, 1);
    v += __shfl_xor_sync(mask, v, 2);
    v += __shfl_xor_sync(mask, v, 4);
    return v;
}

}  // namespace

template <int DT, int NV, int CPT, bool DBG>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_q8k_kernel(const __grid_constant__ GemvArgs a) {
    constexpr uint32_t BB = DT == DT_Q4K ? 144u : 210u;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint8_t *stages = smem + 128;
    int32_t *s_sum = reinterpret_cast<int32_t *>(stages + a.nstages * a.stage_bytes);
    const uint32_t nb = a.nb, rb = a.rb, R = a.R, ncol = nb * 8u;
    int32_t *s_corr = s_sum + R * NV * a.sum_stride;

    if (128u + a.nstages * a.stage_bytes + gemv_scratch_bytes(R, NV, nb, a.sum_stride) > dynamic_smem_size()) {
        if (threadIdx.x == 0) atomicExch(&g_dev_status, (unsigned)DEV_BAD_LAUNCH);
        return;
    }
    const uint32_t tid = threadIdx.x;
    const unsigned gmask = 0xFFu << (tid & 24u);

    // Column ownership: column c = 8*i + l is lane l of super-block i.
    const uint32_t P = CPT == 1 ? GEMV_THREADS / ncol : 1u;
    const uint32_t prow = CPT == 1 ? tid / ncol : 0u;
    uint32_t col[CPT];
    bool colok[CPT];
#pragma unroll
    for (int j = 0; j < CPT; j++) {
        uint32_t c = CPT == 1 ? tid % ncol : tid + (uint32_t)j * GEMV_THREADS;
        colok[j] = prow < P && c < ncol;
        col[j] = colok[j] ? c : 0u;
    }

    const uint32_t G = gridDim.x;
    const uint32_t cnt = blockIdx.x < a.ntiles ? (a.ntiles - blockIdx.x + G - 1) / G : 0u;

    // Producer (thread 0): stage k of this CTA's tile list.
    auto issue = [&](uint32_t k) {
        const uint32_t t = blockIdx.x + k * G;
        const uint32_t st = k % a.nstages;
        const uint64_t row0 = (uint64_t)a.r0 + (uint64_t)t * R;
        const uint32_t nr = (uint32_t)umin64((uint64_t)R, (uint64_t)a.r0 + a.nrows - row0);
        const uint64_t s = row0 * rb, e = s + (uint64_t)nr * rb;
        const uint64_t s_al = s & ~15ull;
        const uint64_t ce = umin64((e + 15ull) & ~15ull, a.tma_limit);
        const uint32_t bytes = ce > s_al ? (uint32_t)(ce - s_al) : 0u;
        uint8_t *dst = stages + st * a.stage_bytes;
        for (uint64_t p = ce > s_al ? ce : s_al; p < e; ++p) dst[p - s_al] = a.w[p];  // <16 B tensor tail
        mbar_arrive_expect_tx(&bars[st], bytes);
        if (bytes) bulk_g2s(dst, a.w + s_al, bytes, &bars[st]);
    };

    if (tid == 0) {
        for (uint32_t s = 0; s < a.nstages; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (uint32_t k = 0; k < cnt && k < a.nstages; k++) issue(k);

    uint32_t Y[CPT][NV][8];
    uint32_t BS[CPT][NV];
    auto load_act = [&](uint32_t g) {
#pragma unroll
        for (int j = 0; j < CPT; j++) {
            const uint32_t i = col[j] >> 3, l = col[j] & 7u;
#pragma unroll
            for (int v = 0; v < NV; v++) {
                const uint32_t vg = g * NV + v;
                const bool ok = colok[j] && vg < a.nvec;
                const int8_t *y = ok ? a.xs[vg] + i * 256u + 4u * l : nullptr;
#pragma unroll
                for (int k = 0; k < 8; k++) Y[j][v][k] = ok ? __ldg(reinterpret_cast<const uint32_t *>(y + 32 * k)) : 0u;
                BS[j][v] = ok ? __ldg(reinterpret_cast<const uint32_t *>(a.xb[vg] + i * 16u + 2u * l)) : 0u;
            }
        }
    };
    const uint32_t ngroups = (a.nvec + NV - 1) / NV;
    if (ngroups == 1) load_act(0);

    for (uint32_t k = 0; k < cnt; k++) {
        const uint32_t st = k % a.nstages;
        const bool ok = mbar_wait_bounded(&bars[st], (k / a.nstages) & 1u, WAIT_LIMIT_NS);
        if (__syncthreads_or(!ok)) {
            // Record, let in-flight copies land (bounded again), and leave.
            if (tid == 0) {
                atomicExch(&g_dev_status, (unsigned)DEV_TIMEOUT_TMA);
                for (uint32_t q = k; q < cnt && q < k + a.nstages; q++)
                    mbar_wait_bounded(&bars[q % a.nstages], (q / a.nstages) & 1u, WAIT_LIMIT_NS);
            }
            __syncthreads();
            return;
        }
        const uint32_t t = blockIdx.x + k * G;
        const uint64_t row0 = (uint64_t)a.r0 + (uint64_t)t * R;
        const uint32_t nr = (uint32_t)umin64((uint64_t)R, (uint64_t)a.r0 + a.nrows - row0);
        const uint8_t *stage = stages + st * a.stage_bytes;
        const uint32_t pre = (uint32_t)((row0 * rb) & 15ull);  // tile start inside the stage

        for (uint32_t g = 0; g < ngroups; g++) {
            if (ngroups > 1) load_act(g);
            const uint32_t nvg = min((uint32_t)NV, a.nvec - g * NV);

            // ---- phase A: exact int32 lane sums and correction sums --------
            for (uint32_t row = prow; row < nr; row += P) {
#pragma unroll
                for (int j = 0; j < CPT; j++) {
                    if (!colok[j]) continue;
                    const uint32_t i = col[j] >> 3, l = col[j] & 7u;
                    const uint32_t boff = pre + row * rb + i * BB;
                    if constexpr (DT == DT_Q4K) {
                        const uint8_t *blk = stage + boff;  // 16-aligned: 144 = 9*16, pre = 0
                        const uint32_t S0 = lds32(blk + 4), S1 = lds32(blk + 8), S2 = lds32(blk + 12);
                        const uint32_t sclo = S0 & 0x3F3F3F3Fu;
                        const uint32_t schi = (S2 & M4) | ((S0 >> 2) & 0x30303030u);
                        const uint32_t mnw = l < 4 ? (S1 & 0x3F3F3F3Fu) : (((S2 >> 4) & M4) | ((S1 >> 2) & 0x30303030u));
                        const int mn = ubyte(mnw, l & 3);
                        uint32_t lo[4], hi[4];
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint32_t q = lds32(blk + 16 + 32 * c + 4 * l);
                            lo[c] = q & M4;
                            hi[c] = (q >> 4) & M4;
                        }
                        const int sc[8] = {ubyte(sclo, 0), ubyte(sclo, 1), ubyte(sclo, 2), ubyte(sclo, 3),
                                           ubyte(schi, 0), ubyte(schi, 1), ubyte(schi, 2), ubyte(schi, 3)};
#pragma unroll
                        for (int v = 0; v < NV; v++) {
                            if (v >= (int)nvg) break;
                            int s = 0;
#pragma unroll
                            for (int c = 0; c < 4; c++) {
                                s += sc[2 * c] * __dp4a((int)lo[c], (int)Y[j][v][2 * c], 0);
                                s += sc[2 * c + 1] * __dp4a((int)hi[c], (int)Y[j][v][2 * c + 1], 0);
                            }
                            s_sum[(row * NV + v) * a.sum_stride + 8 * i + l] = s;
                            if (DBG && v == 0 && g == 0) a.dbg_sums[((row0 - a.r0) + row) * ncol + 8 * i + l] = s;
                            const uint32_t bp = BS[j][v];
                            int c8 = mn * ((int)(int16_t)(bp & 0xFFFFu) + (int)(int16_t)(bp >> 16));
                            c8 = group8_sum(c8, gmask);
                            if (l == 0) s_corr[(row * NV + v) * nb + i] = c8;
                        }
                    } else {
                        uint32_t w[8];
                        int sc[8];
                        const uint32_t hsel = l >= 4 ? 1u : 0u;
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t L0 = lds32_u2(stage, boff + 64 * h + 4 * l);
                            const uint32_t L1 = lds32_u2(stage, boff + 64 * h + 32 + 4 * l);
                            const uint32_t H = lds32_u2(stage, boff + 128 + 32 * h + 4 * l);
                            w[4 * h + 0] = (L0 & M4) | ((H & M2) << 4);
                            w[4 * h + 1] = (L1 & M4) | (((H >> 2) & M2) << 4);
                            w[4 * h + 2] = ((L0 >> 4) & M4) | (((H >> 4) & M2) << 4);
                            w[4 * h + 3] = ((L1 >> 4) & M4) | (((H >> 6) & M2) << 4);
                            const uint32_t W0 = lds32_u2(stage, boff + 192 + 8 * h);
                            const uint32_t W1 = lds32_u2(stage, boff + 196 + 8 * h);
                            // chunk 4h+k uses scale 8h + 2k + hsel
                            sc[4 * h + 0] = sbyte(W0, 0 + hsel);
                            sc[4 * h + 1] = sbyte(W0, 2 + hsel);
                            sc[4 * h + 2] = sbyte(W1, 0 + hsel);
                            sc[4 * h + 3] = sbyte(W1, 2 + hsel);
                        }
                        const uint32_t sp = *reinterpret_cast<const unsigned short *>(stage + boff + 192 + 2 * l);
#pragma unroll
                        for (int v = 0; v < NV; v++) {
                            if (v >= (int)nvg) break;
                            int s = 0;
#pragma unroll
                            for (int kk = 0; kk < 8; kk++) s += sc[kk] * __dp4a((int)w[kk], (int)Y[j][v][kk], 0);
                            s_sum[(row * NV + v) * a.sum_stride + 8 * i + l] = s;
                            if (DBG && v == 0 && g == 0) a.dbg_sums[((row0 - a.r0) + row) * ncol + 8 * i + l] = s;
                            const uint32_t bp = BS[j][v];
                            int c8 = sbyte(sp, 0) * (int)(int16_t)(bp & 0xFFFFu) + sbyte(sp, 1) * (int)(int16_t)(bp >> 16);
                            c8 = group8_sum(c8, gmask);
                            if (l == 0) s_corr[(row * NV + v) * nb + i] = 32 * c8;
                        }
                    }
                }
            }
            __syncthreads();

            // ---- phase B: per-lane FMA chain in block order, tree, correction
            const uint32_t njobs = nr * NV * 8u;
            for (uint32_t job = tid; job < njobs; job += GEMV_THREADS) {
                const uint32_t row = job / (NV * 8u), v = (job >> 3) % NV, l = job & 7u;
                if (v >= nvg) continue;  // uniform across the 8 lanes
                const float *xdv = a.xd[g * NV + v];
                const uint8_t *rowp = stage + pre + row * rb;
                const int32_t *ss = s_sum + (row * NV + v) * a.sum_stride + l;
                float acc = 0.0f;
                for (uint32_t i = 0; i < nb; i++) {
                    const float d = half_at(rowp + i * BB + (DT == DT_Q4K ? 0u : 208u));
                    acc = __fmaf_rn(__fmul_rn(d, __ldg(xdv + i)), __int2float_rn(ss[8 * i]), acc);
                }
                acc = __fadd_rn(acc, __shfl_xor_sync(gmask, acc, 4));
                acc = __fadd_rn(acc, __shfl_xor_sync(gmask, acc, 2));
                acc = __fadd_rn(acc, __shfl_xor_sync(gmask, acc, 1));
                if (l == 0) {
                    const int32_t *cs = s_corr + (row * NV + v) * nb;
                    float corr = 0.0f;
                    for (uint32_t i = 0; i < nb; i++) {
                        const float dm = half_at(rowp + i * BB + (DT == DT_Q4K ? 2u : 208u));
                        corr = __fadd_rn(corr, __fmul_rn(__fmul_rn(dm, __ldg(xdv + i)), __int2float_rn(cs[i])));
                    }
                    a.out[g * NV + v][row0 + row] = __fsub_rn(acc, corr);
                }
            }
            __syncthreads();
        }
        if (tid == 0 && k + a.nstages < cnt) issue(k + a.nstages);
    }
}

// Instantiations: NV * CPT <= 8 keeps the activation registers at <= 72.
#define SG_INST(DT, NV, CPT)                                                                       \
    template __global__ void gemv_q8k_kernel<DT, NV, CPT, false>(const __grid_constant__ GemvArgs); \
    template __global__ void gemv_q8k_kernel<DT, NV, CPT, true>(const __grid_constant__ GemvArgs);
#define SG_INST_DT(DT)                                                                                      \
    SG_INST(DT, 1, 1) SG_INST(DT, 2, 1) SG_INST(DT, 3, 1) SG_INST(DT, 4, 1) SG_INST(DT, 5, 1)              \
    SG_INST(DT, 6, 1) SG_INST(DT, 7, 1) SG_INST(DT, 8, 1) SG_INST(DT, 1, 2) SG_INST(DT, 2, 2)              \
    SG_INST(DT, 3, 2) SG_INST(DT, 4, 2) SG_INST(DT, 1, 4) SG_INST(DT, 2, 4) SG_INST(DT, 1, 8)
SG_INST_DT(DT_Q4K)
SG_INST_DT(DT_Q6K)

}  // namespace sg
