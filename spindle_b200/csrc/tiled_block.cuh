// tiled_block.cuh — per-super-block math of the TILED16 GEMV kernels, shared
// by the single-matrix GEMV (gemv_tiled.cu) and the grouped MoE GEMVs (moe.cu).
// See gemv_tiled.cuh for the layout and the exactness argument.
#pragma once

#include "gemv_tiled.cuh"
#include "glibc_math.h"

namespace sg {

namespace tiled {

constexpr uint32_t M4 = 0x0F0F0F0Fu, B45 = 0x30303030u;

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint32_t w4(const uint4 &v, int m) { return m == 0 ? v.x : m == 1 ? v.y : m == 2 ? v.z : v.w; }
__device__ __forceinline__ int sbyte(uint32_t w, int b) { return (int)(int8_t)(w >> (8 * b)); }
__device__ __forceinline__ int ubyte(uint32_t w, int b) { return (int)((w >> (8 * b)) & 0xFFu); }
// dot of 4 unsigned bytes of a with 4 signed bytes of b
__device__ __forceinline__ int dp4a_us(uint32_t a, int b) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(0));
    return d;
}
__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

// float(s), exact.  Q4_K lane sums satisfy |s| < 2^22, so 1.5*2^23 + s is an
// exact float whose bits are 0x4B400000 + s; subtracting 1.5*2^23 is exact
// too (two ALU/FMA ops instead of a conversion).  Q6_K sums can reach 2^25 and
// use the rounding conversion.
template <int DT>
__device__ __forceinline__ float lane_f(int s) {
    if constexpr (DT == 0) return __fsub_rn(__int_as_float(0x4B400000 + s), 12582912.0f);
    return __int2float_rn(s);
}

// TILED16 stores each row's quant bytes in 16-byte chunks permuted by row so
// that the 8 rows an LDS.128 phase reads fall in 8 different bank groups:
//   Q4_K qs (8 chunks/row):    chunk c at c ^ (r & 7)
//   Q6_K qlqh (12 chunks/row): chunk c at (c & ~3) | ((c ^ (r >> 1)) & 3)
__host__ __device__ __forceinline__ uint32_t q4k_chunk(uint32_t c, uint32_t r) { return c ^ (r & 7u); }
__host__ __device__ __forceinline__ uint32_t q6k_chunk(uint32_t c, uint32_t r) {
    return (c & ~3u) | ((c ^ (r >> 1)) & 3u);
}

// Programmatic dependent launch: wait for the grids this one depends on
// (no-op when launched without the attribute), and let dependents launch.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// exp for the reference's f32::exp: glibc's expf, bit for bit (what f32::exp
// calls on Linux; glibc_math.h restates it).
__device__ __forceinline__ float expf_ref(float x) { return gm_expf(x); }

// silu(x) * u with the reference's roundings (smollm_chat.rs:586-588, :411):
// x / (1 + exp(-x)), then times u.
__device__ __forceinline__ float silu_mul(float x, float u) {
    const float e = expf_ref(-x);
    return __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, e)), u);
}


__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_arrive(uint32_t id, uint32_t n) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// The same per-block arithmetic split in two, so that a kernel running
// several vectors decodes a block's weights once (q4k_weights / q6k_weights)
// and then takes the vectors one at a time (q4k_dot / q6k_dot), each
// vector's lane sums consumed before the next is computed (few live registers).
struct Q4KWeights {
    uint32_t lo[4][4], hi[4][4];
    int sc[8];
    float d, dmin;
    uint32_t mnw;
};

__device__ __forceinline__ void q4k_weights(const uint8_t *col, uint32_t g, uint32_t r, Q4KWeights &w) {
    const uint4 hd = lds128(col + 2048 + 16 * r);
    w.d = h2f_lo(hd.x);
    w.dmin = h2f_hi(hd.x);
    const uint32_t sclo = hd.y & 0x3F3F3F3Fu, schi = (hd.w & M4) | ((hd.y >> 2) & B45);
    w.mnw = g ? (((hd.w >> 4) & M4) | ((hd.z >> 2) & B45)) : (hd.z & 0x3F3F3F3Fu);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        w.sc[k] = ubyte(sclo, k);
        w.sc[k + 4] = ubyte(schi, k);
    }
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        const uint4 qv = lds128(col + 128 * r + 16 * q4k_chunk(2 * cc + g, r));
#pragma unroll
        for (int m = 0; m < 4; m++) {
            w.lo[cc][m] = w4(qv, m) & M4;
            w.hi[cc][m] = w4(qv, m) & 0xF0F0F0F0u;
        }
    }
}

// av: one vector's activation image; s: the int32 lane sums of lanes 4g..4g+3
// of row r, cd = d * xd, ct: the min correction term, for that vector
__device__ __forceinline__ void q4k_dot(const Q4KWeights &w, uint32_t g, uint32_t i, uint32_t nb, const uint8_t *av,
                                        int (&s)[4], float &cd, float &ct) {
    const uint8_t *y = av + 256u * i + 16u * g;
    const float xd = *reinterpret_cast<const float *>(av + 288u * nb + 4u * i);
    int sh[4];
#pragma unroll
    for (int m = 0; m < 4; m++) s[m] = sh[m] = 0;
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        const uint4 Ylo = lds128(y + 64 * cc), Yhi = lds128(y + 64 * cc + 32);
#pragma unroll
        for (int m = 0; m < 4; m++) {
            s[m] += w.sc[2 * cc] * __dp4a((int)w.lo[cc][m], (int)w4(Ylo, m), 0);
            sh[m] += w.sc[2 * cc + 1] * dp4a_us(w.hi[cc][m], (int)w4(Yhi, m));
        }
    }
#pragma unroll
    for (int m = 0; m < 4; m++) s[m] += sh[m] >> 4;
    cd = __fmul_rn(w.d, xd);
    const uint4 B = lds128(av + 256u * nb + 32u * i + 16u * g);
    int sp = 0;
#pragma unroll
    for (int m = 0; m < 4; m++) sp = __dp2a_lo((int)w4(B, m), (int)__byte_perm(w.mnw, 0, 0x11 * m), sp);
    sp += __shfl_xor_sync(0xffffffffu, sp, 16);
    ct = __fmul_rn(__fmul_rn(w.dmin, xd), __int2float_rn(sp));
}

struct Q6KWeights {
    uint32_t w[8][4];
    int scv[8];
    float d;
    uint32_t sw0, sw1;
};

__device__ __forceinline__ void q6k_weights(const uint8_t *col, uint32_t g, uint32_t r, Q6KWeights &q) {
    const uint8_t *qrow = col + 192 * r;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint4 L0 = lds128(qrow + 16 * q6k_chunk(4 * h + g, r));
        const uint4 L1 = lds128(qrow + 16 * q6k_chunk(4 * h + 2 + g, r));
        const uint4 H = lds128(qrow + 16 * q6k_chunk(8 + 2 * h + g, r));
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const uint32_t l0 = w4(L0, m), l1 = w4(L1, m), hh = w4(H, m);
            q.w[4 * h + 0][m] = (l0 & M4) | ((hh << 4) & B45);
            q.w[4 * h + 1][m] = (l1 & M4) | ((hh << 2) & B45);
            q.w[4 * h + 2][m] = ((l0 >> 4) & M4) | (hh & B45);
            q.w[4 * h + 3][m] = ((l1 >> 4) & M4) | ((hh >> 2) & B45);
        }
    }
    const uint4 SC = lds128(col + 3072 + 16 * r);
    q.d = __half2float(*reinterpret_cast<const __half *>(col + 3328 + 2 * r));
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) q.scv[4 * h + kk] = sbyte(w4(SC, 2 * h + (kk >> 1)), 2 * (kk & 1) + (int)g);
    q.sw0 = g ? SC.z : SC.x;
    q.sw1 = g ? SC.w : SC.y;
}

__device__ __forceinline__ void q6k_dot(const Q6KWeights &q, uint32_t g, uint32_t i, uint32_t nb, const uint8_t *av,
                                        int (&s)[4], float &cd, float &ct) {
    const uint8_t *y = av + 256u * i + 16u * g;
    const float xd = *reinterpret_cast<const float *>(av + 288u * nb + 4u * i);
#pragma unroll
    for (int m = 0; m < 4; m++) s[m] = 0;
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
        const uint4 Y = lds128(y + 32 * kk);
#pragma unroll
        for (int m = 0; m < 4; m++) s[m] += q.scv[kk] * __dp4a((int)q.w[kk][m], (int)w4(Y, m), 0);
    }
    cd = __fmul_rn(q.d, xd);
    const uint4 B = lds128(av + 256u * nb + 32u * i + 16u * g);
    int sp = __dp2a_lo((int)B.x, (int)q.sw0, 0);
    sp = __dp2a_hi((int)B.y, (int)q.sw0, sp);
    sp = __dp2a_lo((int)B.z, (int)q.sw1, sp);
    sp = __dp2a_hi((int)B.w, (int)q.sw1, sp);
    sp += __shfl_xor_sync(0xffffffffu, sp, 16);
    ct = __fmul_rn(cd, __int2float_rn(32 * sp));
}


}  // namespace tiled

}  // namespace sg
