// q8k_block.cuh — one warp quantizes one 256-value block to Q8_K exactly as
// Q8K::quantize / quantize_avx2 (quant_q8k.rs:73-121) does, bit for bit,
// including NaN/Inf and all-zero blocks.
//
// amax: the reference keeps 8 running MAXPS lanes (lane j sees x[j], x[j+8],
// ...; MAXPS returns its second operand when either is NaN), then folds
// hi->lo, 2->0, 1->0.  Without a NaN in the block that is the plain maximum,
// whatever the order; a NaN makes a lane keep only what follows its last NaN,
// so that (rare) case replays the lane folds in order.  Each value becomes
// cvtps_epi32(x * (127/amax)) saturated to int8 by two packs: round to
// nearest even, and NaN or |v| >= 2^31 give INT32_MIN, i.e. -128.
// d = amax/127 and 127/amax are correctly rounded divisions.
#pragma once

#include "common.cuh"

namespace sg {

__device__ __forceinline__ float maxps(float a, float b) { return a > b ? a : b; }

__device__ __forceinline__ int8_t cvt_pack_i8(float v) {
    if (isnan(v) || fabsf(v) >= 2147483648.0f) return -128;
    const int q = __float2int_rn(v);
    return (int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
}

// The block's amax; lane t holds x[8t .. 8t+7] in xv (so xv[j] is element t
// of AVX lane j).  Returned to every lane.
__device__ __forceinline__ float q8k_amax(const float (&xv)[8], uint32_t lane) {
    bool nan = false;
#pragma unroll
    for (int k = 0; k < 8; k++) nan |= isnan(xv[k]);
    if (!__any_sync(0xffffffffu, nan)) {
        float m = fabsf(xv[0]);
#pragma unroll
        for (int k = 1; k < 8; k++) m = fmaxf(m, fabsf(xv[k]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        return m;
    }
    // in-order replay: lane j < 8 folds x[j], x[j+8], ..., fetched from lane m
    float lm = 0.0f;
    for (int m = 0; m < 32; m++) {
        float v = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
            const float t = __shfl_sync(0xffffffffu, xv[jj], m);
            if (jj == (int)(lane & 7u)) v = t;
        }
        lm = maxps(lm, fabsf(v));
    }
    const float v4 = maxps(lm, __shfl_down_sync(0xffffffffu, lm, 4));
    const float v2 = maxps(v4, __shfl_down_sync(0xffffffffu, v4, 2));
    return __shfl_sync(0xffffffffu, maxps(v2, __shfl_down_sync(0xffffffffu, v2, 1)), 0);
}

// Values in registers (lane t: x[8t .. 8t+7]); qs: 256 int8 (8-byte aligned);
// bsums: 16 int16; d: one float.  All 32 lanes of the warp call it.
//
// Fast path (no NaN or Inf in the block, 127/amax finite): |x * (127/amax)|
// stays below 127.5, so cvtps_epi32 needs no saturation, and adding 1.5 * 2^23
// to the rounded product rounds it to the nearest integer, ties to even, as
// cvtps_epi32 does: the low byte of the sum's bits is the int8 value.  Any
// other block takes the general path, which replays the reference's NaN,
// Inf and overflow behaviour.
__device__ __forceinline__ void q8k_block_regs(const float (&xv)[8], int8_t *qs, int16_t *bsums, float *d,
                                               uint32_t lane) {
    bool special = false;
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float a = fabsf(xv[k]);
        special |= !(a <= 3.402823466e38f);  // NaN or Inf
        m = fmaxf(m, a);
    }
    uint32_t w0 = 0, w1 = 0;
    bool general = __any_sync(0xffffffffu, special);
    if (!general) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (m > 0.0f) {
            const float inv = __fdiv_rn(127.0f, m);
            if (isinf(inv)) {
                general = true;  // a subnormal amax: the products overflow
            } else {
                if (lane == 0) *d = __fdiv_rn(m, 127.0f);
                uint32_t u[8];
#pragma unroll
                for (int k = 0; k < 8; k++) u[k] = __float_as_uint(__fadd_rn(__fmul_rn(xv[k], inv), 12582912.0f));
                w0 = __byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410);
                w1 = __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410);
            }
        } else if (lane == 0) {
            *d = 0.0f;  // all zero: d = 0, q = 0
        }
    }
    if (general) {
        const float amax = q8k_amax(xv, lane);
        int8_t q[8];
        if (!(amax > 0.0f) || isinf(amax)) {
#pragma unroll
            for (int k = 0; k < 8; k++) q[k] = 0;
            if (lane == 0) *d = 0.0f;
        } else {
            const float inv = __fdiv_rn(127.0f, amax);
            if (lane == 0) *d = __fdiv_rn(amax, 127.0f);
#pragma unroll
            for (int k = 0; k < 8; k++) q[k] = cvt_pack_i8(__fmul_rn(xv[k], inv));
        }
        w0 = w1 = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            w0 |= (uint32_t)(uint8_t)q[k] << (8 * k);
            w1 |= (uint32_t)(uint8_t)q[k + 4] << (8 * k);
        }
    }
    int s = __dp4a((int)w0, 0x01010101, __dp4a((int)w1, 0x01010101, 0));
    reinterpret_cast<uint2 *>(qs)[lane] = make_uint2(w0, w1);
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // a group of 16 values = lanes 2g, 2g+1
    if ((lane & 1u) == 0) bsums[lane / 2] = (int16_t)s;
}

// xb: 256 floats (16-byte aligned, global or shared), read once.
__device__ __forceinline__ void q8k_block(const float *xb, int8_t *qs, int16_t *bsums, float *d, uint32_t lane) {
    const float4 p0 = reinterpret_cast<const float4 *>(xb)[2 * lane];
    const float4 p1 = reinterpret_cast<const float4 *>(xb)[2 * lane + 1];
    const float xv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    q8k_block_regs(xv, qs, bsums, d, lane);
}

}  // namespace sg
