// q8k.cu — Q8_K activation quantizer (Q8K::quantize, quant_q8k.rs:73-121),
// bit-identical to the reference's AVX2 code for every input, including
// NaN/Inf and all-zero blocks.
//
// One warp per 256-value block.  The reference's amax is a running MAXPS over
// 8 lanes (lane j sees x[j], x[j+8], ...; MAXPS returns its second operand
// when either is NaN), then a fixed hi->lo, 2->0, 1->0 fold: lanes 0..7 replay
// exactly that.  Each value becomes cvtps_epi32(x * (127/amax)) saturated to
// int8 by two packs: round-to-nearest-even, and NaN or |v| >= 2^31 gives
// INT32_MIN, i.e. -128.
#include "kernels.cuh"

namespace sg {

namespace {

// MAXPS(a, b): a if a > b, else b (b on NaN).
__device__ __forceinline__ float maxps(float a, float b) { return a > b ? a : b; }

__device__ __forceinline__ int8_t cvt_pack(float v) {
    if (isnan(v) || fabsf(v) >= 2147483648.0f) return -128;
    int q = __float2int_rn(v);
    return (int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
}

}  // namespace

__global__ void __launch_bounds__(256) q8k_quantize_kernel(const __grid_constant__ Q8kArgs a) {
    // Programmatic dependent launch: let the next kernel (the GEMV that reads
    // this output) launch now, so its weight prefetch overlaps this kernel and
    // the one before it; then wait for the kernel that wrote x.
    asm volatile("griddepcontrol.launch_dependents;" :::);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
    if (warp >= a.nb * a.nvec) return;
    const uint32_t vec = warp / a.nb, b = warp % a.nb;
    const float *xb = a.x + vec * a.ldx + (uint64_t)b * 256u;
    const sg_q8k o = a.outs[vec];

    float lm = 0.0f;
    if (lane < 8)
        for (int m = 0; m < 32; m++) lm = maxps(lm, fabsf(xb[8 * m + lane]));
    // _mm_max_ps(lo, hi); _mm_max_ps(v, movehl(v, v)); _mm_max_ss(v, shuffle(v, 0x55))
    const float hi4 = __shfl_down_sync(0xffffffffu, lm, 4);
    const float v4 = maxps(lm, hi4);
    const float v2 = maxps(v4, __shfl_down_sync(0xffffffffu, v4, 2));
    const float amax = __shfl_sync(0xffffffffu, maxps(v2, __shfl_down_sync(0xffffffffu, v2, 1)), 0);

    int8_t q[8];
    if (!(amax > 0.0f) || isinf(amax)) {
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = 0;
        if (lane == 0) o.d[b] = 0.0f;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
        if (lane == 0) o.d[b] = __fdiv_rn(amax, 127.0f);
        const float4 p0 = reinterpret_cast<const float4 *>(xb)[2 * lane];
        const float4 p1 = reinterpret_cast<const float4 *>(xb)[2 * lane + 1];
        const float xv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = cvt_pack(__fmul_rn(xv[k], inv));
    }
    uint32_t w0 = 0, w1 = 0;
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        w0 |= (uint32_t)(uint8_t)q[k] << (8 * k);
        w1 |= (uint32_t)(uint8_t)q[k + 4] << (8 * k);
    }
#pragma unroll
    for (int k = 0; k < 8; k++) s += q[k];
    reinterpret_cast<uint2 *>(o.qs + (uint64_t)b * 256u)[lane] = make_uint2(w0, w1);
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // group of 16 values = lanes 2g, 2g+1
    if ((lane & 1u) == 0) o.bsums[b * 16u + lane / 2] = (int16_t)s;
}

}  // namespace sg
