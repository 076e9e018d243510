// kquant.cu — deterministic f32 -> Q4_K / Q6_K weight quantizer.
//
// The reference has no weight quantizer (its tests fill matrices with random
// bytes); this is the library's own algorithm, written from the block formats
// (q4k_gemv.rs:26-31 + :75-85, quant.rs:34-39 + :1634-1655).  Only correctly
// rounded operations are used (explicit _rn intrinsics, rintf = round to
// nearest even, f32->f16 RNE), so the bytes equal the CPU twin's for the same
// finite input.
//
// Q4_K, per 256 values, sub-block j of 32:
//   lo = min(0, min x), hi = max x, scale_j = (hi - lo)/15, m_j = -lo,
//   d = f16(max scale/63), dmin = f16(max m/63),
//   sc_j = clamp(rne(scale_j/d), 0, 63), mn_j = clamp(rne(m_j/dmin), 0, 63),
//   q = clamp(rne((x + dmin*mn_j)/(d*sc_j)), 0, 15).
// Q6_K, per 256 values, group g of 16:
//   scale_g = max|x|/31, d = f16(max scale/127),
//   sc_g = clamp(rne(scale_g/d), 0, 127), q = clamp(rne(x/(d*sc_g)), -32, 31) + 32.
// A divisor that is not positive gives 0.
#include "kernels.cuh"

namespace sg {

namespace {

__device__ __forceinline__ int qdiv(float a, float b, int lo, int hi) {
    if (!(b > 0.0f)) return 0;
    const float r = rintf(__fdiv_rn(a, b));
    if (r < (float)lo) return lo;
    if (r > (float)hi) return hi;
    return (int)r;
}

__device__ __forceinline__ void put_half(uint8_t *p, float v, float *back) {
    const __half h = __float2half_rn(v);
    *reinterpret_cast<unsigned short *>(p) = __half_as_ushort(h);  // p is 2-byte aligned
    *back = __half2float(h);
}

}  // namespace

__global__ void __launch_bounds__(128) quantize_q4k_kernel(const float *x, uint64_t nblocks, uint8_t *out) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float *v = x + b * 256u;
    uint8_t *blk = out + b * 144u;
    float scale[8], mval[8], smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; j++) {
        float lo = 0.0f, hi = v[32 * j];
        for (int i = 0; i < 32; i++) {
            const float t = v[32 * j + i];
            if (t < lo) lo = t;
            if (t > hi) hi = t;
        }
        scale[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        mval[j] = -lo;
        if (scale[j] > smax) smax = scale[j];
        if (mval[j] > mmax) mmax = mval[j];
    }
    float d, dmin;
    put_half(blk, __fdiv_rn(smax, 63.0f), &d);
    put_half(blk + 2, __fdiv_rn(mmax, 63.0f), &dmin);
    uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)qdiv(scale[j], d, 0, 63);
        mn[j] = (uint8_t)qdiv(mval[j], dmin, 0, 63);
    }
    for (int j = 0; j < 4; j++) {
        blk[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        blk[8 + j] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
        blk[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    for (int c = 0; c < 4; c++) {
        const float ws0 = __fmul_rn(d, (float)sc[2 * c]), wm0 = __fmul_rn(dmin, (float)mn[2 * c]);
        const float ws1 = __fmul_rn(d, (float)sc[2 * c + 1]), wm1 = __fmul_rn(dmin, (float)mn[2 * c + 1]);
        for (int l = 0; l < 32; l++) {
            const int q0 = qdiv(__fadd_rn(v[64 * c + l], wm0), ws0, 0, 15);
            const int q1 = qdiv(__fadd_rn(v[64 * c + 32 + l], wm1), ws1, 0, 15);
            blk[16 + 32 * c + l] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

__global__ void __launch_bounds__(128) quantize_q6k_kernel(const float *x, uint64_t nblocks, uint8_t *out) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float *v = x + b * 256u;
    uint8_t *blk = out + b * 210u;
    float scale[16], smax = 0.0f;
    for (int g = 0; g < 16; g++) {
        float m = 0.0f;
        for (int i = 0; i < 16; i++) {
            const float t = fabsf(v[16 * g + i]);
            if (t > m) m = t;
        }
        scale[g] = __fdiv_rn(m, 31.0f);
        if (scale[g] > smax) smax = scale[g];
    }
    float d;
    put_half(blk + 208, __fdiv_rn(smax, 127.0f), &d);
    float ws[16];
    for (int g = 0; g < 16; g++) {
        const int s = qdiv(scale[g], d, 0, 127);
        blk[192 + g] = (uint8_t)s;
        ws[g] = __fmul_rn(d, (float)s);
    }
    // element 128h + 32k + l: low nibble in ql[64h + 32(k&1) + l] (shift 4*(k>>1)),
    // 2 high bits in qh[32h + l] at bit 2k; its group is (128h + 32k + l) / 16.
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            uint32_t u[4];
            for (int k = 0; k < 4; k++) {
                const int e = 128 * h + 32 * k + l;
                u[k] = (uint32_t)(qdiv(v[e], ws[e / 16], -32, 31) + 32);
            }
            blk[64 * h + l] = (uint8_t)((u[0] & 15) | ((u[2] & 15) << 4));
            blk[64 * h + 32 + l] = (uint8_t)((u[1] & 15) | ((u[3] & 15) << 4));
            blk[128 + 32 * h + l] = (uint8_t)((u[0] >> 4) | ((u[1] >> 4) << 2) | ((u[2] >> 4) << 4) | ((u[3] >> 4) << 6));
        }
}

}  // namespace sg
