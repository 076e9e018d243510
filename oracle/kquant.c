/*
 * kquant.c — f32 -> Q4_K / Q6_K weight quantizer, CPU twin of the product's
 * CUDA quantizer (spindle_b200/csrc/kquant.cu).  TEST INFRASTRUCTURE ONLY.
 *
 * The reference has no weight quantizer (its tests build matrices from random
 * bytes); this is the build's own deterministic algorithm, written from the
 * block formats (q4k_gemv.rs:26-31 + :75-85 for Q4_K, quant.rs:34-39 +
 * :1634-1655 for Q6_K).  It uses only correctly rounded IEEE operations
 * (+, -, *, /, round-to-nearest-even, f32 -> f16 RNE), so the GPU and this
 * file produce identical bytes for the same finite input.
 *
 * Q4_K, per 256 values and sub-block j of 32:
 *   lo_j = min(0, min x), hi_j = max x, scale_j = (hi_j - lo_j) / 15, m_j = -lo_j
 *   d = f16(max_j scale_j / 63), dmin = f16(max_j m_j / 63)
 *   sc_j = clamp(rne(scale_j / d), 0, 63), mn_j = clamp(rne(m_j / dmin), 0, 63)
 *   q = clamp(rne((x + dmin*mn_j) / (d*sc_j)), 0, 15)
 * Q6_K, per 256 values and group g of 16:
 *   scale_g = max|x| / 31, d = f16(max_g scale_g / 127)
 *   sc_g = clamp(rne(scale_g / d), 0, 127), q = clamp(rne(x / (d*sc_g)), -32, 31) + 32
 * A zero divisor gives 0 for the scale or quant it would produce.
 */
#include <immintrin.h>
#include <math.h>
#include <string.h>

#include "sg_oracle.h"

__attribute__((target("f16c"))) static uint16_t to_half(float v)
{
    return (uint16_t)_cvtss_sh(v, 0);
}

/* rne(a / b), clamped; 0 when b is not positive. */
static int qdiv(float a, float b, int lo, int hi)
{
    if (!(b > 0.0f)) return 0;
    float r = rintf(a / b);
    if (r < (float)lo) return lo;
    if (r > (float)hi) return hi;
    return (int)r;
}

void or_quantize_q4k(const float *x, size_t n, uint8_t *out)
{
    for (size_t b = 0; b < n / 256; b++) {
        const float *v = x + b * 256;
        uint8_t *blk = out + b * 144;
        float scale[8], mval[8], smax = 0.0f, mmax = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = v[32 * j];
            for (int i = 0; i < 32; i++) {
                float t = v[32 * j + i];
                if (t < lo) lo = t;
                if (t > hi) hi = t;
            }
            scale[j] = (hi - lo) / 15.0f;
            mval[j] = -lo;
            if (scale[j] > smax) smax = scale[j];
            if (mval[j] > mmax) mmax = mval[j];
        }
        uint16_t dh = to_half(smax / 63.0f), mh = to_half(mmax / 63.0f);
        float d = or_f16_to_f32(dh), dmin = or_f16_to_f32(mh);
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)qdiv(scale[j], d, 0, 63);
            mn[j] = (uint8_t)qdiv(mval[j], dmin, 0, 63);
        }
        blk[0] = (uint8_t)dh; blk[1] = (uint8_t)(dh >> 8);
        blk[2] = (uint8_t)mh; blk[3] = (uint8_t)(mh >> 8);
        for (int j = 0; j < 4; j++) {
            blk[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
            blk[8 + j] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
            blk[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
        }
        uint8_t q[256];
        for (int j = 0; j < 8; j++) {
            float ws = d * (float)sc[j], wm = dmin * (float)mn[j];
            for (int i = 0; i < 32; i++) q[32 * j + i] = (uint8_t)qdiv(v[32 * j + i] + wm, ws, 0, 15);
        }
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++) blk[16 + 32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
}

void or_quantize_q6k(const float *x, size_t n, uint8_t *out)
{
    for (size_t b = 0; b < n / 256; b++) {
        const float *v = x + b * 256;
        uint8_t *blk = out + b * 210;
        float scale[16], smax = 0.0f;
        for (int g = 0; g < 16; g++) {
            float a = 0.0f;
            for (int i = 0; i < 16; i++) {
                float t = fabsf(v[16 * g + i]);
                if (t > a) a = t;
            }
            scale[g] = a / 31.0f;
            if (scale[g] > smax) smax = scale[g];
        }
        uint16_t dh = to_half(smax / 127.0f);
        float d = or_f16_to_f32(dh);
        int8_t sc[16];
        uint8_t u[256];
        for (int g = 0; g < 16; g++) {
            sc[g] = (int8_t)qdiv(scale[g], d, 0, 127);
            float ws = d * (float)sc[g];
            for (int i = 0; i < 16; i++) u[16 * g + i] = (uint8_t)(qdiv(v[16 * g + i], ws, -32, 31) + 32);
        }
        memset(blk, 0, 192);
        for (int h = 0; h < 2; h++)
            for (int k = 0; k < 4; k++)
                for (int l = 0; l < 32; l++) {
                    uint8_t q = u[128 * h + 32 * k + l];
                    int lq = 64 * h + (k & 1) * 32 + l;
                    blk[lq] |= (uint8_t)((q & 15) << ((k >> 1) * 4));
                    blk[128 + 32 * h + l] |= (uint8_t)((q >> 4) << (2 * k));
                }
        memcpy(blk + 192, sc, 16);
        blk[208] = (uint8_t)dh;
        blk[209] = (uint8_t)(dh >> 8);
    }
}
