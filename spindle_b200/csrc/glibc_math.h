/*
 * glibc_math.h — expf, sinf and cosf that return, bit for bit, what glibc's
 * single-precision functions return on an x86_64 host with FMA.
 *
 * Why: the reference calls f32::exp (SiLU, the router softmax, the attention
 * softmax; smollm_chat.rs:586-588, :1200-1203, :3463-3495) and f32::sin_cos
 * (RoPE, smollm_chat.rs:1397-1420).  Rust's std takes those from the platform
 * libm: on Linux, glibc's expf / sinf / cosf.  These are accurate to about
 * half an ulp but not correctly rounded, so a kernel that computes the
 * correctly rounded value differs from the reference by one ulp now and then,
 * and through the next Q8_K quantization that grows into a visible logit
 * difference.  Computing glibc's own algorithm on the device removes that.
 *
 * Algorithm: glibc (since 2.28) ships the single-precision routines of ARM's
 * optimized-routines project (MIT / Apache-2.0 with LLVM exception), files
 * math/expf.c, math/exp2f_data.c, math/sinf.c, math/cosf.c, math/sincosf.h
 * and math/sincosf_data.c.  This file restates those published algorithms:
 *
 *   expf:  x * 32/ln2 = k + r (k rounded to nearest through the 1.5*2^52
 *          shift), 2^(k/32) from a 32-entry table with the exponent added to
 *          its bits, 2^(r/32) by a cubic, everything in double, then one
 *          rounding to float.
 *   sinf / cosf:  |x| < pi/4 straight polynomials in double; |x| < 120 a
 *          reduction x - n*pi/2 with n = round(x*2/pi); larger |x| an exact
 *          integer reduction against 192 bits of 2/pi (24-bit windows of the
 *          mantissa times 32-bit words of the table); odd and even
 *          polynomials of degree 7 and 8 in double, the quadrant picking
 *          sin or cos and the sign.
 *
 * The glibc build that x86_64 hosts with FMA run (the ifunc variants
 * __expf_fma, __sinf_fma, __cosf_fma) is compiled with contraction, so some
 * a*b+c steps are single fused operations; each operation below is written
 * explicitly as a fused or a separately rounded step to match that build.
 * The tables are not copied: the 2^(i/32) entries, 2/pi, pi/2 and the 2/pi
 * bit windows follow from their definitions (computed in high precision and
 * rounded to the nearest double); only the polynomial coefficients, which are
 * minimax fits of the published algorithm, are data.  tests/test_libm.py
 * compares this header with the host's glibc over every float input, and the
 * GPU test with the device build over a stride of all inputs.
 *
 * NaN payloads are not matched (a NaN in gives a NaN out).  Usable from C
 * (the CPU check, compiled with -ffp-contract=off) and from CUDA device code.
 */
#ifndef SG_GLIBC_MATH_H
#define SG_GLIBC_MATH_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define GM_FN static __device__ __forceinline__
#define GM_TABLE static __device__ const
#define GM_MUL(a, b) __dmul_rn((a), (b))
#define GM_ADD(a, b) __dadd_rn((a), (b))
#define GM_SUB(a, b) __dsub_rn((a), (b))
#define GM_FMA(a, b, c) __fma_rn((a), (b), (c))
#define GM_D2F(d) __double2float_rn(d)
#define GM_F2D(f) ((double)(f))
#define GM_I2D(i) __int2double_rn(i)
#define GM_LL2D(i) __ll2double_rn(i)
#define GM_D2I_RZ(d) __double2int_rz(d)
GM_FN uint64_t gm_asu64(double d) { return (uint64_t)__double_as_longlong(d); }
GM_FN double gm_asdouble(uint64_t u) { return __longlong_as_double((long long)u); }
GM_FN uint32_t gm_asu32(float f) { return (uint32_t)__float_as_uint(f); }
#else
#include <math.h>
#define GM_FN static inline
#define GM_TABLE static const
#define GM_MUL(a, b) ((a) * (b))
#define GM_ADD(a, b) ((a) + (b))
#define GM_SUB(a, b) ((a) - (b))
#define GM_FMA(a, b, c) fma((a), (b), (c))
#define GM_D2F(d) ((float)(d))
#define GM_F2D(f) ((double)(f))
#define GM_I2D(i) ((double)(i))
#define GM_LL2D(i) ((double)(i))
#define GM_D2I_RZ(d) ((int32_t)(d))
GM_FN uint64_t gm_asu64(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }
GM_FN double gm_asdouble(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
GM_FN uint32_t gm_asu32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
#endif

/* ---- expf ---------------------------------------------------------------- */

/* bits of RN(2^(i/32)) minus i << 47, so that adding k << 47 for k = 32q + i
   multiplies the entry by 2^q (optimized-routines exp2f_data.c layout) */
GM_TABLE uint64_t gm_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

GM_FN float gm_expf(float x) {
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32; /* 32 / ln 2 */
    const double shift = 0x1.8p+52;                     /* rounds to an integer */
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const uint32_t ux = gm_asu32(x);
    const uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) { /* |x| >= 88 or NaN */
        if (ux == 0xff800000u) return 0.0f;           /* -inf */
        if (abstop >= 0x7f8) return x + x;            /* +inf, NaN */
        if (x > 0x1.62e42ep6f) return (float)INFINITY; /* overflow */
        if (x < -0x1.9fe368p6f) return 0.0f;           /* underflow */
        if (x < -0x1.9d1d9ep6f) return 0x1p-149f;      /* may underflow: the smallest subnormal */
    }
    const double xd = GM_F2D(x);
    /* the FMA build fuses the product into both uses of z = x * 32/ln2 */
    double kd = GM_FMA(inv_ln2_n, xd, shift);
    const uint64_t ki = gm_asu64(kd);
    kd = GM_SUB(kd, shift);
    const double r = GM_FMA(inv_ln2_n, xd, -kd);
    uint64_t t = gm_exp2_tab[ki & 31];
    t += ki << 47;
    const double s = gm_asdouble(t);
    const double z = GM_FMA(c0, r, c1);
    const double r2 = GM_MUL(r, r);
    double y = GM_FMA(c2, r, 1.0);
    y = GM_FMA(z, r2, y);
    y = GM_MUL(y, s);
    return GM_D2F(y);
}

/* ---- sinf / cosf --------------------------------------------------------- */

/* 32-bit windows of the binary expansion of 2/pi: entry i holds the bits
   8i+1 .. 8i+32 after the binary point (floor(2/pi * 2^(8(i+1))) mod 2^32) */
GM_TABLE uint32_t gm_inv_pio4[24] = {
    0xa2,       0xa2f9,     0xa2f983,   0xa2f9836e, 0xf9836e4e, 0x836e4e44, 0x6e4e4415, 0x4e441529,
    0x441529fc, 0x1529fc27, 0x29fc2757, 0xfc2757d1, 0x2757d1f5, 0x57d1f534, 0xd1f534dd, 0xf534ddc0,
    0x34ddc0db, 0xddc0db62, 0xc0db6295, 0xdb629599, 0x6295993c, 0x95993c43, 0x993c4390, 0x3c439041,
};

/* cos polynomial c0..c4 (c0 = +-1 selects the sign of the quadrant), sin
   polynomial s1..s3; index 1 is the negated cos polynomial used for the
   quadrants where cos enters with a minus sign */
#define GM_C1 (-0x1.ffffffd0c621cp-2)
#define GM_C2 (0x1.55553e1068f19p-5)
#define GM_C3 (-0x1.6c087e89a359dp-10)
#define GM_C4 (0x1.99343027bf8c3p-16)
#define GM_S1 (-0x1.555545995a603p-3)
#define GM_S2 (0x1.1107605230bc4p-7)
#define GM_S3 (-0x1.994eb3774cf24p-13)

/* |x| <= pi/4: sin(x) for even n, cos(x) for odd n; neg flips the cos
   polynomial (the second table of the published code) */
GM_FN float gm_sincos_poly(double x, double x2, int neg, int n) {
    if ((n & 1) == 0) {
        const double x3 = GM_MUL(x, x2);
        const double s1 = GM_FMA(x2, GM_S3, GM_S2);
        const double x5 = GM_MUL(x3, x2);
        const double s = GM_FMA(x3, GM_S1, x);
        return GM_D2F(GM_FMA(x5, s1, s));
    } else {
        const double sg = neg ? -1.0 : 1.0;
        const double x4 = GM_MUL(x2, x2);
        const double c2 = GM_FMA(x2, sg * GM_C4, sg * GM_C3);
        const double c1 = GM_FMA(x2, sg * GM_C1, sg);
        const double x6 = GM_MUL(x4, x2);
        const double c = GM_FMA(x4, sg * GM_C2, c1);
        return GM_D2F(GM_FMA(x6, c2, c));
    }
}

/* |x| < 120: x - n*pi/2 with n = round(x * 2/pi) (the published fallback for
   targets without a round-to-integer instruction: truncate x*2^24*2/pi, add
   half, shift) */
GM_FN double gm_reduce_fast(double x, int *np) {
    const double hpi_inv = 0x1.45f306dc9c883p+23; /* 2/pi * 2^24 */
    const double hpi = 0x1.921fb54442d18p+0;      /* pi/2 */
    const double r = GM_MUL(x, hpi_inv);
    const int n = (GM_D2I_RZ(r) + 0x800000) >> 24;
    *np = n;
    return GM_FMA(-GM_I2D(n), hpi, x);
}

/* |x| >= 120: the mantissa times 2/pi in 64-bit fixed point (quadrants in the
   top two bits), exact, then the remainder times pi/2 */
GM_FN double gm_reduce_large(uint32_t xi, int *np) {
    const double pi63 = 0x1.921fb54442d18p-62; /* pi * 2^-63 */
    const uint32_t *arr = &gm_inv_pio4[(xi >> 26) & 15];
    const int shift = (xi >> 23) & 7;
    xi = (xi & 0xffffff) | 0x800000;
    xi <<= shift;
    uint64_t res0 = (uint64_t)(uint32_t)(xi * arr[0]);
    const uint64_t res1 = (uint64_t)xi * arr[4];
    const uint64_t res2 = (uint64_t)xi * arr[8];
    res0 = (res2 >> 32) | (res0 << 32);
    res0 += res1;
    const uint64_t n = (res0 + (1ull << 61)) >> 62;
    res0 -= n << 62;
    *np = (int)n;
    return GM_MUL(GM_LL2D((int64_t)res0), pi63);
}

/* is_cos = 0: sinf, 1: cosf */
GM_FN float gm_sincosf_one(float y, int is_cos) {
    const uint32_t uy = gm_asu32(y);
    const uint32_t abstop = (uy >> 20) & 0x7ff;
    double x = GM_F2D(y);
    int n;
    if (abstop < 0x3f4) { /* |y| < pi/4 (top 12 bits of 0x1.921fb6p-1f) */
        if (abstop < 0x398) return is_cos ? 1.0f : y; /* |y| < 2^-12 */
        return gm_sincos_poly(x, GM_MUL(x, x), 0, is_cos);
    }
    if (abstop < 0x42f) { /* |y| < 120 */
        x = gm_reduce_fast(x, &n);
        const double s = ((n + 1) & 2) ? -1.0 : 1.0; /* signs 1, -1, -1, 1 by n & 3 */
        return gm_sincos_poly(GM_MUL(x, s), GM_MUL(x, x), (n & 2) != 0, n ^ is_cos);
    }
    if (abstop < 0x7f8) {
        const int sign = (int)(uy >> 31);
        x = gm_reduce_large(uy, &n);
        const int q = n + sign;
        const double s = ((q + 1) & 2) ? -1.0 : 1.0;
        return gm_sincos_poly(GM_MUL(x, s), GM_MUL(x, x), (q & 2) != 0, n ^ is_cos);
    }
    return (y - y) / (y - y); /* Inf or NaN: NaN */
}

GM_FN float gm_sinf(float x) { return gm_sincosf_one(x, 0); }
GM_FN float gm_cosf(float x) { return gm_sincosf_one(x, 1); }

#endif
