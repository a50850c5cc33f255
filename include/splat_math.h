/* Scalar math shared bit-for-bit by the CUDA kernels and the CPU oracle.
 *
 * The projection decides which tiles a Gaussian touches (its radius and tile rectangle),
 * and those integers must come out identical on the GPU and in the oracle for the tile
 * lists to match bit for bit. Every operation on that path is a correctly rounded IEEE
 * operation (+, -, *, /, sqrt, fma, floor, ceil, rint) except exp, whose last-bit
 * behaviour differs between math libraries. The exps here are written once, from a
 * published method, and compiled into both sides:
 *
 *   Cody & Waite argument reduction (W. J. Cody, W. Waite, "Software Manual for the
 *   Elementary Functions", 1980): x = n ln2 + r with n = rint(x / ln2), ln2 split into a
 *   short high part (n * hi exact) and a low correction; e^r, |r| <= ln2 / 2, by its Taylor
 *   series in Horner form; scaling by 2^n through the exponent field.
 *
 * sp_expf works in single precision (Taylor degree 7, truncation error below 6e-9 relative):
 * within 1 ulp of the correctly rounded exp, a dozen float operations; it gives the scales,
 * the opacity sigmoid and the SSIM window. sp_expf_exact works in double precision (44-bit
 * high part of ln 2, Taylor degree 12, truncation error below 2e-16) and rounds once to
 * float: the correctly rounded exp on every float in [-105, 88.72] (checked exhaustively
 * against the long-double exp), and therefore monotone non-decreasing. It gives the blend's
 * alpha in the oracle, and the per-Gaussian thresholds on the falloff's power with which the
 * CUDA blend kernels make the same take (alpha >= 1/255) and clamp (alpha >= 0.99) decisions
 * as the oracle whatever exp they use for alpha's value. tests/test_oracle_math.py measures
 * both against the correctly rounded exp, glibc's expf and CUDA's expf.
 */
#ifndef SPLAT_MATH_H
#define SPLAT_MATH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define SP_HD __host__ __device__ __forceinline__
#else
#define SP_HD static inline
#endif

SP_HD float sp_bits_to_float(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

SP_HD uint32_t sp_float_to_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}

SP_HD float sp_fma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return fmaf(a, b, c);
#endif
}

SP_HD float sp_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}

/* 2^k for -126 <= k <= 127. */
SP_HD float sp_pow2i(int k) { return sp_bits_to_float((uint32_t)(k + 127) << 23); }

SP_HD float sp_expf(float x) {
    if (!(x == x)) return x;
    /* Above ln(FLT_MAX) the result overflows; below -104 it is under half the smallest
     * subnormal. */
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    /* 1 / ln 2 */
    const float n = rintf(sp_mul(x, 1.44269502162933349609375f));
    /* ln 2 = LN2_HI + LN2_LO; LN2_HI = 45426 / 65536 has 16 significant bits. */
    float r = sp_fma(-n, 0.693145751953125f, x);
    r = sp_fma(-n, 1.428606820309417e-06f, r);
    /* 1/k! for k = 7..2, rounded to float. */
    float p = 1.98412701138295233249664306640625e-04f;
    p = sp_fma(p, r, 1.388888922519981861114501953125e-03f);
    p = sp_fma(p, r, 8.33333376795053482055664062500e-03f);
    p = sp_fma(p, r, 4.16666679084300994873046875000e-02f);
    p = sp_fma(p, r, 1.66666671633720397949218750000e-01f);
    p = sp_fma(p, r, 0.5f);
    p = sp_fma(p, r, 1.0f);
    p = sp_fma(p, r, 1.0f);
    int k = (int)n;
    if (k > 127) return sp_mul(sp_mul(p, sp_pow2i(k - 1)), 2.0f);
    if (k < -126) return sp_mul(sp_mul(p, sp_pow2i(k + 100)), sp_pow2i(-100));
    return sp_mul(p, sp_pow2i(k));
}

SP_HD double sp_dfma(double a, double b, double c) {
#if defined(__CUDA_ARCH__)
    return __fma_rn(a, b, c);
#else
    return fma(a, b, c);
#endif
}

SP_HD double sp_dmul(double a, double b) {
#if defined(__CUDA_ARCH__)
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}

SP_HD float sp_double_to_float(double d) {
#if defined(__CUDA_ARCH__)
    return __double2float_rn(d);
#else
    return (float)d;
#endif
}

/* 2^k as a double for -1022 <= k <= 1023. */
SP_HD double sp_pow2d(int k) {
    const uint64_t bits = (uint64_t)(k + 1023) << 52;
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)bits);
#else
    double d;
    memcpy(&d, &bits, 8);
    return d;
#endif
}

SP_HD float sp_expf_exact(float x) {
    if (!(x == x)) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const double xd = (double)x;
    /* 1 / ln 2 */
    const double n = rint(sp_dmul(xd, 0x1.71547652b82fep+0));
    /* ln 2 = LN2_HI + LN2_LO; LN2_HI has 44 significant bits. */
    double r = sp_dfma(-n, 0x1.62e42fefa3a00p-1, xd);
    r = sp_dfma(-n, -0x1.0ca86c3898d00p-49, r);
    /* 1/k! for k = 12..2, rounded to double. */
    double p = 0x1.1eed8eff8d898p-29;
    p = sp_dfma(p, r, 0x1.ae64567f544e4p-26);
    p = sp_dfma(p, r, 0x1.27e4fb7789f5cp-22);
    p = sp_dfma(p, r, 0x1.71de3a556c734p-19);
    p = sp_dfma(p, r, 0x1.a01a01a01a01ap-16);
    p = sp_dfma(p, r, 0x1.a01a01a01a01ap-13);
    p = sp_dfma(p, r, 0x1.6c16c16c16c17p-10);
    p = sp_dfma(p, r, 0x1.1111111111111p-7);
    p = sp_dfma(p, r, 0x1.5555555555555p-5);
    p = sp_dfma(p, r, 0x1.5555555555555p-3);
    p = sp_dfma(p, r, 0.5);
    p = sp_dfma(p, r, 1.0);
    p = sp_dfma(p, r, 1.0);
    /* n lies in [-150, 128]: 2^n is a normal double, and the one rounding to float below
     * also rounds subnormal results correctly. */
    return sp_double_to_float(sp_dmul(p, sp_pow2d((int)n)));
}

/* 1 / (1 + e^-x) (common.wgsl:87-89). */
SP_HD float sp_sigmoid(float x) { return 1.0f / (1.0f + sp_expf(-x)); }

#endif
