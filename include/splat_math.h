/* Scalar math shared bit-for-bit by the CUDA kernels and the CPU oracle.
 *
 * The projection decides which tiles a Gaussian touches (its radius and tile rectangle),
 * and those integers must come out identical on the GPU and in the oracle for the tile
 * lists to match bit for bit. Every operation on that path is a correctly rounded IEEE
 * operation (+, -, *, /, sqrt, fma, floor, ceil, rint) except exp, whose last-bit
 * behaviour differs between math libraries. sp_expf is therefore one exp written here
 * once, from a published method, and compiled into both sides:
 *
 *   Cody & Waite argument reduction (W. J. Cody, W. Waite, "Software Manual for the
 *   Elementary Functions", 1980): x = n ln2 + r with n = rint(x / ln2), ln2 split into a
 *   short high part (exact products n * hi for |n| < 2^8) and a low correction; then
 *   e^r, |r| <= ln2 / 2, by its Taylor series to degree 7 in Horner form (truncation
 *   error below 6e-9 relative), then scaling by 2^n through the exponent field.
 *
 * It is within 1 ulp of the correctly rounded exp over its whole range (the correctly
 * rounded result in more than 90 % of arguments), within 1 ulp of glibc's expf and within
 * 2 ulp of CUDA's expf: tests/test_oracle_math.py measures all three.
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

/* 1 / (1 + e^-x) (common.wgsl:87-89). */
SP_HD float sp_sigmoid(float x) { return 1.0f / (1.0f + sp_expf(-x)); }

#endif
