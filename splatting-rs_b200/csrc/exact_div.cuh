// Correctly rounded single-precision division without the IEEE division instruction
// sequence: through a double-precision reciprocal, rounded once. Used where a quotient must
// equal the CPU oracle's (IEEE float32 division) bit for bit: Adam's update and the
// projection's geometry and gradients.
#pragma once

#include "common.cuh"

namespace splat {

// x / b rounded to float, for a float b in [2^-126, 1] given as r = RN64(1 / b): the float
// rounding of the double product x r. It equals the IEEE single-precision quotient for every
// float x (zeros, subnormals, infinities and NaN included), at one double multiply and two
// conversions instead of a single-precision division.
// Proof. Write x = A 2^a and b = B 2^c with integers A < 2^24 and B in [2^23, 2^24). If B is a
// power of two, x r is the exact quotient Q = x / b. Otherwise, for Q in the binade
// [2^e, 2^(e+1)), the float rounding boundaries are M = (2k + 1) 2^(e-24), and
// (Q - M) B 2^(24-e) = A 2^(a-c-e+24) - B (2k + 1) is a nonzero integer (a zero would make B a
// power of two), so |Q - M| >= 2^(e-24) / B > 2^-49 Q. Subnormal quotients lie on the grid
// (2k + 1) 2^-150, at least 2^-150 / B > 2^-174 from it, while Q < 2^-126. The double product
// carries two roundings (r and x r): |x r - Q| < 2^-51 Q, with neither overflow nor underflow
// in double for float x and b. So x r lies strictly between the same two rounding boundaries
// as Q, and rounding it to float gives RN32(Q), the IEEE quotient. tests/test_oracle_math.py
// checks the identity against numpy's IEEE float32 division: every significand of x for a
// sample of the bias corrections, and random x over every exponent for the bias corrections
// of the first 20,000 steps.
__device__ __forceinline__ float div_by_bias(float x, double reciprocal) {
    return __double2float_rn((double)x * reciprocal);
}

// u / d rounded to float for a positive float divisor d whose reciprocal is a normal float
// (d in [2^-126, 2^126]) or d = +inf (the seed rcp(+inf) = +0 and the residual's d held at the
// largest float keep y = 0: u y is then the IEEE u / inf, +-0 or NaN): the reciprocal by
// Newton-Raphson (Markstein's y <- y + y (1 - d y), each step one fused multiply-add for the
// residual and one for the update) in double precision from the hardware's approximate
// single-precision reciprocal, then u y in double rounded once to float. It equals the IEEE
// single-precision quotient for every float u. Proof: the seed's relative error is below
// 2^-20, so the steps leave at most 2^-40 and then 2^-80 plus the roundings, under
// 2^-53 (1 + 2^-26) in all; with the product's rounding, u y is within 2^-51 u / d of the
// exact quotient, which (as for div_by_bias) lies more than 2^-49 of itself from every float
// rounding boundary, so both round to the same float. tests/test_gpu_parity.py checks it
// against IEEE float32 division (sp_debug_adam_quotients).
__device__ __forceinline__ float div_exact(float u, float d) {
    float seed;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(seed) : "f"(d));
    const double dd = (double)fminf(d, 3.40282347e38f);  // the largest float
    double y = (double)seed;
    y = fma(y, fma(-dd, y, 1.0), y);
    y = fma(y, fma(-dd, y, 1.0), y);
    return __double2float_rn((double)u * y);
}

// The compiler's IEEE division, kept out of line so that div_rn's common path does not
// carry its instruction sequence.
static __device__ __noinline__ float div_ieee(float u, float d) { return u / d; }

// u / d, the IEEE single-precision quotient, for every pair of floats: div_exact (on -u and
// -d when d is negative; negation is exact and round-to-nearest is symmetric) where its proof
// holds, |d| in [2^-126, 2^126], the IEEE division elsewhere (zero, subnormal, huge, infinite
// or NaN divisors).
__device__ __forceinline__ float div_rn(float u, float d) {
    const float ad = fabsf(d);
    if (ad >= 1.17549435e-38f && ad <= 8.50705917e37f)  // 2^-126, 2^126
        return div_exact(d < 0.0f ? -u : u, ad);
    return div_ieee(u, d);
}

}  // namespace splat
