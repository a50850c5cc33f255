// The Adam update and the scale clamp (adam.wgsl:20-37, clamp_scales.wgsl:15-29) as device
// functions, shared by the Adam kernel and the projection backward's fused Adam epilogue.
// Both translation units are compiled with -fmad=false, so either path gives the oracle's
// parameters and moments bit for bit.
#pragma once

#include "common.cuh"

namespace splat {

// One Adam step's constants: the learning rate of every parameter slot (optimizer.rs:248-256
// folds the position-rate factor in), the bias corrections 1 - beta^t and the clamp bounds.
// inv_bias1 / inv_bias2 are the bias corrections' reciprocals in double precision, rounded
// once (set_bias): the moments are divided by the corrections through them (adam_update).
struct AdamStep {
    float lr[SP_PARAM_STRIDE(3)];
    float bias1, bias2, max_log_scale, max_log_anisotropy;
    double inv_bias1, inv_bias2;

    __host__ void set_bias(float b1, float b2) {
        bias1 = b1;
        bias2 = b2;
        inv_bias1 = 1.0 / (double)b1;
        inv_bias2 = 1.0 / (double)b2;
    }
};

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

// adam.wgsl:26-35 for one parameter: updates the moments, returns the parameter.
__device__ __forceinline__ float adam_update(float p, float g, float& m, float& v, float lr, const AdamStep& step) {
    const float mm = SP_ADAM_BETA1 * m + (1.0f - SP_ADAM_BETA1) * g;
    const float vv = SP_ADAM_BETA2 * v + (1.0f - SP_ADAM_BETA2) * g * g;
    m = mm;
    v = vv;
    const float m_hat = div_by_bias(mm, step.inv_bias1);  // mm / bias1, IEEE
    const float v_hat = div_by_bias(vv, step.inv_bias2);  // vv / bias2, IEEE
    return p - div_exact(lr * m_hat, __fsqrt_rn(v_hat) + SP_ADAM_EPSILON);  // IEEE quotient
}

// clamp_scales.wgsl:15-29 on one Gaussian's three log scales, with std::min semantics
// ((b < a) ? b : a), as the oracle.
__device__ __forceinline__ void clamp_log_scales(float* ls, float max_log_scale, float max_log_anisotropy) {
    auto lesser = [](float a, float b) { return (b < a) ? b : a; };
    float a = ls[0], b = ls[1], c = ls[2];
    a = lesser(a, max_log_scale);
    b = lesser(b, max_log_scale);
    c = lesser(c, max_log_scale);
    const float smallest = lesser(a, lesser(b, c));
    ls[0] = lesser(a, smallest + max_log_anisotropy);
    ls[1] = lesser(b, smallest + max_log_anisotropy);
    ls[2] = lesser(c, smallest + max_log_anisotropy);
}

// Adam plus the clamp over one block's `here` Gaussians of stride S starting at Gaussian
// g0. `staged` (shared memory, here * S floats) holds their gradients on entry and their
// updated, clamped parameters on return; the parameters are then written back. `lr` is the
// step's rate per slot in shared memory. Every thread of the block must call it.
template <int S>
__device__ __forceinline__ void adam_block(float* __restrict__ params, float* __restrict__ m1,
                                           float* __restrict__ m2, uint64_t g0, uint32_t here, float* staged,
                                           const float* lr, const AdamStep& step) {
    const uint32_t t = threadIdx.x, threads = blockDim.x;
    const uint64_t f0 = g0 * S;
    const uint32_t floats = here * S;
    const bool aligned =
        ((f0 & 3u) == 0) &&
        ((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(m1) | reinterpret_cast<uintptr_t>(m2)) &
         15u) == 0;
    uint32_t done = 0;
    if (aligned) {
        const uint32_t vec = floats / 4;
        float4* p4 = reinterpret_cast<float4*>(params + f0);
        float4* m14 = reinterpret_cast<float4*>(m1 + f0);
        float4* m24 = reinterpret_cast<float4*>(m2 + f0);
        float4* s4 = reinterpret_cast<float4*>(staged);
        for (uint32_t i = t; i < vec; i += threads) {
            float4 p = p4[i];
            const float4 g = s4[i];
            float4 a = m14[i], b = m24[i];
            const uint32_t s0 = (i * 4) % S;
            const uint32_t s1 = (s0 + 1 == (uint32_t)S) ? 0 : s0 + 1;
            const uint32_t s2 = (s1 + 1 == (uint32_t)S) ? 0 : s1 + 1;
            const uint32_t s3 = (s2 + 1 == (uint32_t)S) ? 0 : s2 + 1;
            p.x = adam_update(p.x, g.x, a.x, b.x, lr[s0], step);
            p.y = adam_update(p.y, g.y, a.y, b.y, lr[s1], step);
            p.z = adam_update(p.z, g.z, a.z, b.z, lr[s2], step);
            p.w = adam_update(p.w, g.w, a.w, b.w, lr[s3], step);
            m14[i] = a;
            m24[i] = b;
            s4[i] = p;
        }
        done = vec * 4;
    }
    for (uint32_t i = done + t; i < floats; i += threads) {
        float m = m1[f0 + i], v = m2[f0 + i];
        staged[i] = adam_update(params[f0 + i], staged[i], m, v, lr[i % S], step);
        m1[f0 + i] = m;
        m2[f0 + i] = v;
    }
    __syncthreads();
    if (t < here) clamp_log_scales(staged + t * S + SP_SLOT_LOG_SCALE, step.max_log_scale, step.max_log_anisotropy);
    __syncthreads();
    if (aligned) {
        const uint32_t vec = floats / 4;
        float4* p4 = reinterpret_cast<float4*>(params + f0);
        for (uint32_t i = t; i < vec; i += threads) p4[i] = reinterpret_cast<const float4*>(staged)[i];
    }
    for (uint32_t i = done + t; i < floats; i += threads) params[f0 + i] = staged[i];
}

}  // namespace splat
