// The Adam update and the scale clamp (adam.wgsl:20-37, clamp_scales.wgsl:15-29) as device
// functions, shared by the Adam kernel and the projection backward's fused Adam epilogue.
// Both translation units are compiled with -fmad=false, so either path gives the oracle's
// parameters and moments bit for bit.
#pragma once

#include "common.cuh"
#include "exact_div.cuh"

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
