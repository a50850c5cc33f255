// Adam over the packed parameters with the scale clamp fused in (K11): adam.wgsl:20-37
// then clamp_scales.wgsl:15-29, in one pass over HBM. Each block takes 128 Gaussians:
// parameters, gradients and moments stream through as float4, the updated parameters are
// held in shared memory until the block has clamped every Gaussian's log scales, then
// written back. Compiled with -fmad=false, so the update is bit-identical to the oracle's.
#include "kernels.h"

namespace splat {
namespace {

constexpr int kGaussiansPerBlock = 128;

struct AdamArgs {
    float lr[SP_PARAM_STRIDE(3)];
    float bias1, bias2, max_log_scale, max_log_anisotropy;
};

template <int S>
__global__ void __launch_bounds__(kBlock) k_adam(float* __restrict__ params, const float* __restrict__ gradients,
                                                 float* __restrict__ m1, float* __restrict__ m2, uint64_t first,
                                                 uint64_t end, const AdamArgs args) {
    __shared__ float s_p[kGaussiansPerBlock * S];
    __shared__ float s_lr[S];
    const uint32_t t = threadIdx.x;
    if (t < (uint32_t)S) s_lr[t] = args.lr[t];
    __syncthreads();
    const uint64_t g0 = first + (uint64_t)blockIdx.x * kGaussiansPerBlock;
    const uint32_t here = (uint32_t)min((uint64_t)kGaussiansPerBlock, end - g0);
    const uint64_t f0 = g0 * S;
    const uint32_t floats = here * S;
    auto update = [&](float p, float g, float& m, float& v, uint32_t slot) -> float {
        const float mm = SP_ADAM_BETA1 * m + (1.0f - SP_ADAM_BETA1) * g;
        const float vv = SP_ADAM_BETA2 * v + (1.0f - SP_ADAM_BETA2) * g * g;
        m = mm;
        v = vv;
        const float m_hat = mm / args.bias1;
        const float v_hat = vv / args.bias2;
        return p - s_lr[slot] * m_hat / (__fsqrt_rn(v_hat) + SP_ADAM_EPSILON);
    };
    const bool aligned = ((f0 & 3u) == 0) && ((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(gradients) |
                                               reinterpret_cast<uintptr_t>(m1) | reinterpret_cast<uintptr_t>(m2)) &
                                              15u) == 0;
    uint32_t done = 0;
    if (aligned) {
        const uint32_t vec = floats / 4;
        float4* p4 = reinterpret_cast<float4*>(params + f0);
        const float4* g4 = reinterpret_cast<const float4*>(gradients + f0);
        float4* m14 = reinterpret_cast<float4*>(m1 + f0);
        float4* m24 = reinterpret_cast<float4*>(m2 + f0);
        for (uint32_t i = t; i < vec; i += kBlock) {
            float4 p = p4[i];
            const float4 g = __ldg(g4 + i);
            float4 a = m14[i], b = m24[i];
            const uint32_t s0 = (i * 4) % S;
            const uint32_t s1 = (s0 + 1 == (uint32_t)S) ? 0 : s0 + 1;
            const uint32_t s2 = (s1 + 1 == (uint32_t)S) ? 0 : s1 + 1;
            const uint32_t s3 = (s2 + 1 == (uint32_t)S) ? 0 : s2 + 1;
            p.x = update(p.x, g.x, a.x, b.x, s0);
            p.y = update(p.y, g.y, a.y, b.y, s1);
            p.z = update(p.z, g.z, a.z, b.z, s2);
            p.w = update(p.w, g.w, a.w, b.w, s3);
            m14[i] = a;
            m24[i] = b;
            reinterpret_cast<float4*>(s_p)[i] = p;
        }
        done = vec * 4;
    }
    for (uint32_t i = done + t; i < floats; i += kBlock) {
        float m = m1[f0 + i], v = m2[f0 + i];
        s_p[i] = update(params[f0 + i], gradients[f0 + i], m, v, i % S);
        m1[f0 + i] = m;
        m2[f0 + i] = v;
    }
    __syncthreads();
    if (t < here) {
        // std::min semantics ((b < a) ? b : a), as the oracle.
        auto lesser = [](float a, float b) { return (b < a) ? b : a; };
        float* ls = s_p + t * S + SP_SLOT_LOG_SCALE;
        float a = ls[0], b = ls[1], c = ls[2];
        a = lesser(a, args.max_log_scale);
        b = lesser(b, args.max_log_scale);
        c = lesser(c, args.max_log_scale);
        const float smallest = lesser(a, lesser(b, c));
        ls[0] = lesser(a, smallest + args.max_log_anisotropy);
        ls[1] = lesser(b, smallest + args.max_log_anisotropy);
        ls[2] = lesser(c, smallest + args.max_log_anisotropy);
    }
    __syncthreads();
    if (aligned) {
        const uint32_t vec = floats / 4;
        float4* p4 = reinterpret_cast<float4*>(params + f0);
        for (uint32_t i = t; i < vec; i += kBlock) p4[i] = reinterpret_cast<const float4*>(s_p)[i];
    }
    for (uint32_t i = done + t; i < floats; i += kBlock) params[f0 + i] = s_p[i];
}

}  // namespace

cudaError_t launch_adam(float* params, const float* gradients, float* first_moment, float* second_moment,
                        uint64_t first, uint64_t count, int stride, const float* lr_by_slot_host, float bias1,
                        float bias2, float max_log_scale, float max_log_anisotropy, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    AdamArgs args{};
    for (int k = 0; k < stride; ++k) args.lr[k] = lr_by_slot_host[k];
    args.bias1 = bias1;
    args.bias2 = bias2;
    args.max_log_scale = max_log_scale;
    args.max_log_anisotropy = max_log_anisotropy;
    const unsigned grid = grid_for(count, kGaussiansPerBlock);
    const uint64_t end = first + count;
    switch (stride) {
        case SP_PARAM_STRIDE(0):
            k_adam<SP_PARAM_STRIDE(0)><<<grid, kBlock, 0, stream>>>(params, gradients, first_moment, second_moment,
                                                                    first, end, args);
            break;
        case SP_PARAM_STRIDE(1):
            k_adam<SP_PARAM_STRIDE(1)><<<grid, kBlock, 0, stream>>>(params, gradients, first_moment, second_moment,
                                                                    first, end, args);
            break;
        case SP_PARAM_STRIDE(2):
            k_adam<SP_PARAM_STRIDE(2)><<<grid, kBlock, 0, stream>>>(params, gradients, first_moment, second_moment,
                                                                    first, end, args);
            break;
        case SP_PARAM_STRIDE(3):
            k_adam<SP_PARAM_STRIDE(3)><<<grid, kBlock, 0, stream>>>(params, gradients, first_moment, second_moment,
                                                                    first, end, args);
            break;
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace splat
