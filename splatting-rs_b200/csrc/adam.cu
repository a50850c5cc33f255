// Adam over the packed parameters with the scale clamp fused in (K11): adam.wgsl:20-37
// then clamp_scales.wgsl:15-29, in one pass over HBM. Each block takes 128 Gaussians:
// their gradients are staged in shared memory, parameters and moments stream through as
// float4, and the updated parameters are held in shared memory until the block has clamped
// every Gaussian's log scales, then written back (adam_block). Compiled with -fmad=false,
// so the update is bit-identical to the oracle's.
#include "adam_math.cuh"
#include "kernels.h"

namespace splat {
namespace {

constexpr int kGaussiansPerBlock = 128;

template <int S>
__global__ void __launch_bounds__(kBlock) k_adam(float* __restrict__ params, const float* __restrict__ gradients,
                                                 float* __restrict__ m1, float* __restrict__ m2, uint64_t first,
                                                 uint64_t end, const AdamStep step) {
    __shared__ float4 s_p4[kGaussiansPerBlock * S / 4 + 1];
    __shared__ float s_lr[S];
    float* s_p = reinterpret_cast<float*>(s_p4);
    const uint32_t t = threadIdx.x;
    if (t < (uint32_t)S) s_lr[t] = step.lr[t];
    const uint64_t g0 = first + (uint64_t)blockIdx.x * kGaussiansPerBlock;
    const uint32_t here = (uint32_t)min((uint64_t)kGaussiansPerBlock, end - g0);
    const uint64_t f0 = g0 * S;
    const uint32_t floats = here * S;
    // The gradients into shared memory, then the update in place.
    if (((f0 & 3u) == 0) && (reinterpret_cast<uintptr_t>(gradients) & 15u) == 0) {
        const uint32_t vec = floats / 4;
        const float4* g4 = reinterpret_cast<const float4*>(gradients + f0);
        for (uint32_t i = t; i < vec; i += kBlock) s_p4[i] = __ldg(g4 + i);
        for (uint32_t i = vec * 4 + t; i < floats; i += kBlock) s_p[i] = __ldg(gradients + f0 + i);
    } else {
        for (uint32_t i = t; i < floats; i += kBlock) s_p[i] = __ldg(gradients + f0 + i);
    }
    __syncthreads();
    adam_block<S>(params, m1, m2, g0, here, s_p, s_lr, step);
}

}  // namespace

cudaError_t launch_adam(float* params, const float* gradients, float* first_moment, float* second_moment,
                        uint64_t first, uint64_t count, int stride, const float* lr_by_slot_host, float bias1,
                        float bias2, float max_log_scale, float max_log_anisotropy, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    AdamStep args{};
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
