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

// The peer-memory exchange step: the gradients of the block's Gaussians summed over the
// ranks in rank order (peer loads, float4 when aligned), Adam + clamp in shared memory as
// k_adam (adam_block writes this rank's parameters), then the updated parameters stored into
// every other rank's buffer (peer stores) and fenced at system scope.
template <int S>
__global__ void __launch_bounds__(kBlock) k_adam_peer(const PeerBuffers peers, float* __restrict__ m1,
                                                      float* __restrict__ m2, uint64_t first, uint64_t end,
                                                      const AdamStep step) {
    __shared__ float4 s_p4[kGaussiansPerBlock * S / 4 + 1];
    __shared__ float s_lr[S];
    float* s_p = reinterpret_cast<float*>(s_p4);
    const uint32_t t = threadIdx.x;
    if (t < (uint32_t)S) s_lr[t] = step.lr[t];
    const uint64_t g0 = first + (uint64_t)blockIdx.x * kGaussiansPerBlock;
    const uint32_t here = (uint32_t)min((uint64_t)kGaussiansPerBlock, end - g0);
    const uint64_t f0 = g0 * S;
    const uint32_t floats = here * S;
    bool aligned = (f0 & 3u) == 0;
    for (uint32_t r = 0; r < peers.world; ++r)
        aligned = aligned && ((reinterpret_cast<uintptr_t>(peers.gradients[r]) |
                               reinterpret_cast<uintptr_t>(peers.params[r])) & 15u) == 0;
    const uint32_t vec = aligned ? floats / 4 : 0;
    // kU peer loads in flight per thread and rank (measured: 247 -> 214 us at 2 GPUs).
    constexpr uint32_t kU = 4;
    for (uint32_t i0 = t; i0 < vec; i0 += kBlock * kU) {
        float4 sum[kU];
#pragma unroll
        for (uint32_t u = 0; u < kU; ++u) {
            const uint32_t i = i0 + u * kBlock;
            if (i < vec) sum[u] = reinterpret_cast<const float4*>(peers.gradients[0] + f0)[i];
        }
        for (uint32_t r = 1; r < peers.world; ++r) {
            float4 g[kU];
#pragma unroll
            for (uint32_t u = 0; u < kU; ++u) {
                const uint32_t i = i0 + u * kBlock;
                if (i < vec) g[u] = reinterpret_cast<const float4*>(peers.gradients[r] + f0)[i];
            }
#pragma unroll
            for (uint32_t u = 0; u < kU; ++u) {
                sum[u].x = sum[u].x + g[u].x;
                sum[u].y = sum[u].y + g[u].y;
                sum[u].z = sum[u].z + g[u].z;
                sum[u].w = sum[u].w + g[u].w;
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < kU; ++u) {
            const uint32_t i = i0 + u * kBlock;
            if (i < vec) s_p4[i] = sum[u];
        }
    }
    for (uint32_t i = vec * 4 + t; i < floats; i += kBlock) {
        float sum = peers.gradients[0][f0 + i];
        for (uint32_t r = 1; r < peers.world; ++r) sum = sum + peers.gradients[r][f0 + i];
        s_p[i] = sum;
    }
    __syncthreads();
    float* own = peers.params[peers.rank];
    adam_block<S>(own, m1, m2, g0, here, s_p, s_lr, step);
    // adam_block leaves the updated, clamped parameters in s_p.
    for (uint32_t r = 0; r < peers.world; ++r) {
        if (r == peers.rank) continue;
        float* dst = peers.params[r] + f0;
        for (uint32_t i = t; i < vec; i += kBlock) reinterpret_cast<float4*>(dst)[i] = s_p4[i];
        for (uint32_t i = vec * 4 + t; i < floats; i += kBlock) dst[i] = s_p[i];
    }
    __threadfence_system();
}

// Test support: the Adam step's two exact divisions on given operands, out[2i] = x / y by
// div_by_bias (y a bias correction in (0, 1]) and out[2i + 1] = x / y by div_exact.
__global__ void k_adam_quotients(const float* __restrict__ x, const float* __restrict__ y, uint64_t n,
                                 float* __restrict__ out) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float a = x[i], b = y[i];
    const bool exact_domain = (b >= 1.17549435e-38f && b <= 8.50705917e37f) || b == INFINITY;
    out[3 * i + 0] = b > 0.0f && b <= 1.0f ? div_by_bias(a, 1.0 / (double)b) : 0.0f;
    out[3 * i + 1] = exact_domain ? div_exact(a, b) : 0.0f;
    out[3 * i + 2] = div_rn(a, b);
}

}  // namespace

cudaError_t launch_adam_peer(const PeerBuffers& peers, float* first_moment, float* second_moment, uint64_t first,
                             uint64_t count, int stride, const float* lr_by_slot_host, float bias1, float bias2,
                             float max_log_scale, float max_log_anisotropy, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    if (peers.world == 0 || peers.world > (uint32_t)kMaxPeers || peers.rank >= peers.world) return cudaErrorInvalidValue;
    AdamStep args{};
    for (int k = 0; k < stride; ++k) args.lr[k] = lr_by_slot_host[k];
    args.set_bias(bias1, bias2);
    args.max_log_scale = max_log_scale;
    args.max_log_anisotropy = max_log_anisotropy;
    const unsigned grid = grid_for(count, kGaussiansPerBlock);
    const uint64_t end = first + count;
#define SP_ADAM_PEER(D)                                                                                         \
    k_adam_peer<SP_PARAM_STRIDE(D)><<<grid, kBlock, 0, stream>>>(peers, first_moment, second_moment, first, end, \
                                                                 args)
    switch (stride) {
        case SP_PARAM_STRIDE(0): SP_ADAM_PEER(0); break;
        case SP_PARAM_STRIDE(1): SP_ADAM_PEER(1); break;
        case SP_PARAM_STRIDE(2): SP_ADAM_PEER(2); break;
        case SP_PARAM_STRIDE(3): SP_ADAM_PEER(3); break;
        default: return cudaErrorInvalidValue;
    }
#undef SP_ADAM_PEER
    return cudaGetLastError();
}

namespace {

// Reads `count` float4 of a (peer's) buffer, four loads in flight per thread as the exchange
// kernel issues them, and stores one sum per block into `sink` so that no load is dropped:
// the read bandwidth of the link as the exchange uses it.
__global__ void __launch_bounds__(kBlock) k_peer_read(const float4* __restrict__ src, uint64_t count,
                                                      float4* __restrict__ sink) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const uint64_t threads = (uint64_t)gridDim.x * kBlock;
    uint64_t i = (uint64_t)blockIdx.x * kBlock + threadIdx.x;
    for (; i + 3 * threads < count; i += 4 * threads) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __ldcg(src + i + k * threads);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc.x += v[k].x;
            acc.y += v[k].y;
            acc.z += v[k].z;
            acc.w += v[k].w;
        }
    }
    for (; i < count; i += threads) {
        const float4 v = __ldcg(src + i);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    __shared__ float4 s[kBlock];
    s[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float4 total = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < kBlock; ++k) {
            total.x += s[k].x;
            total.y += s[k].y;
            total.z += s[k].z;
            total.w += s[k].w;
        }
        sink[blockIdx.x] = total;
    }
}

}  // namespace

cudaError_t launch_peer_read(const float4* src, uint64_t count, float4* sink, unsigned blocks, cudaStream_t stream) {
    k_peer_read<<<blocks, kBlock, 0, stream>>>(src, count, sink);
    return cudaGetLastError();
}

cudaError_t launch_adam(float* params, const float* gradients, float* first_moment, float* second_moment,
                        uint64_t first, uint64_t count, int stride, const float* lr_by_slot_host, float bias1,
                        float bias2, float max_log_scale, float max_log_anisotropy, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    AdamStep args{};
    for (int k = 0; k < stride; ++k) args.lr[k] = lr_by_slot_host[k];
    args.set_bias(bias1, bias2);
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

extern "C" sp_status sp_debug_adam_quotients(const float* d_x, const float* d_y, uint64_t count, float* d_quotients,
                                             void* stream) {
    using namespace splat;
    if (count == 0) return SP_OK;
    if (!d_x || !d_y || !d_quotients || (reinterpret_cast<uintptr_t>(d_quotients) & 7u) != 0) return SP_ERR_INVALID;
    const unsigned blocks = (unsigned)((count + 255) / 256);
    k_adam_quotients<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_x, d_y, count, d_quotients);
    return cudaGetLastError() == cudaSuccess ? SP_OK : SP_ERR_CUDA;
}
