// The training loss (K7): masked SSIM with its partial derivatives (ssim_forward.wgsl:34-91)
// and the loss gradient per pixel (loss.wgsl:35-97), weights of loss.rs:32-36.
//
// The reference sums the 121 taps of the 11 x 11 window directly per pixel. Here each block
// computes a 16 x 16 tile of outputs from a 26 x 26 halo staged in shared memory, and the
// window is applied separably (11 taps along x, then 11 along y), which is the same sum
// reordered: results match within float rounding, not bit for bit.
#include "kernels.h"

namespace splat {
namespace {

constexpr int kOut = 16;
constexpr int kR = SP_SSIM_RADIUS;
constexpr int kHalo = kOut + 2 * kR;
constexpr int kTaps = 2 * kR + 1;

struct Taps {
    float w[kTaps];
};

__device__ __forceinline__ float sign_of(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

__global__ void __launch_bounds__(kOut* kOut) k_ssim(const float4* __restrict__ image, const float4* __restrict__ gt,
                                                     uint32_t width, uint32_t height, const Taps taps,
                                                     float4* __restrict__ partials) {
    __shared__ float s_x[kHalo][kHalo][3];
    __shared__ float s_y[kHalo][kHalo][3];
    __shared__ float s_h[kHalo][kOut][15];
    const int t = threadIdx.x;
    const int ox = blockIdx.x * kOut, oy = blockIdx.y * kOut;
    for (int i = t; i < kHalo * kHalo; i += kOut * kOut) {
        const int ly = i / kHalo, lx = i % kHalo;
        const int qx = ox + lx - kR, qy = oy + ly - kR;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f), y = x;
        if (qx >= 0 && qy >= 0 && qx < (int)width && qy < (int)height) {
            const size_t q = (size_t)qy * width + qx;
            x = image[q];
            y = gt[q];
        }
        s_x[ly][lx][0] = x.x;
        s_x[ly][lx][1] = x.y;
        s_x[ly][lx][2] = x.z;
        s_y[ly][lx][0] = y.x;
        s_y[ly][lx][1] = y.y;
        s_y[ly][lx][2] = y.z;
    }
    __syncthreads();
    // Along x: per channel mu_x, mu_y, E[x^2], E[y^2], E[xy].
    for (int i = t; i < kHalo * kOut; i += kOut * kOut) {
        const int row = i / kOut, col = i % kOut;
        float s[15];
#pragma unroll
        for (int k = 0; k < 15; ++k) s[k] = 0.0f;
#pragma unroll
        for (int d = 0; d < kTaps; ++d) {
            const float w = taps.w[d];
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float x = s_x[row][col + d][c], y = s_y[row][col + d][c];
                s[c * 5 + 0] += w * x;
                s[c * 5 + 1] += w * y;
                s[c * 5 + 2] += w * x * x;
                s[c * 5 + 3] += w * y * y;
                s[c * 5 + 4] += w * x * y;
            }
        }
#pragma unroll
        for (int k = 0; k < 15; ++k) s_h[row][col][k] = s[k];
    }
    __syncthreads();
    const int lx = t % kOut, ly = t / kOut;
    const int px = ox + lx, py = oy + ly;
    if (px >= (int)width || py >= (int)height) return;
    float m[15];
#pragma unroll
    for (int k = 0; k < 15; ++k) m[k] = 0.0f;
#pragma unroll
    for (int d = 0; d < kTaps; ++d) {
        const float w = taps.w[d];
#pragma unroll
        for (int k = 0; k < 15; ++k) m[k] += w * s_h[ly + d][lx][k];
    }
    const size_t i = (size_t)py * width + px;
    const float mask = gt[i].w;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float mu_x = m[c * 5 + 0], mu_y = m[c * 5 + 1];
        const float sigma_xx = m[c * 5 + 2] - mu_x * mu_x;
        const float sigma_yy = m[c * 5 + 3] - mu_y * mu_y;
        const float sigma_xy = m[c * 5 + 4] - mu_x * mu_y;
        const float a = mu_x * mu_x + mu_y * mu_y + SP_SSIM_C1;
        const float b = sigma_xx + sigma_yy + SP_SSIM_C2;
        const float cc = 2.0f * mu_x * mu_y + SP_SSIM_C1;
        const float d = 2.0f * sigma_xy + SP_SSIM_C2;
        const float ab = a * b;
        const float ssim = cc * d / ab;
        const float d_mu = mask * (2.0f * mu_y * (d - cc) / ab - 2.0f * mu_x * cc * d * (b - a) / (ab * ab));
        const float d_exx = mask * (-cc * d / (ab * b));
        const float d_exy = mask * (2.0f * cc / ab);
        partials[i * 3 + c] = make_float4(ssim, d_mu, d_exx, d_exy);
    }
}

__global__ void __launch_bounds__(kOut* kOut) k_loss(const float4* __restrict__ image, const float4* __restrict__ gt,
                                                     const float4* __restrict__ partials, uint32_t width,
                                                     uint32_t height, const Taps taps, const sp_loss_weights weights,
                                                     float4* __restrict__ loss_gradient,
                                                     float4* __restrict__ pixel_loss) {
    __shared__ float s_p[kHalo][kHalo][9];
    __shared__ float s_h[kHalo][kOut][9];
    const int t = threadIdx.x;
    const int ox = blockIdx.x * kOut, oy = blockIdx.y * kOut;
    for (int i = t; i < kHalo * kHalo; i += kOut * kOut) {
        const int ly = i / kHalo, lx = i % kHalo;
        const int qx = ox + lx - kR, qy = oy + ly - kR;
        const bool in = qx >= 0 && qy >= 0 && qx < (int)width && qy < (int)height;
        const size_t q = in ? (size_t)qy * width + qx : 0;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float4 p = in ? partials[q * 3 + c] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            s_p[ly][lx][c * 3 + 0] = p.y;
            s_p[ly][lx][c * 3 + 1] = p.z;
            s_p[ly][lx][c * 3 + 2] = p.w;
        }
    }
    __syncthreads();
    for (int i = t; i < kHalo * kOut; i += kOut * kOut) {
        const int row = i / kOut, col = i % kOut;
        float s[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) s[k] = 0.0f;
#pragma unroll
        for (int d = 0; d < kTaps; ++d) {
            const float w = taps.w[d];
#pragma unroll
            for (int k = 0; k < 9; ++k) s[k] += w * s_p[row][col + d][k];
        }
#pragma unroll
        for (int k = 0; k < 9; ++k) s_h[row][col][k] = s[k];
    }
    __syncthreads();
    const int lx = t % kOut, ly = t / kOut;
    const int px = ox + lx, py = oy + ly;
    if (px >= (int)width || py >= (int)height) return;
    float m[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) m[k] = 0.0f;
#pragma unroll
    for (int d = 0; d < kTaps; ++d) {
        const float w = taps.w[d];
#pragma unroll
        for (int k = 0; k < 9; ++k) m[k] += w * s_h[ly + d][lx][k];
    }
    const size_t i = (size_t)py * width + px;
    const float pixels = (float)((size_t)width * height);
    const float4 x = image[i], y = gt[i];
    const float mask = y.w;
    const float xs[3] = {x.x, x.y, x.z}, ys[3] = {y.x, y.y, y.z};
    float dssim = 0.0f, d_rgb[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        dssim += mask * (1.0f - partials[i * 3 + c].x);
        const float d_ssim = m[c * 3 + 0] + 2.0f * xs[c] * m[c * 3 + 1] + ys[c] * m[c * 3 + 2];
        d_rgb[c] = (weights.l1 * mask * sign_of(xs[c] - ys[c]) - weights.dssim * d_ssim) / (3.0f * pixels);
    }
    const float coverage = 1.0f - x.w;
    const float alpha_difference = coverage - mask;
    loss_gradient[i] = make_float4(d_rgb[0], d_rgb[1], d_rgb[2], -weights.alpha * sign_of(alpha_difference) / pixels);
    const float l1 = mask * (fabsf(xs[0] - ys[0]) + fabsf(xs[1] - ys[1]) + fabsf(xs[2] - ys[2])) / 3.0f;
    const float alpha_error = fabsf(alpha_difference);
    pixel_loss[i] = make_float4(l1, alpha_error, dssim / 3.0f,
                                weights.l1 * l1 + weights.alpha * alpha_error + weights.dssim * dssim / 3.0f);
}

Taps window() {
    // common.wgsl:110-122, with the same exp as the oracle.
    Taps taps;
    float sum = 0.0f;
    for (int k = 0; k < kTaps; ++k) {
        const float d = (float)(k - kR);
        taps.w[k] = sp_expf(-d * d / (2.0f * SP_SSIM_SIGMA * SP_SSIM_SIGMA));
        sum += taps.w[k];
    }
    for (int k = 0; k < kTaps; ++k) taps.w[k] /= sum;
    return taps;
}

}  // namespace

cudaError_t launch_ssim(const float4* image, const float4* ground_truth, uint32_t width, uint32_t height,
                        float4* partials, cudaStream_t stream) {
    const dim3 grid(grid_for(width, kOut), grid_for(height, kOut));
    k_ssim<<<grid, kOut * kOut, 0, stream>>>(image, ground_truth, width, height, window(), partials);
    return cudaGetLastError();
}

cudaError_t launch_loss(const float4* image, const float4* ground_truth, const float4* partials, uint32_t width,
                        uint32_t height, const sp_loss_weights& weights, float4* loss_gradient, float4* pixel_loss,
                        cudaStream_t stream) {
    const dim3 grid(grid_for(width, kOut), grid_for(height, kOut));
    k_loss<<<grid, kOut * kOut, 0, stream>>>(image, ground_truth, partials, width, height, window(), weights,
                                             loss_gradient, pixel_loss);
    return cudaGetLastError();
}

}  // namespace splat

namespace splat {
namespace {

constexpr int kSumBlocks = 256;

// Sums of the 4 per-pixel loss terms in double, in a fixed order (each block a strided
// share, a tree per block, then the last block adds the block sums in block order), so
// that the reported loss does not depend on scheduling.
__global__ void __launch_bounds__(kBlock) k_loss_sums(const float4* __restrict__ pixel_loss, uint64_t pixels,
                                                      double* __restrict__ workspace) {
    __shared__ double s[4][kBlock];
    __shared__ bool last;
    double* result = workspace;
    double* partials = workspace + 4;
    unsigned int* done = reinterpret_cast<unsigned int*>(workspace + 4 + 4 * kSumBlocks);
    const uint32_t t = threadIdx.x;
    double a = 0.0, b = 0.0, c = 0.0, d = 0.0;
    for (uint64_t i = (uint64_t)blockIdx.x * kBlock + t; i < pixels; i += (uint64_t)gridDim.x * kBlock) {
        const float4 v = pixel_loss[i];
        a += v.x;
        b += v.y;
        c += v.z;
        d += v.w;
    }
    s[0][t] = a;
    s[1][t] = b;
    s[2][t] = c;
    s[3][t] = d;
    __syncthreads();
    for (int half = kBlock / 2; half > 0; half >>= 1) {
        if (t < (uint32_t)half)
            for (int k = 0; k < 4; ++k) s[k][t] += s[k][t + half];
        __syncthreads();
    }
    if (t < 4) partials[blockIdx.x * 4 + t] = s[t][0];
    __threadfence();
    __syncthreads();
    if (t == 0) last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (t < 4) {
        double sum = 0.0;
        for (uint32_t k = 0; k < gridDim.x; ++k) sum += __ldcg(partials + k * 4 + t);
        result[t] = sum;
    }
    if (t == 0) *done = 0;
}

}  // namespace

cudaError_t launch_loss_sums(const float4* pixel_loss, uint64_t pixels, double* workspace, cudaStream_t stream) {
    k_loss_sums<<<kSumBlocks, kBlock, 0, stream>>>(pixel_loss, pixels, workspace);
    return cudaGetLastError();
}

}  // namespace splat
