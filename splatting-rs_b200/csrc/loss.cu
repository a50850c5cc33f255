// The training loss (K7): masked SSIM with its partial derivatives (ssim_forward.wgsl:34-91)
// and the loss gradient per pixel (loss.wgsl:35-97), weights of loss.rs:32-36.
//
// The reference sums the 121 taps of the 11 x 11 window directly per pixel. Here the window
// is applied separably (11 taps along x, then 11 along y; the same sum reordered, so results
// match within float rounding, not bit for bit). Each block computes a 32 x 32 tile of
// outputs from its 42 x 42 halo in shared memory, one colour channel at a time; the passes
// are register-blocked: a thread convolves 8 consecutive outputs of a row from 18 loaded
// inputs, then 4 consecutive outputs of a column from 14 loaded row sums.
#include "kernels.h"

namespace splat {
namespace {

constexpr int kR = SP_SSIM_RADIUS;
constexpr int kTaps = 2 * kR + 1;
constexpr int kTile = 32;                 // outputs per block edge
constexpr int kSpan = kTile + 2 * kR;     // 42: halo rows / columns
constexpr int kPitch = kTile + 4;         // row pitch of the row-sum planes (bank spread)
constexpr int kThreads = 256;
constexpr int kRowOut = 8;                // outputs per thread along x
constexpr int kColOut = 4;                // outputs per thread along y
constexpr int kRowItems = kSpan * (kTile / kRowOut);  // 168 row segments per plane set
constexpr int kHaloLoads = (kSpan * kSpan + kThreads - 1) / kThreads;  // 7 halo pixels per thread
static_assert(kTile / kColOut * kTile == kThreads, "one column segment per thread");

struct Taps {
    float w[kTaps];
};

__device__ __forceinline__ float sign_of(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

// Row pass: thread item (row, segment) of the halo convolves kRowOut outputs of each of the
// P planes along x; load(j, p) is input column seg * kRowOut + j of plane p.
template <int P, typename Load>
__device__ __forceinline__ void row_pass(const Taps& taps, int row, int seg, Load load, float* rows) {
    float acc[P][kRowOut];
#pragma unroll
    for (int p = 0; p < P; ++p)
#pragma unroll
        for (int o = 0; o < kRowOut; ++o) acc[p][o] = 0.0f;
#pragma unroll
    for (int j = 0; j < kRowOut + 2 * kR; ++j) {
        float v[P];
        load(j, v);
#pragma unroll
        for (int o = 0; o < kRowOut; ++o) {
            const int d = j - o;
            if (d >= 0 && d < kTaps)
#pragma unroll
                for (int p = 0; p < P; ++p) acc[p][o] = fmaf(taps.w[d], v[p], acc[p][o]);
        }
    }
#pragma unroll
    for (int p = 0; p < P; ++p) {
        float4* out = reinterpret_cast<float4*>(rows + (p * kSpan + row) * kPitch + seg * kRowOut);
        out[0] = make_float4(acc[p][0], acc[p][1], acc[p][2], acc[p][3]);
        out[1] = make_float4(acc[p][4], acc[p][5], acc[p][6], acc[p][7]);
    }
}

// Column pass: output rows y0 .. y0 + kColOut - 1 of column col, all P planes.
template <int P>
__device__ __forceinline__ void column_pass(const Taps& taps, const float* rows, int col, int y0,
                                            float acc[P][kColOut]) {
#pragma unroll
    for (int p = 0; p < P; ++p)
#pragma unroll
        for (int o = 0; o < kColOut; ++o) acc[p][o] = 0.0f;
#pragma unroll
    for (int j = 0; j < kColOut + 2 * kR; ++j) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
            const float v = rows[(p * kSpan + y0 + j) * kPitch + col];
#pragma unroll
            for (int o = 0; o < kColOut; ++o) {
                const int d = j - o;
                if (d >= 0 && d < kTaps) acc[p][o] = fmaf(taps.w[d], v, acc[p][o]);
            }
        }
    }
}

constexpr size_t kSsimSmem = (size_t)3 * kSpan * kSpan * sizeof(float2) + (size_t)5 * kSpan * kPitch * sizeof(float);
constexpr size_t kLossSmem = (size_t)3 * kSpan * kSpan * sizeof(float) + (size_t)3 * kSpan * kPitch * sizeof(float);

// ssim_forward.wgsl:34-91: per pixel and channel the SSIM and its partials with respect to
// mu_x, E[x^2] and E[xy] (masked), into planar partials[channel][pixel].
__global__ void __launch_bounds__(kThreads, 2) k_ssim(const float4* __restrict__ image, const float4* __restrict__ gt,
                                                      uint32_t width, uint32_t height, const Taps taps,
                                                      float4* __restrict__ partials) {
    chain_enter();
    extern __shared__ float4 smem4[];
    float2* s_in = reinterpret_cast<float2*>(smem4);         // [3][kSpan][kSpan]: (x, y) per channel
    float* s_rows = reinterpret_cast<float*>(s_in + 3 * kSpan * kSpan);  // [5][kSpan][kPitch]
    const int t = threadIdx.x;
    const int ox = blockIdx.x * kTile, oy = blockIdx.y * kTile;
    // The halo, all loads in flight before the first store.
    {
        float4 x[kHaloLoads], y[kHaloLoads];
#pragma unroll
        for (int k = 0; k < kHaloLoads; ++k) {
            const int i = t + k * kThreads;
            const int qx = ox + i % kSpan - kR, qy = oy + i / kSpan - kR;
            x[k] = y[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < kSpan * kSpan && qx >= 0 && qy >= 0 && qx < (int)width && qy < (int)height) {
                const size_t q = (size_t)qy * width + qx;
                x[k] = image[q];
                y[k] = gt[q];
            }
        }
#pragma unroll
        for (int k = 0; k < kHaloLoads; ++k) {
            const int i = t + k * kThreads;
            if (i < kSpan * kSpan) {
                s_in[i] = make_float2(x[k].x, y[k].x);
                s_in[kSpan * kSpan + i] = make_float2(x[k].y, y[k].y);
                s_in[2 * kSpan * kSpan + i] = make_float2(x[k].z, y[k].z);
            }
        }
    }
    const int col = t % kTile, y0 = (t / kTile) * kColOut;
    const int px = ox + col;
    const size_t pixels = (size_t)width * height;
    float mask[kColOut];
#pragma unroll
    for (int o = 0; o < kColOut; ++o) {
        const int py = oy + y0 + o;
        mask[o] = px < (int)width && py < (int)height ? gt[(size_t)py * width + px].w : 0.0f;
    }
    for (int c = 0; c < 3; ++c) {
        __syncthreads();
        if (t < kRowItems) {
            const int row = t / (kTile / kRowOut), seg = t % (kTile / kRowOut);
            const float2* in = s_in + (c * kSpan + row) * kSpan + seg * kRowOut;
            // The five moments of the window: mu_x, mu_y, E[x^2], E[y^2], E[xy].
            row_pass<5>(taps, row, seg, [&](int j, float v[5]) {
                const float2 xy = in[j];
                v[0] = xy.x;
                v[1] = xy.y;
                v[2] = xy.x * xy.x;
                v[3] = xy.y * xy.y;
                v[4] = xy.x * xy.y;
            }, s_rows);
        }
        __syncthreads();
        float m[5][kColOut];
        column_pass<5>(taps, s_rows, col, y0, m);
#pragma unroll
        for (int o = 0; o < kColOut; ++o) {
            const int py = oy + y0 + o;
            if (px >= (int)width || py >= (int)height) continue;
            const size_t i = (size_t)py * width + px;
            const float mu_x = m[0][o], mu_y = m[1][o];
            const float sigma_xx = m[2][o] - mu_x * mu_x;
            const float sigma_yy = m[3][o] - mu_y * mu_y;
            const float sigma_xy = m[4][o] - mu_x * mu_y;
            const float a = mu_x * mu_x + mu_y * mu_y + SP_SSIM_C1;
            const float b = sigma_xx + sigma_yy + SP_SSIM_C2;
            const float cc = 2.0f * mu_x * mu_y + SP_SSIM_C1;
            const float d = 2.0f * sigma_xy + SP_SSIM_C2;
            // a, b >= the positive constants C1, C2: the reciprocals are finite.
            const float inv_ab = __fdividef(1.0f, a * b);
            const float ssim = cc * d * inv_ab;
            const float d_mu =
                mask[o] * (2.0f * mu_y * (d - cc) * inv_ab - 2.0f * mu_x * ssim * (b - a) * inv_ab);
            const float d_exx = mask[o] * -ssim * __fdividef(1.0f, b);
            const float d_exy = mask[o] * (2.0f * cc * inv_ab);
            partials[c * pixels + i] = make_float4(ssim, d_mu, d_exx, d_exy);
        }
    }
}

// loss.wgsl:35-97: the window applied to the SSIM partials (the chain rule through the
// moments), then the per-pixel loss gradient and loss terms. Three blocks per SM (at most 85
// registers, 39 KB of shared memory each): measured 47.5 -> 44.3 us against two at config 2.
__global__ void __launch_bounds__(kThreads, 3) k_loss(const float4* __restrict__ image, const float4* __restrict__ gt,
                                                      const float4* __restrict__ partials, uint32_t width,
                                                      uint32_t height, const Taps taps,
                                                      const sp_loss_weights weights,
                                                      float4* __restrict__ loss_gradient,
                                                      float4* __restrict__ pixel_loss, float4* __restrict__ clear,
                                                      uint64_t clear_count) {
    // The atomic backward's per-Gaussian blend sums are zeroed here, a slice per block, for the
    // backward that follows this loss (instead of a memset that would break the launch chain;
    // here rather than in k_ssim, which is issue-bound, while these blocks mostly wait on their
    // loads). No grid of the chain before this one touches them: before the wait.
    if (clear) {
        const uint64_t blocks = (uint64_t)gridDim.x * gridDim.y, block = (uint64_t)blockIdx.y * gridDim.x + blockIdx.x;
        const uint64_t per = (clear_count + blocks - 1) / blocks;
        const uint64_t end = min(clear_count, (block + 1) * per);
        for (uint64_t i = block * per + threadIdx.x; i < end; i += kThreads) clear[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    chain_enter();
    extern __shared__ float4 smem4[];
    float* s_in = reinterpret_cast<float*>(smem4);           // [3][kSpan][kSpan]: d_mu, d_exx, d_exy
    float* s_rows = s_in + 3 * kSpan * kSpan;                // [3][kSpan][kPitch]
    const int t = threadIdx.x;
    const int ox = blockIdx.x * kTile, oy = blockIdx.y * kTile;
    const int col = t % kTile, y0 = (t / kTile) * kColOut;
    const int px = ox + col;
    const size_t pixels = (size_t)width * height;
    float d_ssim[3][kColOut], ssim_sum[kColOut];
#pragma unroll
    for (int o = 0; o < kColOut; ++o) ssim_sum[o] = 0.0f;
    // The halo of one channel's partials, loaded into registers (all loads in flight) and
    // stored to shared memory later: the next channel's loads overlap this channel's
    // column pass.
    float4 p[kHaloLoads];
    auto fetch = [&](int c) {
        const float4* plane = partials + c * pixels;
#pragma unroll
        for (int k = 0; k < kHaloLoads; ++k) {
            const int i = t + k * kThreads;
            const int qx = ox + i % kSpan - kR, qy = oy + i / kSpan - kR;
            p[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < kSpan * kSpan && qx >= 0 && qy >= 0 && qx < (int)width && qy < (int)height)
                p[k] = plane[(size_t)qy * width + qx];
        }
    };
    auto stage = [&]() {
#pragma unroll
        for (int k = 0; k < kHaloLoads; ++k) {
            const int i = t + k * kThreads;
            if (i < kSpan * kSpan) {
                s_in[i] = p[k].y;
                s_in[kSpan * kSpan + i] = p[k].z;
                s_in[2 * kSpan * kSpan + i] = p[k].w;
            }
        }
    };
    fetch(0);
    stage();
    for (int c = 0; c < 3; ++c) {
        const float4* plane = partials + c * pixels;
        __syncthreads();
        if (t < kRowItems) {
            const int row = t / (kTile / kRowOut), seg = t % (kTile / kRowOut);
            const float* in = s_in + row * kSpan + seg * kRowOut;
            row_pass<3>(taps, row, seg, [&](int j, float v[3]) {
                v[0] = in[j];
                v[1] = in[kSpan * kSpan + j];
                v[2] = in[2 * kSpan * kSpan + j];
            }, s_rows);
        }
        __syncthreads();
        if (c < 2) fetch(c + 1);
        float x[kColOut], y[kColOut], ssim[kColOut];
#pragma unroll
        for (int o = 0; o < kColOut; ++o) {
            const int py = oy + y0 + o;
            x[o] = y[o] = 0.0f;
            ssim[o] = 1.0f;
            if (px < (int)width && py < (int)height) {
                const size_t i = (size_t)py * width + px;
                x[o] = reinterpret_cast<const float*>(image + i)[c];
                y[o] = reinterpret_cast<const float*>(gt + i)[c];
                ssim[o] = plane[i].x;
            }
        }
        float m[3][kColOut];
        column_pass<3>(taps, s_rows, col, y0, m);
#pragma unroll
        for (int o = 0; o < kColOut; ++o) {
            d_ssim[c][o] = m[0][o] + 2.0f * x[o] * m[1][o] + y[o] * m[2][o];
            ssim_sum[o] += 1.0f - ssim[o];
        }
        if (c < 2) stage();  // s_in is free: every row pass of this channel is behind the barrier
    }
#pragma unroll
    for (int o = 0; o < kColOut; ++o) {
        const int py = oy + y0 + o;
        if (px >= (int)width || py >= (int)height) continue;
        const size_t i = (size_t)py * width + px;
        const float fpixels = (float)pixels;
        const float4 x = image[i], y = gt[i];
        const float mask = y.w;
        const float xs[3] = {x.x, x.y, x.z}, ys[3] = {y.x, y.y, y.z};
        float d_rgb[3];
#pragma unroll
        for (int c = 0; c < 3; ++c)
            d_rgb[c] = (weights.l1 * mask * sign_of(xs[c] - ys[c]) - weights.dssim * d_ssim[c][o]) / (3.0f * fpixels);
        const float dssim = mask * ssim_sum[o];
        const float coverage = 1.0f - x.w;
        const float alpha_difference = coverage - mask;
        loss_gradient[i] =
            make_float4(d_rgb[0], d_rgb[1], d_rgb[2], -weights.alpha * sign_of(alpha_difference) / fpixels);
        const float l1 = mask * (fabsf(xs[0] - ys[0]) + fabsf(xs[1] - ys[1]) + fabsf(xs[2] - ys[2])) / 3.0f;
        const float alpha_error = fabsf(alpha_difference);
        pixel_loss[i] = make_float4(l1, alpha_error, dssim / 3.0f,
                                    weights.l1 * l1 + weights.alpha * alpha_error + weights.dssim * dssim / 3.0f);
    }
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
    static std::atomic<unsigned long long> configured{0};
    const cudaError_t err = allow_smem_once(k_ssim, kSsimSmem, configured);
    if (err != cudaSuccess) return err;
    const dim3 grid(grid_for(width, kTile), grid_for(height, kTile));
    launch_chained(k_ssim, grid, kThreads, kSsimSmem, stream, image, ground_truth, width, height, window(), partials);
    return cudaGetLastError();
}

cudaError_t launch_loss(const float4* image, const float4* ground_truth, const float4* partials, uint32_t width,
                        uint32_t height, const sp_loss_weights& weights, float4* loss_gradient, float4* pixel_loss,
                        float4* clear, uint64_t clear_count, cudaStream_t stream) {
    static std::atomic<unsigned long long> configured{0};
    const cudaError_t err = allow_smem_once(k_loss, kLossSmem, configured);
    if (err != cudaSuccess) return err;
    const dim3 grid(grid_for(width, kTile), grid_for(height, kTile));
    launch_chained(k_loss, grid, kThreads, kLossSmem, stream, image, ground_truth, partials, width, height, window(), weights,
                                                  loss_gradient, pixel_loss, clear, clear_count);
    return cudaGetLastError();
}

}  // namespace splat

namespace splat {
namespace {

constexpr int kSumBlocks = 256;

// Sums of the 4 per-pixel loss terms in double, in a fixed order (each block a strided
// share, a tree per block, then the last block adds the block sums in block order), so
// that the reported loss does not depend on scheduling.
// The last block also copies the step's status word and overflow flag (from `meta`, when
// given) next to the sums, so that a step's read-back is one block of words; with
// `mirror_dst` (page-locked host memory mapped for the device) it then copies those
// `mirror_words` words from `mirror_src` there itself, so that no copy follows the kernel.
__global__ void __launch_bounds__(kBlock) k_loss_sums(const float4* __restrict__ pixel_loss, uint64_t pixels,
                                                      double* __restrict__ workspace, double* __restrict__ result,
                                                      const DeviceMeta* meta, uint32_t* status_dst,
                                                      const uint32_t* mirror_src, uint32_t* mirror_dst,
                                                      uint32_t mirror_words) {
    chain_enter();
    __shared__ double s[4][kBlock];
    __shared__ bool last;
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
    if (t == 0) {
        *done = 0;
        if (meta) {
            status_dst[0] = meta->status;
            status_dst[1] = meta->overflow;
        }
    }
    if (mirror_dst) {
        __syncthreads();  // the sums and the status words above are written
        for (uint32_t i = t; i < mirror_words; i += kBlock) mirror_dst[i] = __ldcg(mirror_src + i);
    }
}

}  // namespace

cudaError_t launch_loss_sums(const float4* pixel_loss, uint64_t pixels, double* workspace, double* result,
                             const DeviceMeta* meta, uint32_t* status_dst, cudaStream_t stream,
                             const uint32_t* mirror_src, uint32_t* mirror_dst, uint32_t mirror_words) {
    launch_chained(k_loss_sums, kSumBlocks, kBlock, 0, stream, pixel_loss, pixels, workspace, result, meta, status_dst,
                   mirror_src, mirror_dst, mirror_words);
    return cudaGetLastError();
}

}  // namespace splat
