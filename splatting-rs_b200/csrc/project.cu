// Projection forward (K1) with the first level of the tile-count scan (K2), the scan of
// the block totals, and the projection backward (K9) with the camera-gradient reduction
// (K10) fused in. This file is compiled with -fmad=false: the projection's depth, radius
// and tile rectangle must match the CPU oracle bit for bit (tile lists are compared
// exactly), and the backward shares the same forward recomputation. The backward's
// divisions go through div_rn (csrc/exact_div.cuh), the same IEEE quotients in fewer
// instructions, so its gradients are the oracle's bit for bit too.
#include <cuda/atomic>

#include "adam_math.cuh"
#include "kernels.h"
#include "tile_cull.cuh"
#include "project_math.cuh"

namespace splat {
namespace {

// Copies `count` floats from global to shared memory, float4 at a time when the source
// is 16-byte aligned. Every thread of the block takes part.
__device__ __forceinline__ void stage_in(const float* __restrict__ src, uint32_t count, float* dst) {
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const uint32_t vec = count / 4;
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (uint32_t i = threadIdx.x; i < vec; i += blockDim.x) d4[i] = __ldg(s4 + i);
        for (uint32_t i = vec * 4 + threadIdx.x; i < count; i += blockDim.x) dst[i] = __ldg(src + i);
    } else {
        for (uint32_t i = threadIdx.x; i < count; i += blockDim.x) dst[i] = __ldg(src + i);
    }
}

// Exclusive block-wide prefix sum of one value per thread (256 threads); also returns
// the block total.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t value, uint32_t* total) {
    __shared__ uint32_t warp_totals[kBlock / 32];
    const uint32_t lane = lane_id(), warp = threadIdx.x / 32;
    uint32_t inclusive = value;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t up = __shfl_up_sync(0xffffffffu, inclusive, o);
        if (lane >= (uint32_t)o) inclusive += up;
    }
    if (lane == 31) warp_totals[warp] = inclusive;
    __syncthreads();
    uint32_t before = 0, sum = 0;
#pragma unroll
    for (int w = 0; w < kBlock / 32; ++w) {
        const uint32_t t = warp_totals[w];
        if ((uint32_t)w < warp) before += t;
        sum += t;
    }
    *total = sum;
    return before + inclusive - value;
}

// The smallest float power p <= 0 at which opacity * sp_expf_exact(p) >= level in float
// arithmetic (+inf when not even at p = 0). sp_expf_exact is monotone (include/splat_math.h),
// so the blend's per-pixel test "opacity * exp(power) >= level", as the oracle evaluates it,
// holds exactly when power >= this threshold, whatever exp the blend kernels use for alpha.
// Searched over the float order of -p in [0, 104]: from a guess by the hardware log (a few
// floats from the answer, so that two to four evaluations decide it), a walk of a few floats,
// then, if the guess was further off, bisection over a bracket of 16 floats either side or,
// failing that, the whole range.
__device__ __noinline__ float alpha_threshold(float opacity, float level) {
    if (!(opacity >= level)) return INFINITY;
    auto holds = [&](uint32_t u) { return __fmul_rn(opacity, sp_expf_exact(-__uint_as_float(u))) >= level; };
    const uint32_t last = __float_as_uint(104.0f);  // sp_expf_exact(-104) is 0: never holds there
    const float guess = -__logf(__fdividef(level, opacity));
    const uint32_t g = guess > 0.0f ? min(__float_as_uint(guess), last) : 0u;
    // The answer is -float(u) for the largest u with holds(u) (holds(0) is true, holds(last) false).
    if (holds(g)) {
        for (uint32_t u = g, k = 0; k < 4 && u < last; ++k, ++u)
            if (!holds(u + 1u)) return -__uint_as_float(u);
    } else {
        for (uint32_t u = g, k = 0; k < 4 && u > 0u; ++k) {
            --u;
            if (holds(u)) return -__uint_as_float(u);
        }
    }
    // holds(lo) and !holds(hi).
    uint32_t lo = g > 16u ? g - 16u : 0u, hi = min(g + 16u, last);
    if (!holds(lo) || holds(hi)) {
        lo = 0u;
        hi = last;
    }
    while (hi - lo > 1u) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        if (holds(mid)) lo = mid;
        else hi = mid;
    }
    return -__uint_as_float(lo);
}

// The blend's decision thresholds of a Gaussian of opacity `opacity` (record word [3]).
__device__ __forceinline__ float4 alpha_thresholds(float opacity) {
    return make_float4(alpha_threshold(opacity, SP_MIN_ALPHA), alpha_threshold(opacity, SP_MAX_ALPHA), 0.0f, 0.0f);
}

template <int DEG>
__device__ __forceinline__ void project_one(const float* p, const sp_camera_uniform& cam, float4 rec[kRecord],
                                            uint32_t* radius_out, uint32_t* count_out) {
    rec[0] = rec[1] = rec[2] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    rec[3] = make_float4(INFINITY, INFINITY, 0.0f, 0.0f);
    *radius_out = 0;
    *count_out = 0;
    const float (*rows)[4] = cam.world_to_camera_rows;
    const float pz = row_dot(rows[2], p[0], p[1], p[2]);
    if (pz < SP_NEAR_Z) return;
    Geometry g;
    geometry(p, cam, g);
    if (g.det <= 0.0f) return;
    const float conic0 = g.c / g.det, conic1 = -g.b / g.det, conic2 = g.a / g.det;
    const float mid = 0.5f * (g.a + g.c);
    const float largest = mid + __fsqrt_rn(max_of(0.1f, mid * mid - g.det));
    const float radius = ceilf(3.0f * __fsqrt_rn(largest));
    const float mean0 = cam.focal[0] * g.pc[0] / g.pc[2] + cam.principal_point[0];
    const float mean1 = cam.focal[1] * g.pc[1] / g.pc[2] + cam.principal_point[1];
    const float tiles0 = (float)cam.tiles_x, tiles1 = (float)cam.tiles_y;
    const float tmin0 = min_of(max_of(floorf((mean0 - radius) / (float)SP_TILE), 0.0f), tiles0);
    const float tmin1 = min_of(max_of(floorf((mean1 - radius) / (float)SP_TILE), 0.0f), tiles1);
    const float tmax0 = min_of(max_of(floorf((mean0 + radius) / (float)SP_TILE) + 1.0f, 0.0f), tiles0);
    const float tmax1 = min_of(max_of(floorf((mean1 + radius) / (float)SP_TILE) + 1.0f, 0.0f), tiles1);
    const float cnt = (tmax0 - tmin0) * (tmax1 - tmin1);
    if (cnt <= 0.0f) return;
    float col[3];
    raw_color<DEG>(p, p + SP_SLOT_SH, cam, col);
    const float opacity = sp_sigmoid(p[SP_SLOT_OPACITY]);
    const uint32_t rect_lo = (uint32_t)tmin0 | ((uint32_t)tmin1 << 16);
    const uint32_t rect_hi = (uint32_t)tmax0 | ((uint32_t)tmax1 << 16);
    rec[0] = make_float4(mean0, mean1, conic0, conic1);
    rec[1] = make_float4(conic2, opacity, max_of(0.0f, col[0]), max_of(0.0f, col[1]));
    rec[2] = make_float4(max_of(0.0f, col[2]), g.pc[2], __uint_as_float(rect_lo), __uint_as_float(rect_hi));
    rec[3] = alpha_thresholds(opacity);
    *radius_out = (uint32_t)radius;
    *count_out = (uint32_t)cnt;
}

// The camera of the pass. Set by the host (sp_set_camera) it is a kernel argument, whose
// fields the instructions read as constant-bank operands; written on the device (the device
// pose step: DEV) it is copied from device memory into shared memory by the first threads,
// visible after the next barrier.
__device__ __forceinline__ void load_camera(const sp_camera_uniform* __restrict__ camera, sp_camera_uniform& s_cam) {
    constexpr uint32_t kWords = sizeof(sp_camera_uniform) / sizeof(uint32_t);
    if (threadIdx.x < kWords)
        reinterpret_cast<uint32_t*>(&s_cam)[threadIdx.x] = reinterpret_cast<const uint32_t*>(camera)[threadIdx.x];
}

template <bool DEV>
__device__ __forceinline__ const sp_camera_uniform& pick_camera(const sp_camera_uniform& argument,
                                                                const sp_camera_uniform& shared) {
    if constexpr (DEV) return shared;
    else return argument;
}

// The blend kernels' culling constants of a projected Gaussian (record a, b): the half
// extents (ex, ey) of the ellipse d^T C d <= q, q = 2.02 ln(255 opacity) + 0.02, outside of
// which its alpha is below 1/255 (padded by 1 % in the level and 0.05 px), and the slopes
// -b/c, -b/a of the conic's minimum along a vertical and a horizontal line. ex < 0: the
// opacity alone keeps alpha below 1/255; ex = inf: a degenerate conic, never culled.
__device__ __forceinline__ float4 reach_of(float4 a, float4 b) {
    const float level = b.y * 255.0f;
    if (!(level > 1.0f)) return make_float4(-1.0f, -1.0f, 0.0f, 0.0f);
    const float det = a.z * b.x - a.w * a.w;
    if (!(det > 0.0f) || !(a.z > 0.0f) || !(b.x > 0.0f)) return make_float4(INFINITY, INFINITY, 0.0f, 0.0f);
    const float q = 2.02f * __logf(level) + 0.02f;
    return make_float4(sqrtf(q * b.x / det) + 0.05f, sqrtf(q * a.z / det) + 0.05f, -a.w / b.x, -a.w / a.z);
}

template <int DEG, bool DEV>
__global__ void __launch_bounds__(kBlock) k_project(const float* __restrict__ params, uint32_t n,
                                                    const sp_camera_uniform camera_argument,
                                                    const sp_camera_uniform* __restrict__ camera_device,
                                                    float4* __restrict__ records, uint32_t* __restrict__ radii,
                                                    uint32_t* __restrict__ local_offsets,
                                                    uint32_t* __restrict__ block_totals, DeviceMeta* depth_range,
                                                    float4* __restrict__ reach, uint32_t cull) {
    chain_enter();
    constexpr int S = SP_PARAM_STRIDE(DEG);
    extern __shared__ float4 smem4[];
    __shared__ sp_camera_uniform s_cam;
    const sp_camera_uniform& cam = pick_camera<DEV>(camera_argument, s_cam);
    float* sp = reinterpret_cast<float*>(smem4);
    const uint32_t g0 = blockIdx.x * kBlock;
    const uint32_t here = min((uint32_t)kBlock, n - g0);
    // The block's whole parameter slice requested at once: the staging loop's loads then
    // meet it in L2 (measured at config 2: 62 -> 52 us).
    if (threadIdx.x == 0) prefetch_l2(params + (size_t)g0 * S, here * S * (uint32_t)sizeof(float));
    if constexpr (DEV) load_camera(camera_device, s_cam);
    stage_in(params + (size_t)g0 * S, here * S, sp);
    __syncthreads();
    const uint32_t t = threadIdx.x;
    uint32_t count = 0;
    if (t < here) {
        float4 rec[kRecord];
        uint32_t radius;
        project_one<DEG>(sp + t * S, cam, rec, &radius, &count);
        float4* out = records + (size_t)(g0 + t) * kRecord;
#pragma unroll
        for (int k = 0; k < kRecord; ++k) out[k] = rec[k];
        radii[g0 + t] = radius;
        reach[g0 + t] = radius > 0 ? reach_of(rec[0], rec[1]) : make_float4(-1.0f, -1.0f, 0.0f, 0.0f);
        if (cull && count) {
            // Only the rectangle's tiles the ellipse reaches get keys (tile_cull.cuh).
            const uint32_t lo = __float_as_uint(rec[2].z), hi = __float_as_uint(rec[2].w);
            count = culled_tile_count(cull_ellipse(rec[0], rec[1]), lo & 0xffffu, lo >> 16, hi & 0xffffu, hi >> 16);
        }
    }
    uint32_t total;
    const uint32_t exclusive = block_exclusive_scan(count, &total);
    if (t < here) local_offsets[g0 + t] = exclusive;
    if (t == 0) block_totals[blockIdx.x] = total;
    if (depth_range) {
        // The range of the depth keys of the Gaussians that emit keys, for compressed keys.
        __shared__ uint32_t s_lo[kBlock / 32], s_hi[kBlock / 32];
        const bool emits = t < here && count > 0;
        const uint32_t key =
            emits ? __float_as_uint(records[(size_t)(g0 + t) * kRecord + 2].y) >> (32 - SP_DEPTH_BITS) : 0u;
        const uint32_t lo = __reduce_min_sync(0xffffffffu, emits ? key : 0xffffffffu);
        const uint32_t hi = __reduce_max_sync(0xffffffffu, key);
        if ((t & 31u) == 0) {
            s_lo[t / 32] = lo;
            s_hi[t / 32] = hi;
        }
        __syncthreads();
        if (t == 0) {
            uint32_t block_lo = s_lo[0], block_hi = s_hi[0];
#pragma unroll
            for (int w = 1; w < kBlock / 32; ++w) {
                block_lo = min(block_lo, s_lo[w]);
                block_hi = max(block_hi, s_hi[w]);
            }
            if (block_lo <= block_hi) {
                atomicMin(&depth_range->depth_lo, block_lo);
                atomicMax(&depth_range->depth_hi, block_hi);
            }
        }
    }
}

// scan.wgsl:64-81 over the block totals: one block of 1024 threads loops over chunks.
__global__ void __launch_bounds__(1024) k_scan_blocks(const uint32_t* __restrict__ block_totals,
                                                      unsigned long long* __restrict__ block_offsets, uint32_t blocks,
                                                      unsigned long long capacity, DeviceMeta* meta,
                                                      uint32_t* sort_histograms, uint32_t* sort_tickets,
                                                      const SortPlan plan) {
    chain_enter();
    __shared__ unsigned long long warp_sums[32];
    __shared__ unsigned long long carry;
    const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
    if (t == 0) carry = 0;
    for (uint32_t i = t; i < kSortMaxPasses * kSortRadix; i += blockDim.x) sort_histograms[i] = 0;
    if (t < kSortMaxPasses) sort_tickets[t] = 0;
    __syncthreads();
    for (uint32_t base = 0; base < blocks; base += 1024) {
        const uint32_t i = base + t;
        const unsigned long long v = i < blocks ? block_totals[i] : 0ull;
        unsigned long long inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long up = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= (uint32_t)o) inc += up;
        }
        if (lane == 31) warp_sums[warp] = inc;
        __syncthreads();
        unsigned long long before = 0, chunk = 0;
        for (uint32_t w = 0; w < 32; ++w) {
            const unsigned long long s = warp_sums[w];
            if (w < warp) before += s;
            chunk += s;
        }
        if (i < blocks) block_offsets[i] = carry + before + inc - v;
        __syncthreads();
        if (t == 0) carry += chunk;
        __syncthreads();
    }
    if (t == 0) {
        const unsigned long long total = carry;
        const unsigned long long count = total < capacity ? total : capacity;
        meta->count = (uint32_t)count;
        meta->overflow = total > capacity ? 1u : 0u;
        meta->sort_blocks = (uint32_t)((count + 1023) / 1024);
        meta->histogram_length = 16u * meta->sort_blocks;
        meta->capacity = (uint32_t)capacity;
        meta->partitions = (uint32_t)((count + kSortPartition - 1) / kSortPartition);
        meta->total_lo = (uint32_t)total;
        meta->total_hi = (uint32_t)(total >> 32);
        // The key geometry of this frame.
        uint32_t passes = (uint32_t)plan.passes, shift = (uint32_t)plan.tile_shift, base = 0;
        if (plan.compressed) {
            const uint32_t lo = meta->depth_lo, hi = meta->depth_hi;
            base = lo <= hi ? lo : 0u;
            const uint32_t range = lo <= hi ? hi - lo : 0u;  // largest key offset
            shift = range ? 32u - __clz(range) : 0u;
            const uint32_t bits = (uint32_t)plan.tile_bits + shift;
            passes = max(1u, (bits + 7u) / 8u);
            // Reset for the next frame's projection.
            meta->depth_lo = 0xffffffffu;
            meta->depth_hi = 0u;
        }
        meta->key_shift = shift;
        meta->key_base = base;
        meta->passes = passes;
        meta->first_buffer = ((uint32_t)plan.passes ^ passes) & 1u;
    }
}

// project_backward.wgsl:30-194 for one Gaussian: `grads` (stride floats, in shared memory,
// holding the Gaussian's parameters on entry) and the camera gradient.
template <int DEG, int MODE>
__device__ __forceinline__ void project_backward_one(float* p, uint32_t g, const sp_camera_uniform& cam,
                                                     const float4* __restrict__ records, uint32_t radius,
                                                     const uint32_t* __restrict__ offsets,
                                                     const float* __restrict__ slot_gradients, uint64_t capacity,
                                                     const float4* __restrict__ gaussian_gradients,
                                                     float4* __restrict__ densify_stats, float cgrad[14]) {
    constexpr int S = SP_PARAM_STRIDE(DEG);
    // Position, log scale, rotation and opacity logit in registers; the SH coefficients
    // stay in shared memory, each read before its gradient overwrites it.
    float prm[SP_SLOT_SH];
#pragma unroll
    for (int k = 0; k < SP_SLOT_SH; ++k) {
        prm[k] = p[k];
        p[k] = 0.0f;
    }
    float* sh = p + SP_SLOT_SH;
    auto zero_sh = [&]() {
#pragma unroll
        for (int k = SP_SLOT_SH; k < S; ++k) p[k] = 0.0f;
    };
    if (radius == 0) {
        zero_sh();
        return;
    }
    const float4 r0 = records[(size_t)g * kRecord + 0];
    const float4 r1 = records[(size_t)g * kRecord + 1];
    const float4 r2 = records[(size_t)g * kRecord + 2];
    float d_mean[2] = {0.0f, 0.0f}, d_conic[3] = {0.0f, 0.0f, 0.0f}, d_color[3] = {0.0f, 0.0f, 0.0f};
    float d_opacity = 0.0f;
    if (MODE == SP_BWD_DETERMINISTIC) {
        // project_backward.wgsl:38-55: the slots of the Gaussian's tiles, in slot order.
        const uint32_t lo = __float_as_uint(r2.z), hi = __float_as_uint(r2.w);
        const uint32_t count = ((hi & 0xffffu) - (lo & 0xffffu)) * ((hi >> 16) - (lo >> 16));
        for (uint32_t k = 0; k < count; ++k) {
            const uint64_t slot = (uint64_t)offsets[g] + k;
            if (slot >= capacity) break;
            const float* s = slot_gradients + slot * SP_GRAD_STRIDE;
            d_mean[0] += s[0];
            d_mean[1] += s[1];
            d_conic[0] += s[2];
            d_conic[1] += s[3];
            d_conic[2] += s[4];
            d_color[0] += s[5];
            d_color[1] += s[6];
            d_color[2] += s[7];
            d_opacity += s[8];
        }
    } else {
        const float4 a = gaussian_gradients[(size_t)g * 3 + 0];
        const float4 b = gaussian_gradients[(size_t)g * 3 + 1];
        const float4 c = gaussian_gradients[(size_t)g * 3 + 2];
        d_mean[0] = a.x;
        d_mean[1] = a.y;
        d_conic[0] = a.z;
        d_conic[1] = a.w;
        d_conic[2] = b.x;
        d_color[0] = b.y;
        d_color[1] = b.z;
        d_color[2] = b.w;
        d_opacity = c.x;
    }
    // project_backward.wgsl:56-63.
    {
        const float half0 = 0.5f * (float)cam.width, half1 = 0.5f * (float)cam.height;
        const float m0 = d_mean[0] * half0, m1 = d_mean[1] * half1;
        float4 st = densify_stats[g];
        st.x = st.x + __fsqrt_rn(m0 * m0 + m1 * m1);
        st.y = st.y + 1.0f;
        st.z = max_of(st.z, (float)radius);
        st.w = 0.0f;
        densify_stats[g] = st;
    }
    Geometry geo;
    geometry<true>(prm, cam, geo);
    if (geo.det <= 0.0f) {
        zero_sh();
        return;
    }
    const float fx = cam.focal[0], fy = cam.focal[1];
    const float* pc = geo.pc;
    const float z3 = geo.z2 * pc[2];
    // Opacity and colour (project_backward.wgsl:103-110).
    const float opacity = r1.y;
    p[SP_SLOT_OPACITY] = d_opacity * opacity * (1.0f - opacity);
    // The colour's clamp at zero passes the gradient where the raw colour is positive. The
    // forward stored max(0, raw) in the record (words 6-8), positive exactly where raw is
    // (a NaN raw colour is stored as 0 and fails both tests), so the record decides it
    // without evaluating the SH colour again.
    const float color_raw[3] = {r1.z, r1.w, r2.x};
    float d_position_sh[3] = {0.0f, 0.0f, 0.0f};
    if (DEG == 0) {
#pragma unroll
        for (int c = 0; c < 3; ++c) sh[c] = SP_SH_C0 * d_color[c] * (color_raw[c] > 0.0f ? 1.0f : 0.0f);
    } else {
        float d_col[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) d_col[c] = color_raw[c] > 0.0f ? d_color[c] : 0.0f;
        float dir[3], len;
        view_direction<true>(cam, prm, dir, &len);
        float b[16];
        sh_basis<DEG>(dir[0], dir[1], dir[2], b);
        constexpr int kCount = (DEG + 1) * (DEG + 1);
        float d_dir[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k = 0; k < kCount; ++k) {
            float bg[3];
            sh_basis_gradient_of<DEG>(k, dir[0], dir[1], dir[2], bg);
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float w = d_col[c] * sh[3 * k + c];
                sh[3 * k + c] = b[k] * d_col[c];
#pragma unroll
                for (int a = 0; a < 3; ++a) d_dir[a] += w * bg[a];
            }
        }
        const float dd = dir[0] * d_dir[0] + dir[1] * d_dir[1] + dir[2] * d_dir[2];
#pragma unroll
        for (int a = 0; a < 3; ++a) d_position_sh[a] = div_rn(d_dir[a] - dir[a] * dd, len);
    }
    // dL/dcov2d from dL/dconic (project_backward.wgsl:112-121).
    const float C[2][2] = {{r0.z, r0.w}, {r0.w, r1.x}};
    const float dC[2][2] = {{d_conic[0], 0.5f * d_conic[1]}, {0.5f * d_conic[1], d_conic[2]}};
    float CdC[2][2], F[2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) CdC[i][j] = C[i][0] * dC[0][j] + C[i][1] * dC[1][j];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) F[i][j] = -1.0f * (CdC[i][0] * C[0][j] + CdC[i][1] * C[1][j]);
    const float off = 0.5f * (F[1][0] + F[0][1]);
    const float G[2][2] = {{F[0][0], off}, {off, F[1][1]}};
    // project_backward.wgsl:123-127.
    float A[3][2], dS[3][3], B[2][3], dT[2][3], dJ[2][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int s = 0; s < 2; ++s) A[i][s] = geo.T[0][i] * G[0][s] + geo.T[1][i] * G[1][s];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) dS[i][j] = A[i][0] * geo.T[0][j] + A[i][1] * geo.T[1][j];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j) B[r][j] = G[r][0] * geo.T[0][j] + G[r][1] * geo.T[1][j];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            dT[r][j] = 2.0f * (B[r][0] * geo.Sigma[0][j] + B[r][1] * geo.Sigma[1][j] + B[r][2] * geo.Sigma[2][j]);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 3; ++k)
            dJ[r][k] = dT[r][0] * geo.W[k][0] + dT[r][1] * geo.W[k][1] + dT[r][2] * geo.W[k][2];
    // project_backward.wgsl:129-141.
    float d_pc[3] = {0.0f, 0.0f, 0.0f};
    // The shader's divisions, each the IEEE quotient (div_rn; -(a / b) is (-a) / b exactly).
    const float fx_z2 = div_rn(fx, geo.z2), fy_z2 = div_rn(fy, geo.z2);
    d_pc[0] += geo.clamped[0] ? 0.0f : -fx_z2 * dJ[0][2];
    d_pc[1] += geo.clamped[1] ? 0.0f : -fy_z2 * dJ[1][2];
    d_pc[2] += -fx_z2 * dJ[0][0] - fy_z2 * dJ[1][1] + div_rn(2.0f * fx * geo.tx, z3) * dJ[0][2] +
               div_rn(2.0f * fy * geo.ty, z3) * dJ[1][2];
    d_pc[0] += div_rn(d_mean[0] * fx, pc[2]);
    d_pc[1] += div_rn(d_mean[1] * fy, pc[2]);
    d_pc[2] += div_rn(-d_mean[0] * fx * pc[0], geo.z2) - div_rn(d_mean[1] * fy * pc[1], geo.z2);
#pragma unroll
    for (int j = 0; j < 3; ++j)
        p[SP_SLOT_POSITION + j] = geo.W[0][j] * d_pc[0] + geo.W[1][j] * d_pc[1] + geo.W[2][j] * d_pc[2];
    // The camera (project_backward.wgsl:143-157).
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float jt_dt = geo.J[0][r] * dT[0][c] + geo.J[1][r] * dT[1][c];
            cgrad[r * 3 + c] = d_pc[r] * prm[c] + jt_dt;
        }
    cgrad[9] = d_pc[0];
    cgrad[10] = d_pc[1];
    cgrad[11] = d_pc[2];
    cgrad[12] = div_rn(d_mean[0] * pc[0], pc[2]) + div_rn(dJ[0][0], pc[2]) +
                (geo.clamped[0] ? 0.0f : div_rn(-geo.tx, geo.z2) * dJ[0][2]);
    cgrad[13] = div_rn(d_mean[1] * pc[1], pc[2]) + div_rn(dJ[1][1], pc[2]) +
                (geo.clamped[1] ? 0.0f : div_rn(-geo.ty, geo.z2) * dJ[1][2]);
    if (DEG > 0) {
        // The view direction moves with the position and the camera centre -W^T t.
#pragma unroll
        for (int a = 0; a < 3; ++a) p[SP_SLOT_POSITION + a] += d_position_sh[a];
        const float (*rows)[4] = cam.world_to_camera_rows;
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            cgrad[9 + i] += geo.W[i][0] * d_position_sh[0] + geo.W[i][1] * d_position_sh[1] +
                            geo.W[i][2] * d_position_sh[2];
#pragma unroll
            for (int j = 0; j < 3; ++j) cgrad[i * 3 + j] += rows[i][3] * d_position_sh[j];
        }
    }
    // Scales and rotation (project_backward.wgsl:159-192).
    float dM[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k)
            dM[i][k] = 2.0f * (dS[i][0] * geo.M[0][k] + dS[i][1] * geo.M[1][k] + dS[i][2] * geo.M[2][k]);
#pragma unroll
    for (int k = 0; k < 3; ++k)
        p[SP_SLOT_LOG_SCALE + k] =
            (geo.R[0][k] * dM[0][k] + geo.R[1][k] * dM[1][k] + geo.R[2][k] * dM[2][k]) * geo.scale[k];
    float dR[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k) dR[i][k] = dM[i][k] * geo.scale[k];
    const float r00 = dR[0][0], r01 = dR[0][1], r02 = dR[0][2];
    const float r10 = dR[1][0], r11 = dR[1][1], r12 = dR[1][2];
    const float r20 = dR[2][0], r21 = dR[2][1], r22 = dR[2][2];
    const float qw = geo.q[0], qx = geo.q[1], qy = geo.q[2], qz = geo.q[3];
    const float du[4] = {
        2.0f * (qz * (r10 - r01) + qy * (r02 - r20) + qx * (r21 - r12)),
        2.0f * (qy * (r01 + r10) + qz * (r02 + r20) + qw * (r21 - r12)) - 4.0f * qx * (r11 + r22),
        2.0f * (qx * (r01 + r10) + qw * (r02 - r20) + qz * (r12 + r21)) - 4.0f * qy * (r00 + r22),
        2.0f * (qw * (r10 - r01) + qx * (r02 + r20) + qy * (r12 + r21)) - 4.0f * qz * (r00 + r11),
    };
    const float qdu = geo.q[0] * du[0] + geo.q[1] * du[1] + geo.q[2] * du[2] + geo.q[3] * du[3];
#pragma unroll
    for (int k = 0; k < 4; ++k) p[SP_SLOT_ROTATION + k] = div_rn(du[k] - geo.q[k] * qdu, geo.q_length);
}

// FUSED: Adam and the scale clamp are applied to the block's Gaussians as soon as their
// gradients are complete (adam_block), instead of writing the gradients out for a separate
// Adam pass; `adam` then holds the parameters (the same buffer as `params`, written after
// every read of it) and the moments.
struct FusedAdam {
    float* params;
    float* first_moment;
    float* second_moment;
    AdamStep step;
};

template <int DEG, int MODE, bool FUSED, bool DEV>
__global__ void __launch_bounds__(kBlock, 3) k_project_backward(
    const float* params, uint32_t n, const sp_camera_uniform camera_argument,
    const sp_camera_uniform* __restrict__ camera_device, const float4* __restrict__ records,
    const uint32_t* __restrict__ radii, const uint32_t* __restrict__ offsets, const float* __restrict__ slot_gradients,
    unsigned long long capacity, const float4* __restrict__ gaussian_gradients, float* __restrict__ param_gradients,
    int accumulate, float* __restrict__ camera_partials, uint32_t* camera_done, float* __restrict__ camera_gradient,
    float4* __restrict__ densify_stats, const FusedAdam adam, uint32_t first_block, uint32_t total_blocks) {
    constexpr int S = SP_PARAM_STRIDE(DEG);
    __shared__ sp_camera_uniform s_cam;
    const sp_camera_uniform& cam = pick_camera<DEV>(camera_argument, s_cam);
    if constexpr (DEV) load_camera(camera_device, s_cam);
    extern __shared__ float4 smem4[];
    float* sp = reinterpret_cast<float*>(smem4);
    __shared__ float warp_camera[kBlock / 32][SP_CAMERA_GRAD_STRIDE];
    __shared__ float s_lr[FUSED ? S : 1];
    __shared__ bool last_block;
    // Blocks [first_block, first_block + gridDim.x) of the total_blocks covering the n
    // Gaussians: all at once, or in chunks launched one after the other on one stream; the
    // last block of all to finish reduces the camera gradient.
    const uint32_t block = first_block + blockIdx.x;
    const uint32_t g0 = block * kBlock;
    const uint32_t here = min((uint32_t)kBlock, n - g0);
    // The parameters, the camera and the rates do not depend on the previous grid of the
    // chain (the blend backward, which writes only the blend sums): they are staged before
    // waiting for it, so the first wave's loads overlap that grid's last blocks. Everything
    // below the wait may read what the blend backward wrote.
    stage_in(params + (size_t)g0 * S, here * S, sp);
    if (FUSED && threadIdx.x < (uint32_t)S) s_lr[threadIdx.x] = adam.step.lr[threadIdx.x];
    chain_enter();
    __syncthreads();
    const uint32_t t = threadIdx.x;
    float cgrad[SP_CAMERA_GRAD_STRIDE];
#pragma unroll
    for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) cgrad[c] = 0.0f;
    if (t < here)
        project_backward_one<DEG, MODE>(sp + t * S, g0 + t, cam, records, radii[g0 + t], offsets, slot_gradients,
                                        capacity, gaussian_gradients, densify_stats, cgrad);
    __syncthreads();
    if constexpr (FUSED) {
        adam_block<S>(adam.params, adam.first_moment, adam.second_moment, g0, here, sp, s_lr, adam.step);
        __syncthreads();  // sp is reused by the last block below
    } else {
        // The gradients, coalesced out of shared memory.
        float* out = param_gradients + (size_t)g0 * S;
        for (uint32_t i = t; i < here * S; i += kBlock) out[i] = accumulate ? out[i] + sp[i] : sp[i];
    }
    // The block's camera partial: warp sums, then the 8 warps in order.
    const uint32_t lane = lane_id(), warp = t / 32;
#pragma unroll
    for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) {
        const float v = warp_sum(cgrad[c]);
        if (lane == 0) warp_camera[warp][c] = v;
    }
    __syncthreads();
    if (t < SP_CAMERA_GRAD_STRIDE) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kBlock / 32; ++w) s += warp_camera[w][t];
        camera_partials[(size_t)block * SP_CAMERA_GRAD_STRIDE + t] = s;
    }
    // reduce_camera_gradient.wgsl:10-34 by the last block to finish, in block order.
    __threadfence();
    __syncthreads();
    if (t == 0) {
        cuda::atomic_ref<uint32_t, cuda::thread_scope_device> done(*camera_done);
        last_block = done.fetch_add(1u, cuda::memory_order_acq_rel) == total_blocks - 1;
    }
    __syncthreads();
    if (!last_block) return;
    __threadfence();
    float sums[SP_CAMERA_GRAD_STRIDE];
#pragma unroll
    for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) sums[c] = 0.0f;
    for (uint32_t b = t; b < total_blocks; b += kBlock)
#pragma unroll
        for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) sums[c] += __ldcg(camera_partials + (size_t)b * SP_CAMERA_GRAD_STRIDE + c);
    // The staging buffer (at least 14 floats per thread) is free again: reuse it.
    float (*reduce)[SP_CAMERA_GRAD_STRIDE] = reinterpret_cast<float (*)[SP_CAMERA_GRAD_STRIDE]>(sp);
#pragma unroll
    for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) reduce[t][c] = sums[c];
    __syncthreads();
    for (int half = kBlock / 2; half > 0; half >>= 1) {
        if (t < (uint32_t)half)
#pragma unroll
            for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) reduce[t][c] += reduce[t + half][c];
        __syncthreads();
    }
    if (t < SP_CAMERA_GRAD_STRIDE) camera_gradient[t] = reduce[0][t];
    if (t == 0) *camera_done = 0;
}

__global__ void k_to_projected(const float4* __restrict__ records, const uint32_t* __restrict__ radii, uint32_t n,
                               sp_projected* __restrict__ out) {
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float4 a = records[(size_t)g * kRecord], b = records[(size_t)g * kRecord + 1],
                 c = records[(size_t)g * kRecord + 2];
    sp_projected p;
    p.mean[0] = a.x;
    p.mean[1] = a.y;
    p._pad0[0] = p._pad0[1] = 0.0f;
    p.conic[0] = a.z;
    p.conic[1] = a.w;
    p.conic[2] = b.x;
    p.depth = c.y;
    p.color[0] = b.z;
    p.color[1] = b.w;
    p.color[2] = c.x;
    p.opacity = b.y;
    p.radius = radii[g];
    p._pad1 = 0;
    const uint32_t lo = __float_as_uint(c.z), hi = __float_as_uint(c.w);
    p.tile_min[0] = lo & 0xffffu;
    p.tile_min[1] = lo >> 16;
    p.tile_max[0] = hi & 0xffffu;
    p.tile_max[1] = hi >> 16;
    p._pad2[0] = p._pad2[1] = 0;
    out[g] = p;
}

template <typename Kernel>
cudaError_t set_smem(Kernel kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

cudaError_t launch_project(const float* params, uint64_t n, int sh_degree, const sp_camera_uniform& cam,
                           const sp_camera_uniform* cam_device, float4* records, uint32_t* radii,
                           uint32_t* local_offsets, uint32_t* block_totals, DeviceMeta* depth_range,
                           float4* reach, int tile_culling, cudaStream_t stream) {
    const unsigned grid = grid_for(n, kBlock);
    const size_t smem = (size_t)kBlock * SP_PARAM_STRIDE(sh_degree) * sizeof(float);
    cudaError_t err = cudaSuccess;
#define SPLAT_PROJECT_ONE(D, V)                                                                           \
    if ((err = set_smem(k_project<D, V>, smem)) != cudaSuccess) return err;                                \
    launch_chained(k_project<D, V>, grid, kBlock, smem, stream, params, (uint32_t)n, cam, cam_device, records, radii,  \
                                                    local_offsets, block_totals, depth_range, reach,      \
                                                    (uint32_t)tile_culling);                              \
    return cudaGetLastError();
#define SPLAT_PROJECT(D)                \
    if (sh_degree == D) {               \
        if (cam_device) {               \
            SPLAT_PROJECT_ONE(D, true)  \
        } else {                        \
            SPLAT_PROJECT_ONE(D, false) \
        }                               \
    }
    SPLAT_PROJECT(0)
    SPLAT_PROJECT(1)
    SPLAT_PROJECT(2)
    SPLAT_PROJECT(3)
#undef SPLAT_PROJECT
#undef SPLAT_PROJECT_ONE
    return cudaErrorInvalidValue;
}

cudaError_t launch_scan_blocks(const uint32_t* block_totals, unsigned long long* block_offsets, uint32_t blocks,
                               uint64_t capacity, DeviceMeta* meta, uint32_t* sort_histograms,
                               uint32_t* sort_tickets, const SortPlan& plan, cudaStream_t stream) {
    launch_chained(k_scan_blocks, 1, 1024, 0, stream, block_totals, block_offsets, blocks, capacity, meta, sort_histograms,
                                          sort_tickets, plan);
    return cudaGetLastError();
}

cudaError_t launch_project_backward(const float* params, uint64_t n, int sh_degree, int mode,
                                    const sp_camera_uniform& cam, const sp_camera_uniform* cam_device,
                                    const float4* records, const uint32_t* radii,
                                    const uint32_t* offsets, const float* slot_gradients, uint64_t capacity,
                                    const float4* gaussian_gradients, float* param_gradients, int accumulate,
                                    float* camera_partials, uint32_t* camera_done, float* camera_gradient,
                                    float4* densify_stats, const AdamLaunch* adam, uint64_t first, uint64_t count,
                                    cudaStream_t stream) {
    const unsigned total_blocks = grid_for(n, kBlock);
    if (first % kBlock != 0 || first > n || count > n - first) return cudaErrorInvalidValue;
    const unsigned first_block = (unsigned)(first / kBlock);
    const unsigned grid = grid_for(count, kBlock);
    if (grid == 0) return cudaSuccess;
    const size_t smem = (size_t)kBlock * SP_PARAM_STRIDE(sh_degree) * sizeof(float);
    cudaError_t err = cudaSuccess;
    FusedAdam fused{};
    if (adam) {
        fused.params = adam->params;
        fused.first_moment = adam->first_moment;
        fused.second_moment = adam->second_moment;
        for (int k = 0; k < SP_PARAM_STRIDE(sh_degree); ++k) fused.step.lr[k] = adam->lr_by_slot[k];
        fused.step.set_bias(adam->bias1, adam->bias2);
        fused.step.max_log_scale = adam->max_log_scale;
        fused.step.max_log_anisotropy = adam->max_log_anisotropy;
    }
#define SPLAT_PB_ONE(D, M, F, V)                                                                               \
    if ((err = set_smem(k_project_backward<D, M, F, V>, smem)) != cudaSuccess) return err;                     \
    launch_chained(k_project_backward<D, M, F, V>, grid, kBlock, smem, stream,                                             \
        params, (uint32_t)n, cam, cam_device, records, radii, offsets, slot_gradients, capacity,               \
        gaussian_gradients, param_gradients, accumulate, camera_partials, camera_done, camera_gradient,        \
        densify_stats, fused, first_block, total_blocks);                                                      \
    return cudaGetLastError();
#define SPLAT_PB_CAM(D, M, F)              \
    if (cam_device) {                      \
        SPLAT_PB_ONE(D, M, F, true)        \
    } else {                               \
        SPLAT_PB_ONE(D, M, F, false)       \
    }
#define SPLAT_PB(D, M)                    \
    if (sh_degree == D && mode == M) {    \
        if (adam) {                       \
            SPLAT_PB_CAM(D, M, true)      \
        } else {                          \
            SPLAT_PB_CAM(D, M, false)     \
        }                                 \
    }
    SPLAT_PB(0, SP_BWD_DETERMINISTIC)
    SPLAT_PB(0, SP_BWD_ATOMIC)
    SPLAT_PB(1, SP_BWD_DETERMINISTIC)
    SPLAT_PB(1, SP_BWD_ATOMIC)
    SPLAT_PB(2, SP_BWD_DETERMINISTIC)
    SPLAT_PB(2, SP_BWD_ATOMIC)
    SPLAT_PB(3, SP_BWD_DETERMINISTIC)
    SPLAT_PB(3, SP_BWD_ATOMIC)
#undef SPLAT_PB
#undef SPLAT_PB_CAM
#undef SPLAT_PB_ONE
    return cudaErrorInvalidValue;
}

cudaError_t launch_to_projected(const float4* records, const uint32_t* radii, uint64_t n, sp_projected* out,
                                cudaStream_t stream) {
    k_to_projected<<<grid_for(n, kBlock), kBlock, 0, stream>>>(records, radii, (uint32_t)n, out);
    return cudaGetLastError();
}

}  // namespace splat
