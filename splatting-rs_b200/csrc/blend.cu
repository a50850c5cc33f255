// Alpha blending: forward (K6, rasterize_forward.wgsl:22-88) and backward (K8,
// rasterize_backward.wgsl:30-133).
//
// Forward and atomic backward: one block of 128 threads per 16 x 16 tile; each warp owns an
// 8 x 8 block of it and each lane two pixels of that block, (x, y) and (x, y + 4), whose
// arithmetic runs as packed f32x2 instructions (FFMA2 / FMUL2 / FADD2 of sm_100). Each warp
// walks the tile's sorted list on its own, 32 entries at a time: the entries' 48-B records
// (an L2-resident array) are gathered, one per lane, for the entries whose sorted value
// marks them as reaching the warp's pixels (block bits set once per key by the emission),
// compacted into the warp's shared-memory stage, and read back as broadcasts.
// "Can reach": the Gaussian's alpha is at least 1/255 somewhere in the block's rectangle of
// pixel centres (the exact ellipse-rectangle test, padded), so only pairs the exact
// per-pixel test rejects are left out and no result changes.
//
// The deterministic backward keeps one pixel per thread (256 threads, 8 x 4 pixels per
// warp) and block-synchronous batches, because it writes per-(Gaussian, tile) slots.
//
// The arithmetic per (pixel, Gaussian) is the reference's; exp is the hardware 2^x
// approximation of e^x, and the backward divides by (1 - alpha) through one reciprocal, so
// images and gradients match the oracle within a tolerance rather than bit for bit. The
// decisions that depend on alpha's last bits do not depend on that exp: whether a pixel takes
// a Gaussian (alpha >= 1/255) and whether its alpha is clamped at 0.99 are tests of the
// falloff's power (which is the oracle's bit for bit) against the Gaussian's thresholds in
// record word [3], which the projection derived from the shared, monotone sp_expf_exact; only the
// termination test (transmittance below 1e-4) reads the blended alpha.
#include "kernels.h"

namespace splat {
namespace {

constexpr int kBatch = 256;                  // records per batch (forward, backward atomic mode)
constexpr int kDeterministicBatch = 32;      // backward deterministic mode (per-warp partials)
constexpr int kWarps = kTilePixels / 32;
constexpr uint32_t kFull = 0xffffffffu;

// Pixel of thread (warp, lane) within the tile: warps tile it as 2 x 4 blocks of 8 x 4.
__device__ __forceinline__ uint32_t local_x(uint32_t warp, uint32_t lane) { return ((warp & 1u) << 3) | (lane & 7u); }
__device__ __forceinline__ uint32_t local_y(uint32_t warp, uint32_t lane) { return ((warp >> 1) << 2) | (lane >> 3); }

// Whether the ellipse a x^2 + 2 b x y + c y^2 <= q (a, c > 0, ac > b^2) meets the rectangle
// [x0, x1] x [y0, y1] (coordinates relative to its centre): the minimum of the convex form
// over the rectangle is 0 if the centre is inside, else on an edge, where it is a clamped
// 1-D quadratic.
__device__ __forceinline__ bool ellipse_meets_rect(float a, float b, float c, float q, float x0, float x1, float y0,
                                                   float y1) {
    if (x0 <= 0.0f && x1 >= 0.0f && y0 <= 0.0f && y1 >= 0.0f) return true;
    float best = INFINITY;
    const float xs[2] = {x0, x1}, ys[2] = {y0, y1};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float x = xs[e];
        const float y = fminf(fmaxf(-b * x / c, y0), y1);
        best = fminf(best, a * x * x + 2.0f * b * x * y + c * y * y);
        const float yy = ys[e];
        const float xx = fminf(fmaxf(-b * yy / a, x0), x1);
        best = fminf(best, a * xx * xx + 2.0f * b * xx * yy + c * yy * yy);
    }
    return best <= q;
}

// The warp blocks of tile (gx, gy) that a Gaussian can reach, one bit per warp: where
// op * exp(power) >= 1/255 can hold, i.e. inside the ellipse d^T C d <= 2 ln(255 op) of the
// conic C, padded by 1 % in the level; each block's rectangle of pixel centres is padded
// by 0.05 px. A bounding-box test first, then the exact ellipse test.
__device__ __forceinline__ uint32_t warp_mask(float4 a, float4 b, uint32_t gx, uint32_t gy) {
    const float level = b.y * 255.0f;
    if (!(level > 1.0f)) return 0u;
    const float det = a.z * b.x - a.w * a.w;
    if (!(det > 0.0f) || !(a.z > 0.0f) || !(b.x > 0.0f)) return 0xffu;
    const float q = 2.02f * __logf(level) + 0.02f;
    const float ex = sqrtf(q * b.x / det) + 0.05f;
    const float ey = sqrtf(q * a.z / det) + 0.05f;
    const float x0 = (float)(gx * SP_TILE) - a.x, y0 = (float)(gy * SP_TILE) - a.y;
    uint32_t mask = 0;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float lo_y = y0 + 4.0f * r - 0.05f, hi_y = lo_y + 3.1f;
        if (ey < lo_y || -ey > hi_y) continue;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float lo_x = x0 + 8.0f * c - 0.05f, hi_x = lo_x + 7.1f;
            if (ex < lo_x || -ex > hi_x) continue;
            if (ellipse_meets_rect(a.z, a.w, b.x, q, lo_x, hi_x, lo_y, hi_y)) mask |= 1u << (2 * r + c);
        }
    }
    return mask;
}

// This warp's list of batch entries k < n whose mask has its bit (and that pass `keep`),
// in increasing k, written to `list`; returns its length.
template <int B, typename Keep>
__device__ __forceinline__ uint32_t compact(const uint8_t* masks, uint32_t n, uint32_t warp, uint32_t lane,
                                            uint16_t* list, Keep keep) {
    uint32_t length = 0;
#pragma unroll
    for (int chunk = 0; chunk < B / 32; ++chunk) {
        const uint32_t k = chunk * 32 + lane;
        const bool take = k < n && ((masks[k] >> warp) & 1u) && keep(k);
        const uint32_t ballot = __ballot_sync(kFull, take);
        if (take) list[length + __popc(ballot & ((1u << lane) - 1u))] = (uint16_t)k;
        length += __popc(ballot);
    }
    __syncwarp();
    return length;
}

// One warp's staging area: the records of a 32-entry chunk of the tile list that reach the
// warp's 8 x 4 pixels, compacted in list order.
struct WarpStage {
    float4 a[32];     // mean.x, mean.y, conic.a, conic.b
    float4 b[32];     // conic.c, opacity, colour.r, colour.g
    float4 c[32];     // colour.b, take_from, clamp_from (record word [3]), 0
    uint32_t j[32];   // index in the tile list
    uint32_t g[32];   // Gaussian
};

// Takes entries base .. base + 31 (below `end`) of the tile list, one per lane, keeps those
// whose value marks them as reaching the warp's 8 x 8 block `warp` (the emission's block
// bits), gathers only their records, compacted into `st`; returns how many.
__device__ __forceinline__ uint32_t stage_chunk(const float4* __restrict__ records, const uint32_t* __restrict__ sorted,
                                                uint32_t first, uint32_t base, uint32_t end, uint32_t warp,
                                                uint32_t lane, WarpStage& st) {
    const uint32_t j = base + lane;
    bool take = false;
    float4 a, b, c;
    uint32_t g = 0;
    if (j < end) {
        const uint32_t value = sorted[first + j];
        g = value & kGaussianMask;
        take = (value >> (kGaussianBits + warp)) & 1u;
    }
    if (take) {
        const float4* rec = records + (size_t)g * kRecord;
        a = rec[0];
        b = rec[1];
        const float2 thresholds = *reinterpret_cast<const float2*>(rec + 3);
        c = make_float4(rec[2].x, thresholds.x, thresholds.y, 0.0f);
    }
    const uint32_t ballot = __ballot_sync(kFull, take);
    if (take) {
        const uint32_t p = __popc(ballot & ((1u << lane) - 1u));
        st.a[p] = a;
        st.b[p] = b;
        st.c[p] = c;
        st.j[p] = j;
        st.g[p] = g;
    }
    __syncwarp();
    return __popc(ballot);
}

// Packed f32x2 arithmetic (sm_100).
__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }

// 2^x by the hardware approximation (PTX ex2.approx).
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kPairWarps = 4;                     // forward / atomic backward: 8 x 8 pixels per warp
constexpr int kPairThreads = kPairWarps * 32;
// Atomic backward: a Gaussian's terms from at most this many active lanes are added by those
// lanes directly instead of through the warp reduction (~50 instructions): two float4 vector
// atomics (sm_90+) and one scalar each, so each lane costs the L2 three atomic operations, not
// nine. Measured at config 2: 8 -> 20 lanes took the backward from 342 to 319 us (12-24 within
// 3 us of it; 28 gave 329 us, 32 -- no reduction at all -- 477 us: the L2's atomic units
// saturate). With scalar atomics the best threshold had been 8.
constexpr int kDirectAtomicLanes = 20;

// The falloff of one Gaussian at a lane's two pixels (fpx, fpy.x) and (fpx, fpy.y)
// (rasterize_forward.wgsl:60-66): power = -1/2 (a dx^2 + c dy^2) - b dx dy of the conic
// (a, b, c), d = mean - pixel, rounded operation by operation in the reference's order
// (no fused multiply-adds), so that power is the oracle's bit for bit; gaussian = e^power,
// evaluated as 2^(power log2 e) in packed arithmetic.
struct Falloff {
    float dx;
    float2 dy;
    float2 power;
    float2 gaussian;
    bool below0, below1;  // power <= 0
};

__device__ __forceinline__ Falloff falloff(float4 a, float4 b, float fpx, float2 fpy) {
    Falloff f;
    // Rounded operation by operation, as the oracle: the sums and differences are scalar
    // operations with explicit rounding, which the compiler never contracts into a fused
    // multiply-add; the products are packed (FMUL2, one rounding per lane), which is safe
    // because every product feeds one of those scalar sums or another product. Packed sums
    // are not used: the compiler contracts packed products and sums into FFMA2 whatever their
    // rounding modifier, as intrinsics (__fadd2_rn) and as inline PTX (add.rn.f32x2) alike
    // (measured: 14 % of such powers differed from the oracle's where the three terms cancel;
    // tests/test_gpu_parity.py pins this form bit for bit through sp_debug_falloff_powers).
    // The row offsets dy are sums too, but of no product: packed.
    f.dx = __fadd_rn(a.x, -fpx);
    f.dy = __fadd2_rn(splat(a.y), make_float2(-fpy.x, -fpy.y));
    const float t0 = __fmul_rn(__fmul_rn(a.z, f.dx), f.dx), cross = __fmul_rn(a.w, f.dx);
    const float2 q = __fmul2_rn(__fmul2_rn(splat(b.x), f.dy), f.dy);
    const float2 cd = __fmul2_rn(splat(cross), f.dy);
    const float2 quad = make_float2(__fadd_rn(t0, q.x), __fadd_rn(t0, q.y));
    const float2 h = __fmul2_rn(splat(-0.5f), quad);
    const float2 power = make_float2(__fadd_rn(h.x, -cd.x), __fadd_rn(h.y, -cd.y));
    f.power = power;
    f.below0 = power.x <= 0.0f;
    f.below1 = power.y <= 0.0f;
    const float2 power2 = mul2(power, splat(kLog2e));
    f.gaussian = make_float2(exp2_approx(power2.x), exp2_approx(power2.y));
    return f;
}

// falloff() at one pixel, with the same roundings (for the one-pixel-per-thread kernels).
__device__ __forceinline__ float falloff1(float4 a, float4 b, float fpx, float fpy, float& dx, float& dy,
                                          bool& below, float& power) {
    dx = __fadd_rn(a.x, -fpx);
    dy = __fadd_rn(a.y, -fpy);
    const float quad = __fadd_rn(__fmul_rn(__fmul_rn(a.z, dx), dx), __fmul_rn(__fmul_rn(b.x, dy), dy));
    power = __fadd_rn(__fmul_rn(-0.5f, quad), -__fmul_rn(__fmul_rn(a.w, dx), dy));
    below = power <= 0.0f;
    return exp2_approx(__fmul_rn(power, kLog2e));
}

// Each warp walks the tile's list on its own, 32 entries at a time, over only the
// Gaussians that reach its 8 x 8 pixels; no block barrier, and a warp whose pixels are all
// done leaves.
__global__ void __launch_bounds__(kPairThreads, 8) k_blend_forward(const float4* __restrict__ records,
                                                                   const uint32_t* __restrict__ sorted,
                                                                   const uint2* __restrict__ ranges,
                                                                   const uint32_t* __restrict__ order,
                                                                   const sp_camera_uniform cam,
                                                                   float4* __restrict__ image,
                                                                   uint32_t* __restrict__ contributions) {
    chain_enter();
    __shared__ WarpStage s_stage[kPairWarps];
    const uint32_t tile = order[blockIdx.x];
    const uint32_t gx = tile % cam.tiles_x, gy = tile / cam.tiles_x;
    const uint32_t warp = threadIdx.x / 32, lane = lane_id();
    const uint32_t bx = gx * SP_TILE + ((warp & 1u) << 3), by = gy * SP_TILE + ((warp >> 1) << 3);
    const uint32_t px = bx + (lane & 7u), py = by + (lane >> 3);
    const bool inside0 = px < cam.width && py < cam.height, inside1 = px < cam.width && py + 4 < cam.height;
    const float fpx = (float)px;
    const float2 fpy = make_float2((float)py, (float)(py + 4));
    const uint2 range = ranges[tile];
    const uint32_t count = range.y - range.x;
    WarpStage& st = s_stage[warp];

    // rasterize_forward.wgsl:58-77 at both pixels.
    float2 transmittance = splat(1.0f), cr = splat(0.0f), cg = splat(0.0f), cb = splat(0.0f);
    uint32_t contributed0 = 0, contributed1 = 0;
    bool done0 = !inside0, done1 = !inside1;
    for (uint32_t base = 0; base < count; base += 32) {
        if (__all_sync(kFull, done0 && done1)) break;
        const uint32_t n =
            stage_chunk(records, sorted, range.x, base, count, warp, lane, st);
        for (uint32_t i = 0; i < n && !(done0 && done1); ++i) {
            const float4 a = st.a[i], b = st.b[i];
            const float2 c = *reinterpret_cast<const float2*>(&st.c[i]);  // colour.b, take_from
            const Falloff f = falloff(a, b, fpx, fpy);
            const float2 unclamped = mul2(splat(b.y), f.gaussian);
            const float2 alpha = make_float2(fminf(SP_MAX_ALPHA, unclamped.x), fminf(SP_MAX_ALPHA, unclamped.y));
            bool take0 = !done0 && f.below0 && f.power.x >= c.y;
            bool take1 = !done1 && f.below1 && f.power.y >= c.y;
            const float2 next = mul2(transmittance, add2(splat(1.0f), neg2(alpha)));
            // A pixel whose transmittance would fall below the floor ends before this one.
            const bool end0 = take0 && next.x < SP_MIN_TRANSMITTANCE, end1 = take1 && next.y < SP_MIN_TRANSMITTANCE;
            take0 = take0 && !end0;
            take1 = take1 && !end1;
            done0 = done0 || end0;
            done1 = done1 || end1;
            float2 w = mul2(alpha, transmittance);
            w.x = take0 ? w.x : 0.0f;
            w.y = take1 ? w.y : 0.0f;
            cr = fma2(splat(b.z), w, cr);
            cg = fma2(splat(b.w), w, cg);
            cb = fma2(splat(c.x), w, cb);
            const uint32_t j1 = st.j[i] + 1;
            if (take0) {
                transmittance.x = next.x;
                contributed0 = j1;
            }
            if (take1) {
                transmittance.y = next.y;
                contributed1 = j1;
            }
        }
        __syncwarp();
    }
    const size_t index = (size_t)py * cam.width + px;
    if (inside0) {
        image[index] = make_float4(cr.x, cg.x, cb.x, transmittance.x);
        contributions[index] = contributed0;
    }
    if (inside1) {
        image[index + 4 * (size_t)cam.width] = make_float4(cr.y, cg.y, cb.y, transmittance.y);
        contributions[index + 4 * (size_t)cam.width] = contributed1;
    }
}

// The slot of (Gaussian, tile) in the reference's per-intersection gradient list: the
// Gaussian's tile offset plus the tile's row-major index in its rectangle
// (emit_tile_keys.wgsl:21-33).
__device__ __forceinline__ uint64_t slot_of(const float4* __restrict__ records, const uint32_t* __restrict__ offsets,
                                            uint32_t g, uint32_t gx, uint32_t gy) {
    const float4 r2 = records[(size_t)g * kRecord + 2];
    const uint32_t lo = __float_as_uint(r2.z), hi = __float_as_uint(r2.w);
    const uint32_t x0 = lo & 0xffffu, y0 = lo >> 16, x1 = hi & 0xffffu;
    return (uint64_t)offsets[g] + (uint64_t)(gy - y0) * (x1 - x0) + (gx - x0);
}

// Warp sums of 8 values with 9 shuffles instead of 40: at each of the first three levels
// a lane keeps half of its values and trades the other half with its partner, so that
// after them lane l holds a partial of value (l >> 2) & 7 only; two full levels finish.
// Returns the warp total of value (lane >> 2) & 7.
__device__ __forceinline__ float reduce8_transposed(const float v[8], uint32_t lane) {
    const bool b4 = lane & 16u, b3 = lane & 8u, b2 = lane & 4u;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = b4 ? v[i + 4] : v[i];
        const float send = b4 ? v[i] : v[i + 4];
        x[i] = keep + __shfl_xor_sync(kFull, send, 16);
    }
    float y[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float keep = b3 ? x[i + 2] : x[i];
        const float send = b3 ? x[i] : x[i + 2];
        y[i] = keep + __shfl_xor_sync(kFull, send, 8);
    }
    float z = (b2 ? y[1] : y[0]) + __shfl_xor_sync(kFull, b2 ? y[0] : y[1], 4);
    z += __shfl_xor_sync(kFull, z, 2);
    z += __shfl_xor_sync(kFull, z, 1);
    return z;
}

template <int MODE>
__global__ void __launch_bounds__(kTilePixels) k_blend_backward(
    const float4* __restrict__ records, const uint32_t* __restrict__ sorted, const uint2* __restrict__ ranges,
    const uint32_t* __restrict__ order, const uint32_t* __restrict__ offsets, const sp_camera_uniform cam,
    const float4* __restrict__ image,
    const uint32_t* __restrict__ contributions, const float4* __restrict__ loss_gradient,
    float* __restrict__ slot_gradients, float4* __restrict__ gaussian_gradients) {
    constexpr bool kDet = MODE == SP_BWD_DETERMINISTIC;
    constexpr int B = kDet ? kDeterministicBatch : kBatch;
    __shared__ float4 s_a[B];
    __shared__ float4 s_b[B];
    __shared__ float4 s_c[B];  // colour.b, take_from, clamp_from, 0
    __shared__ uint32_t s_g[B];
    __shared__ uint8_t s_mask[B];
    __shared__ uint16_t s_list[kWarps][B];
    __shared__ float s_part[kDet ? B : 1][kWarps][9];
    __shared__ uint32_t s_limit;

    const uint32_t tile = order[blockIdx.x];
    const uint32_t gx = tile % cam.tiles_x, gy = tile / cam.tiles_x;
    const uint32_t t = threadIdx.x, lane = lane_id(), warp = t / 32;
    const uint32_t px = gx * SP_TILE + local_x(warp, lane), py = gy * SP_TILE + local_y(warp, lane);
    const bool inside = px < cam.width && py < cam.height;
    const float fpx = (float)px, fpy = (float)py;
    const uint2 range = ranges[tile];
    const uint32_t count = range.y - range.x;
    uint16_t* list = s_list[warp];

    float transmittance = 0.0f;
    uint32_t contributed = 0;
    float4 grad = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (inside) {
        const size_t index = (size_t)py * cam.width + px;
        transmittance = image[index].w;
        contributed = contributions[index];
        grad = loss_gradient[index];
    }
    // No pixel replays past its contributor count: the warp's list stops at its largest,
    // the block's batches at the largest of all.
    if (t == 0) s_limit = 0;
    __syncthreads();
    const uint32_t warp_limit = __reduce_max_sync(kFull, contributed);
    if (lane == 0) atomicMax(&s_limit, warp_limit);
    __syncthreads();
    const uint32_t limit = min(s_limit, count);

    float behind_r = 0.0f, behind_g = 0.0f, behind_b = 0.0f, behind_t = transmittance;
    const uint32_t batches = (limit + B - 1) / B;
    for (uint32_t bb = 0; bb < batches; ++bb) {
        const uint32_t base = (batches - 1 - bb) * B;
        __syncthreads();
        if (t < (uint32_t)B && base + t < limit) {
            const uint32_t g = sorted[range.x + base + t] & kGaussianMask;
            const float4* rec = records + (size_t)g * kRecord;
            const float4 a = rec[0], b = rec[1];
            s_g[t] = g;
            s_a[t] = a;
            s_b[t] = b;
            const float2 thresholds = *reinterpret_cast<const float2*>(rec + 3);
            s_c[t] = make_float4(rec[2].x, thresholds.x, thresholds.y, 0.0f);
            s_mask[t] = (uint8_t)warp_mask(a, b, gx, gy);
        }
        if (kDet)
            for (uint32_t i = lane; i < (uint32_t)B * 9; i += 32) s_part[i / 9][warp][i % 9] = 0.0f;
        __syncthreads();
        const uint32_t n = min((uint32_t)B, limit - base);
        const uint32_t length =
            compact<B>(s_mask, n, warp, lane, list, [&](uint32_t k) { return base + k < warp_limit; });
        for (int i = (int)length - 1; i >= 0; --i) {
            const uint32_t k = list[i];
            const uint32_t j = base + k;
            float v[9];
#pragma unroll
            for (int c = 0; c < 9; ++c) v[c] = 0.0f;
            bool active = false;
            if (j < contributed) {
                const float4 a = s_a[k];
                const float4 b = s_b[k];
                const float4 c = s_c[k];
                float dx, dy, power;
                bool below;
                const float gaussian = falloff1(a, b, fpx, fpy, dx, dy, below, power);
                if (below) {
                    const float opacity = b.y;
                    const float alpha_unclamped = opacity * gaussian;
                    const float alpha = fminf(SP_MAX_ALPHA, alpha_unclamped);
                    if (power >= c.y) {
                        active = true;
                        const float inv = __fdividef(1.0f, 1.0f - alpha);
                        transmittance = transmittance * inv;
                        const float cr = b.z, cgr = b.w, cbl = c.x;
                        const float d_alpha = grad.x * (cr * transmittance - behind_r * inv) +
                                              grad.y * (cgr * transmittance - behind_g * inv) +
                                              grad.z * (cbl * transmittance - behind_b * inv) -
                                              grad.w * (behind_t * inv);
                        const float w = alpha * transmittance;
                        v[5] = grad.x * w;
                        v[6] = grad.y * w;
                        v[7] = grad.z * w;
                        behind_r += cr * w;
                        behind_g += cgr * w;
                        behind_b += cbl * w;
                        if (power < c.z) {
                            v[8] = d_alpha * gaussian;
                            const float d_power = d_alpha * opacity * gaussian;
                            v[0] = -d_power * (a.z * dx + a.w * dy);
                            v[1] = -d_power * (a.w * dx + b.x * dy);
                            v[2] = -0.5f * d_power * dx * dx;
                            v[3] = -d_power * dx * dy;
                            v[4] = -0.5f * d_power * dy * dy;
                        }
                    }
                }
            }
            if (__ballot_sync(kFull, active)) {
                const float total = reduce8_transposed(v, lane);
                const float opacity_total = warp_sum(v[8]);
                const uint32_t which = (lane >> 2) & 7u;
                if (!kDet) {
                    float* out = reinterpret_cast<float*>(gaussian_gradients + (size_t)s_g[k] * 3);
                    if ((lane & 3u) == 0) atomicAdd(out + which, total);
                    if (lane == 0) atomicAdd(out + 8, opacity_total);
                } else {
                    if ((lane & 3u) == 0) s_part[k][warp][which] = total;
                    if (lane == 0) s_part[k][warp][8] = opacity_total;
                }
            }
        }
        if (kDet) {
            // One write per (Gaussian, tile) slot: the warps' sums in warp order.
            __syncthreads();
            for (uint32_t i = t; i < n * SP_GRAD_STRIDE; i += kTilePixels) {
                const uint32_t k = i / SP_GRAD_STRIDE, c = i % SP_GRAD_STRIDE;
                float s = 0.0f;
                if (c < 9)
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) s += s_part[k][w][c];
                slot_gradients[slot_of(records, offsets, s_g[k], gx, gy) * SP_GRAD_STRIDE + c] = s;
            }
        }
    }
    if (kDet) {
        // Entries past every pixel's last contributor get zero slots, as the reference
        // writes every entry of the tile.
        for (uint32_t i = t; i < (count - limit) * SP_GRAD_STRIDE; i += kTilePixels) {
            const uint32_t j = limit + i / SP_GRAD_STRIDE, c = i % SP_GRAD_STRIDE;
            const uint32_t g = sorted[range.x + j] & kGaussianMask;
            slot_gradients[slot_of(records, offsets, g, gx, gy) * SP_GRAD_STRIDE + c] = 0.0f;
        }
    }
}

// The backward with per-Gaussian sums by float atomics (SP_BWD_ATOMIC): each warp walks
// the tile's list on its own, back to front from its pixels' largest contributor count, 32
// entries at a time, over only the Gaussians that reach its 8 x 8 pixels. Per (Gaussian,
// warp) a lane adds its two pixels' 9 gradient terms, the lanes' sums are reduced
// (reduce8_transposed plus one butterfly) and added into the Gaussian's sums by up to 9
// lanes at once.
__global__ void __launch_bounds__(kPairThreads, 6) k_blend_backward_atomic(
    const float4* __restrict__ records, const uint32_t* __restrict__ sorted, const uint2* __restrict__ ranges,
    const uint32_t* __restrict__ order, const sp_camera_uniform cam,
    const float4* __restrict__ image, const uint32_t* __restrict__ contributions,
    const float4* __restrict__ loss_gradient, float4* __restrict__ gaussian_gradients) {
    chain_enter();
    __shared__ WarpStage s_stage[kPairWarps];
    const uint32_t tile = order[blockIdx.x];
    const uint32_t gx = tile % cam.tiles_x, gy = tile / cam.tiles_x;
    const uint32_t warp = threadIdx.x / 32, lane = lane_id();
    const uint32_t bx = gx * SP_TILE + ((warp & 1u) << 3), by = gy * SP_TILE + ((warp >> 1) << 3);
    const uint32_t px = bx + (lane & 7u), py = by + (lane >> 3);
    const bool inside0 = px < cam.width && py < cam.height, inside1 = px < cam.width && py + 4 < cam.height;
    const float fpx = (float)px;
    const float2 fpy = make_float2((float)py, (float)(py + 4));
    const uint2 range = ranges[tile];
    WarpStage& st = s_stage[warp];

    // Per pixel: final transmittance, contributor count, dL/d(rgb, transmittance).
    float2 transmittance = splat(0.0f), gr = splat(0.0f), gg = splat(0.0f), gb = splat(0.0f), gt = splat(0.0f);
    uint32_t contributed0 = 0, contributed1 = 0;
    const size_t index = (size_t)py * cam.width + px;
    if (inside0) {
        const float4 g = loss_gradient[index];
        transmittance.x = image[index].w;
        contributed0 = contributions[index];
        gr.x = g.x, gg.x = g.y, gb.x = g.z, gt.x = g.w;
    }
    if (inside1) {
        const size_t i1 = index + 4 * (size_t)cam.width;
        const float4 g = loss_gradient[i1];
        transmittance.y = image[i1].w;
        contributed1 = contributions[i1];
        gr.y = g.x, gg.y = g.y, gb.y = g.z, gt.y = g.w;
    }
    const uint32_t end = min(__reduce_max_sync(kFull, max(contributed0, contributed1)), range.y - range.x);
    // rasterize_backward.wgsl:166-200. The colour behind each entry accumulates back to
    // front; dL/dalpha = T (g . c) - (g . behind + g_T T_final) / (1 - alpha), with T the
    // transmittance in front of the entry.
    float2 behind_r = splat(0.0f), behind_g = splat(0.0f), behind_b = splat(0.0f);
    const float2 behind_t = mul2(gt, transmittance);
    for (int base = end ? (int)((end - 1) & ~31u) : -32; base >= 0; base -= 32) {
        const uint32_t n =
            stage_chunk(records, sorted, range.x, (uint32_t)base, end, warp, lane, st);
        for (int i = (int)n - 1; i >= 0; --i) {
            const uint32_t j = st.j[i];
            const float4 a = st.a[i], b = st.b[i];
            const float4 c = st.c[i];  // colour.b, take_from, clamp_from
            const Falloff f = falloff(a, b, fpx, fpy);
            const float2 unclamped = mul2(splat(b.y), f.gaussian);
            float2 alpha = make_float2(fminf(SP_MAX_ALPHA, unclamped.x), fminf(SP_MAX_ALPHA, unclamped.y));
            const bool take0 = j < contributed0 && f.below0 && f.power.x >= c.y;
            const bool take1 = j < contributed1 && f.below1 && f.power.y >= c.y;
            const uint32_t active = __ballot_sync(kFull, take0 || take1);
            if (!active) continue;
            alpha.x = take0 ? alpha.x : 0.0f;
            alpha.y = take1 ? alpha.y : 0.0f;
            const float2 one_minus = add2(splat(1.0f), neg2(alpha));
            const float2 inv = make_float2(__fdividef(1.0f, one_minus.x), __fdividef(1.0f, one_minus.y));
            const float2 divided = mul2(transmittance, inv);
            transmittance.x = take0 ? divided.x : transmittance.x;
            transmittance.y = take1 ? divided.y : transmittance.y;
            const float cbl = c.x;
            const float2 g_dot_c = fma2(gb, splat(cbl), fma2(gg, splat(b.w), mul2(gr, splat(b.z))));
            const float2 g_dot_behind = fma2(gb, behind_b, fma2(gg, behind_g, fma2(gr, behind_r, behind_t)));
            const float2 d_alpha = fma2(neg2(inv), g_dot_behind, mul2(transmittance, g_dot_c));
            const float2 w = mul2(alpha, transmittance);
            const float2 d_r = mul2(gr, w), d_g = mul2(gg, w), d_b = mul2(gb, w);
            behind_r = fma2(splat(b.z), w, behind_r);
            behind_g = fma2(splat(b.w), w, behind_g);
            behind_b = fma2(splat(cbl), w, behind_b);
            // The clamp at 0.99 passes no gradient to opacity or the falloff.
            const float2 gate = make_float2(take0 && f.power.x < c.z ? f.gaussian.x : 0.0f,
                                            take1 && f.power.y < c.z ? f.gaussian.y : 0.0f);
            const float2 d_opacity = mul2(d_alpha, gate);
            const float2 nd_power = mul2(d_opacity, splat(-b.y));  // -dL/dpower
            const float2 d_mx = mul2(nd_power, fma2(splat(a.w), f.dy, splat(a.z * f.dx)));
            const float2 d_my = mul2(nd_power, fma2(splat(b.x), f.dy, splat(a.w * f.dx)));
            const float2 d_ca = mul2(nd_power, splat(0.5f * f.dx * f.dx));
            const float2 d_cb = mul2(mul2(nd_power, splat(f.dx)), f.dy);
            const float2 d_cc = mul2(mul2(nd_power, mul2(splat(0.5f), f.dy)), f.dy);
            const float v[8] = {d_mx.x + d_mx.y, d_my.x + d_my.y, d_ca.x + d_ca.y, d_cb.x + d_cb.y,
                                d_cc.x + d_cc.y, d_r.x + d_r.y,   d_g.x + d_g.y,   d_b.x + d_b.y};
            float* out = reinterpret_cast<float*>(gaussian_gradients + (size_t)st.g[i] * 3);
            if (__popc(active) <= kDirectAtomicLanes) {
                // Few lanes hold terms: they add their own, without the warp reduction.
                if (take0 || take1) {
                    // Sums 0-3 (mean, conic a, b) and 4-7 (conic c, colour): float4 words 0 and 1.
                    float4* out4 = gaussian_gradients + (size_t)st.g[i] * 3;
                    atomicAdd(out4, make_float4(v[0], v[1], v[2], v[3]));
                    atomicAdd(out4 + 1, make_float4(v[4], v[5], v[6], v[7]));
                    atomicAdd(out + 8, d_opacity.x + d_opacity.y);
                }
            } else {
                const float total = reduce8_transposed(v, lane);
                const float opacity_total = warp_sum(d_opacity.x + d_opacity.y);
                if ((lane & 3u) == 0) atomicAdd(out + ((lane >> 2) & 7u), total);
                if (lane == 0) atomicAdd(out + 8, opacity_total);
            }
        }
        __syncwarp();
    }
}

// Tiles in decreasing order of list length: a counting sort on the length's quarter-octave
// bucket (the bit length and the two bits below the leading one), by one block; the order
// within a bucket is the atomics' and does not matter, each tile's results being its own.
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 129;  // 128 for lengths 1 .. 2^32 - 1, the last for empty tiles

__device__ __forceinline__ uint32_t order_bucket(uint2 range) {
    const uint32_t count = range.y - range.x;
    if (count == 0) return kOrderBuckets - 1;
    const uint32_t msb = 31u - __clz(count);
    const uint32_t below = msb >= 2 ? (count >> (msb - 2)) & 3u : (count << (2 - msb)) & 3u;
    return 127u - (msb * 4u + below);
}

__global__ void __launch_bounds__(kOrderThreads) k_tile_order(const uint2* __restrict__ ranges, uint32_t tiles,
                                                              uint32_t* __restrict__ order) {
    chain_enter();
    __shared__ uint32_t s_next[kOrderBuckets];
    const uint32_t t = threadIdx.x;
    for (uint32_t b = t; b < kOrderBuckets; b += kOrderThreads) s_next[b] = 0;
    __syncthreads();
    for (uint32_t tile = t; tile < tiles; tile += kOrderThreads) atomicAdd(&s_next[order_bucket(ranges[tile])], 1u);
    __syncthreads();
    if (t < 32) {
        // Exclusive scan of the bucket sizes: 5 consecutive buckets per lane, then the lanes.
        constexpr int kPer = (kOrderBuckets + 31) / 32;
        uint32_t own[kPer], total = 0;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t b = t * kPer + k;
            own[k] = b < kOrderBuckets ? s_next[b] : 0u;
            total += own[k];
        }
        uint32_t inclusive = total;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(kFull, inclusive, o);
            if (t >= (uint32_t)o) inclusive += v;
        }
        uint32_t start = inclusive - total;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t b = t * kPer + k;
            if (b < kOrderBuckets) s_next[b] = start;
            start += own[k];
        }
    }
    __syncthreads();
    for (uint32_t tile = t; tile < tiles; tile += kOrderThreads)
        order[atomicAdd(&s_next[order_bucket(ranges[tile])], 1u)] = tile;
}

// The forward's per-pixel walk without the colour, counting the entries visited (up to
// and including the terminating one), the entries taken (blended: alpha at least 1/255,
// before the termination), plus the contributor counts the backward replays.
__global__ void __launch_bounds__(kTilePixels) k_count_blend(const float4* __restrict__ records,
                                                             const uint32_t* __restrict__ sorted,
                                                             const uint2* __restrict__ ranges,
                                                             const sp_camera_uniform cam,
                                                             const uint32_t* __restrict__ contributions,
                                                             unsigned long long* counts) {
    const uint32_t tile = blockIdx.x;
    const uint32_t gx = tile % cam.tiles_x, gy = tile / cam.tiles_x;
    const uint32_t t = threadIdx.x;
    const uint32_t px = gx * SP_TILE + local_x(t / 32, lane_id()), py = gy * SP_TILE + local_y(t / 32, lane_id());
    unsigned long long visited = 0, replayed = 0, taken = 0;
    if (px < cam.width && py < cam.height) {
        const uint2 range = ranges[tile];
        const float fpx = (float)px, fpy = (float)py;
        float transmittance = 1.0f;
        for (uint32_t j = range.x; j < range.y; ++j) {
            ++visited;
            const float4* rec = records + (size_t)(sorted[j] & kGaussianMask) * kRecord;
            const float4 a = rec[0], b = rec[1];
            float dx, dy, power;
            bool below;
            const float gaussian = falloff1(a, b, fpx, fpy, dx, dy, below, power);
            if (!below || power < rec[3].x) continue;
            const float alpha = fminf(SP_MAX_ALPHA, b.y * gaussian);
            const float next = transmittance * (1.0f - alpha);
            if (next < SP_MIN_TRANSMITTANCE) break;
            transmittance = next;
            ++taken;
        }
        replayed = contributions[(size_t)py * cam.width + px];
    }
    visited = __reduce_add_sync(kFull, (unsigned)visited);
    replayed = __reduce_add_sync(kFull, (unsigned)replayed);
    taken = __reduce_add_sync(kFull, (unsigned)taken);
    if (lane_id() == 0) {
        atomicAdd(counts, visited);
        atomicAdd(counts + 1, replayed);
        atomicAdd(counts + 2, taken);
    }
}

// Test support: the falloff power of item i (record words a = in[3i], b = in[3i + 1], pixel
// column in[3i + 2].x, rows .y and .z) as falloff() gives it to the forward and the atomic
// backward.
__global__ void k_falloff_powers(const float4* __restrict__ in, uint64_t n, float2* __restrict__ out) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float4 pixel = in[3 * i + 2];
    out[i] = falloff(in[3 * i], in[3 * i + 1], pixel.x, make_float2(pixel.y, pixel.z)).power;
}

}  // namespace

cudaError_t launch_count_blend(const float4* records, const uint32_t* sorted_gaussians, const uint2* ranges,
                               const sp_camera_uniform& cam, const uint32_t* contributions,
                               unsigned long long* counts, cudaStream_t stream) {
    k_count_blend<<<cam.tiles_x * cam.tiles_y, kTilePixels, 0, stream>>>(records, sorted_gaussians, ranges, cam,
                                                                          contributions, counts);
    return cudaGetLastError();
}

cudaError_t launch_tile_order(const uint2* ranges, uint32_t tiles, uint32_t* order, cudaStream_t stream) {
    launch_chained(k_tile_order, 1, kOrderThreads, 0, stream, ranges, tiles, order);
    return cudaGetLastError();
}

cudaError_t launch_blend_forward(const float4* records, const uint32_t* sorted_gaussians,
                                 const uint2* ranges, const uint32_t* order, const sp_camera_uniform& cam,
                                 float4* image, uint32_t* contributions, cudaStream_t stream) {
    const unsigned tiles = cam.tiles_x * cam.tiles_y;
    launch_chained(k_blend_forward, tiles, kPairThreads, 0, stream, records, sorted_gaussians, ranges, order, cam, image,
                                                        contributions);
    return cudaGetLastError();
}

cudaError_t launch_blend_backward(int mode, const float4* records, const uint32_t* sorted_gaussians,
                                  const uint2* ranges, const uint32_t* order, const uint32_t* offsets,
                                  const sp_camera_uniform& cam, const float4* image, const uint32_t* contributions,
                                  const float4* loss_gradient, float* slot_gradients, float4* gaussian_gradients,
                                  cudaStream_t stream) {
    const unsigned tiles = cam.tiles_x * cam.tiles_y;
    if (mode == SP_BWD_DETERMINISTIC)
        k_blend_backward<SP_BWD_DETERMINISTIC><<<tiles, kTilePixels, 0, stream>>>(
            records, sorted_gaussians, ranges, order, offsets, cam, image, contributions, loss_gradient,
            slot_gradients, gaussian_gradients);
    else
        launch_chained(k_blend_backward_atomic, tiles, kPairThreads, 0, stream, records, sorted_gaussians, ranges, order,
                                                                    cam, image, contributions, loss_gradient,
                                                                    gaussian_gradients);
    return cudaGetLastError();
}

}  // namespace splat

extern "C" sp_status sp_debug_falloff_powers(const float* d_items, uint64_t count, float* d_powers, void* stream) {
    using namespace splat;
    if (count == 0) return SP_OK;
    if (!d_items || !d_powers || (reinterpret_cast<uintptr_t>(d_items) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(d_powers) & 7u) != 0)
        return SP_ERR_INVALID;
    const unsigned blocks = (unsigned)((count + 255) / 256);
    k_falloff_powers<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<const float4*>(d_items),
                                                                             count, reinterpret_cast<float2*>(d_powers));
    return cudaGetLastError() == cudaSuccess ? SP_OK : SP_ERR_CUDA;
}
