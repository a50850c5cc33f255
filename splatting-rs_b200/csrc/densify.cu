// Adaptive density control on the device: densify (instantsplat-rs/src/densify.rs:147-257)
// over the parameters, Adam's moments and the densify statistics where they already are, so
// that a densification costs a few launches and one small read-back instead of the
// reference's read-back of every buffer and rebuild on the CPU (training.rs:238-266).
//
// The Gaussians are processed in tiles of 1024 (256 threads, four consecutive Gaussians per
// thread, so that in-tile prefix sums follow index order):
//
//   classify    fate (kept / transparent / oversized), candidate flag and the candidate's
//               sort key (f32::total_cmp order of its mean gradient); counts; the key's top
//               byte histogram.
//   select x4   one block: the growth budget, and when it is below the candidate count the
//               budget-th largest key, one byte per pass (a radix select), with the
//               histogram of the next byte between passes. Candidates above the key are
//               taken; of those equal to it, the first ones in index order (the stable sort of
//               densify.rs:192).
//   ties        per tile, the candidates equal to the selected key; scanned.
//   decide      the final fates (clone or split by the largest log scale) and per tile the
//               copies, new Gaussians and splits; scanned, with the report.
//   write       the kept Gaussians with their moments in index order, then the clones' copies
//               and the split children with zero moments; the opacity reset on the way.
//
// Compiled with -fmad=false: the mean gradient, the largest log scale against the split
// threshold and the quaternion arithmetic round as the CPU restatement does. The reference
// evaluates exp, ln and cos in single precision with the host's libm (sigmoid in
// gaussians.rs:87-89, split_child, SplitMix64::standard_normal); here each is the f64 function
// rounded once to f32, which is the correctly rounded single-precision result except within
// about 1e-16 of a rounding boundary, so it agrees with a libm that is itself correctly
// rounded at almost every argument (the split children's positions are compared with a
// tolerance of a few ulps for that reason).
#include <algorithm>

#include "densify.h"

namespace splat {
namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 4;
constexpr int kTile = kThreads * kPerThread;
constexpr uint8_t kCandidateBit = 0x80;
constexpr uint32_t kNone = 0xFFFFFFFFu;

// exp, ln and cos of an f32 argument through the f64 functions, rounded once.
__device__ __forceinline__ float exp_rounded(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log_rounded(float x) { return (float)log((double)x); }
__device__ __forceinline__ float cos_rounded(float x) { return (float)cos((double)x); }

// gaussians.rs:87-89.
__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + exp_rounded(-x)); }

__device__ __forceinline__ uint32_t total_order_key(float value) {
    const uint32_t bits = __float_as_uint(value);
    return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

__device__ __forceinline__ unsigned long long warp_inclusive(unsigned long long v) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const unsigned long long u = __shfl_up_sync(0xFFFFFFFFu, v, d);
        if ((threadIdx.x & 31u) >= (uint32_t)d) v += u;
    }
    return v;
}

// Exclusive prefix over the block's threads (kThreads) of `v`; `total` gets the block sum.
// Every thread must call it.
__device__ __forceinline__ unsigned long long block_exclusive(unsigned long long v, unsigned long long* scratch,
                                                              unsigned long long& total) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const unsigned long long inclusive = warp_inclusive(v);
    if (lane == 31) scratch[warp] = inclusive;
    __syncthreads();
    if (warp == 0) {
        const unsigned long long w = lane < kThreads / 32 ? scratch[lane] : 0ull;
        const unsigned long long wi = warp_inclusive(w);
        if (lane < kThreads / 32) scratch[kThreads / 32 + lane] = wi - w;
        if (lane == kThreads / 32 - 1) scratch[2 * (kThreads / 32)] = wi;
    }
    __syncthreads();
    const unsigned long long out = scratch[kThreads / 32 + warp] + inclusive - v;
    total = scratch[2 * (kThreads / 32)];
    __syncthreads();
    return out;
}

__device__ __forceinline__ float mean_gradient(const float4& stat) {
    return stat.y > 0.0f ? __fdiv_rn(stat.x, stat.y) : 0.0f;  // densify.rs:181-188
}

__global__ void __launch_bounds__(kThreads) k_classify(const float* __restrict__ params,
                                                       const float4* __restrict__ stats, uint64_t n, uint32_t stride,
                                                       DensifyConstants c, uint8_t* __restrict__ fate,
                                                       uint32_t* __restrict__ keys, DensifyState* state) {
    __shared__ uint32_t histogram[256];
    __shared__ unsigned long long scratch[2 * (kThreads / 32) + 1];
    for (int i = threadIdx.x; i < 256; i += kThreads) histogram[i] = 0;
    __syncthreads();
    const uint64_t g0 = (uint64_t)blockIdx.x * kTile + (uint64_t)threadIdx.x * kPerThread;
    uint32_t kept = 0, candidates = 0, transparent = 0, oversized = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        const uint64_t g = g0 + j;
        if (g >= n) break;
        const float4 stat = stats[g];
        uint8_t f;
        uint32_t key = 0;
        // densify.rs:169-180.
        if (sigmoid(params[g * stride + SP_SLOT_OPACITY]) < c.prune_opacity) {
            f = kDensifyPrunedTransparent;
            ++transparent;
        } else if (stat.z >= c.max_screen_radius) {
            f = kDensifyPrunedOversized;
            ++oversized;
        } else {
            f = kDensifyKept;
            ++kept;
            const float mg = mean_gradient(stat);
            if (mg > c.gradient_threshold) {
                f |= kCandidateBit;
                key = total_order_key(mg);
                ++candidates;
                atomicAdd(&histogram[key >> 24], 1u);
            }
        }
        fate[g] = f;
        keys[g] = key;
    }
    unsigned long long total;
    block_exclusive(kept, scratch, total);
    if (threadIdx.x == 0) atomicAdd(&state->kept, total);
    block_exclusive(candidates, scratch, total);
    if (threadIdx.x == 0) atomicAdd(&state->candidates, total);
    block_exclusive(transparent, scratch, total);
    if (threadIdx.x == 0) atomicAdd(&state->pruned_transparent, total);
    block_exclusive(oversized, scratch, total);
    if (threadIdx.x == 0) atomicAdd(&state->pruned_oversized, total);
    for (int i = threadIdx.x; i < 256; i += kThreads)
        if (histogram[i]) atomicAdd(&state->histogram[0][i], (unsigned long long)histogram[i]);
}

// One byte of the radix select (pass 0: the top byte). One block of 256 threads.
__global__ void __launch_bounds__(kThreads) k_select(DensifyState* state, uint64_t max_count, int pass) {
    __shared__ unsigned long long scratch[2 * (kThreads / 32) + 1];
    if (pass == 0) {
        if (threadIdx.x == 0) {
            // densify.rs:193-195: clones and splits each add one Gaussian.
            const unsigned long long room = max_count > state->kept ? max_count - state->kept : 0ull;
            const unsigned long long budget = room < state->candidates ? room : state->candidates;
            state->budget = budget;
            state->mode = budget == state->candidates ? kSelectAll : (budget == 0 ? kSelectNone : kSelectByKey);
            state->remaining = budget;
            state->prefix = 0;
        }
        __syncthreads();
    }
    if (state->mode != kSelectByKey) return;
    // Thread t holds digit 255 - t: the inclusive prefix counts the keys at or above it.
    const uint32_t digit = 255u - threadIdx.x;
    const unsigned long long count = state->histogram[pass][digit];
    unsigned long long total;
    const unsigned long long above = block_exclusive(count, scratch, total);
    const unsigned long long remaining = state->remaining;
    __syncthreads();
    // The digit where the count from the top first reaches the remaining budget.
    if (above < remaining && above + count >= remaining) {
        state->prefix |= digit << (24 - 8 * pass);
        state->remaining = remaining - above;
    }
}

// The next byte's histogram of the candidates whose higher bytes equal the selected prefix.
__global__ void __launch_bounds__(kThreads) k_histogram(const uint8_t* __restrict__ fate,
                                                        const uint32_t* __restrict__ keys, uint64_t n,
                                                        DensifyState* state, int pass) {
    if (state->mode != kSelectByKey) return;
    __shared__ uint32_t histogram[256];
    for (int i = threadIdx.x; i < 256; i += kThreads) histogram[i] = 0;
    __syncthreads();
    const int shift = 32 - 8 * pass;  // bits above the byte this pass counts
    const uint32_t prefix = state->prefix >> shift;
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (uint64_t)gridDim.x * blockDim.x) {
        if (!(fate[g] & kCandidateBit)) continue;
        const uint32_t key = keys[g];
        if ((key >> shift) == prefix) atomicAdd(&histogram[(key >> (shift - 8)) & 255u], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += kThreads)
        if (histogram[i]) atomicAdd(&state->histogram[pass][i], (unsigned long long)histogram[i]);
}

// Per tile: the candidates whose key equals the selected one (index order decides among them).
__global__ void __launch_bounds__(kThreads) k_ties(const uint8_t* __restrict__ fate, const uint32_t* __restrict__ keys,
                                                   uint64_t n, const DensifyState* state, DensifyTally* tallies) {
    __shared__ unsigned long long scratch[2 * (kThreads / 32) + 1];
    const bool by_key = state->mode == kSelectByKey;
    const uint32_t threshold = state->prefix;
    const uint64_t g0 = (uint64_t)blockIdx.x * kTile + (uint64_t)threadIdx.x * kPerThread;
    uint32_t ties = 0;
    if (by_key) {
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
            const uint64_t g = g0 + j;
            if (g < n && (fate[g] & kCandidateBit) && keys[g] == threshold) ++ties;
        }
    }
    unsigned long long total;
    block_exclusive(ties, scratch, total);
    if (threadIdx.x == 0) tallies[blockIdx.x].ties = total;
}

// Exclusive scan of the tiles' tallies in place (one block): `which` 0 scans the ties, 1 the
// copies, new Gaussians and splits, and then fills the report.
__global__ void __launch_bounds__(1024) k_scan_tallies(DensifyTally* tallies, uint32_t tiles, DensifyState* state,
                                                       int which, uint64_t n, uint32_t reset_opacity) {
    constexpr int kScanThreads = 1024;
    __shared__ unsigned long long warp_totals[3][kScanThreads / 32];
    const uint32_t per = (tiles + kScanThreads - 1) / kScanThreads;
    const uint32_t first = threadIdx.x * per;
    const uint32_t last = min(first + per, tiles);
    unsigned long long sum[3] = {0, 0, 0};
    for (uint32_t i = first; i < last; ++i) {
        if (which == 0) {
            sum[0] += tallies[i].ties;
        } else {
            sum[0] += tallies[i].copies;
            sum[1] += tallies[i].news;
            sum[2] += tallies[i].splits;
        }
    }
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    unsigned long long base[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const unsigned long long inclusive = warp_inclusive(sum[k]);
        if (lane == 31) warp_totals[k][warp] = inclusive;
        base[k] = inclusive - sum[k];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const unsigned long long w = warp_totals[k][lane];
            const unsigned long long wi = warp_inclusive(w);
            warp_totals[k][lane] = wi - w;
            if (lane == 31) {
                if (which == 0 && k == 0) state->ties = wi;
                if (which == 1) (&state->copies)[k] = wi;
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 3; ++k) base[k] += warp_totals[k][warp];
    for (uint32_t i = first; i < last; ++i) {
        if (which == 0) {
            const unsigned long long t = tallies[i].ties;
            tallies[i].ties = base[0];
            base[0] += t;
        } else {
            const unsigned long long c = tallies[i].copies, w = tallies[i].news, s = tallies[i].splits;
            tallies[i].copies = base[0];
            tallies[i].news = base[1];
            tallies[i].splits = base[2];
            base[0] += c;
            base[1] += w;
            base[2] += s;
        }
    }
    if (which == 1) {
        __syncthreads();
        if (threadIdx.x == 0) {
            sp_densify_report& r = state->report;
            r.before = n;
            r.split = state->splits;
            r.cloned = state->news - 2 * state->splits;
            r.pruned_transparent = state->pruned_transparent;
            r.pruned_oversized = state->pruned_oversized;
            r.over_budget = state->candidates - state->budget;
            r.after = state->copies + state->news;
            r.opacity_reset = reset_opacity;
        }
    }
}

// The final fates and per tile the copies (kept or cloned), new Gaussians (one per clone, two
// per split) and splits.
__global__ void __launch_bounds__(kThreads) k_decide(const float* __restrict__ params, uint64_t n, uint32_t stride,
                                                     DensifyConstants c, uint8_t* __restrict__ fate,
                                                     const uint32_t* __restrict__ keys, const DensifyState* state,
                                                     DensifyTally* tallies) {
    __shared__ unsigned long long scratch[2 * (kThreads / 32) + 1];
    const uint32_t mode = state->mode;
    const uint32_t threshold = state->prefix;
    const unsigned long long ties_taken = state->remaining;
    const uint64_t g0 = (uint64_t)blockIdx.x * kTile + (uint64_t)threadIdx.x * kPerThread;
    uint8_t f[kPerThread];
    uint32_t ties = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        const uint64_t g = g0 + j;
        f[j] = g < n ? fate[g] : (uint8_t)kDensifyPrunedTransparent;
        if (mode == kSelectByKey && (f[j] & kCandidateBit) && keys[g] == threshold) ++ties;
    }
    unsigned long long total;
    unsigned long long tie_rank = block_exclusive(ties, scratch, total);
    if (mode == kSelectByKey) tie_rank += tallies[blockIdx.x].ties;
    uint32_t copies = 0, news = 0, splits = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        const uint64_t g = g0 + j;
        if (g >= n) break;
        uint8_t out = f[j] & (uint8_t)~kCandidateBit;
        if (f[j] & kCandidateBit) {
            bool taken = mode == kSelectAll;
            if (mode == kSelectByKey) {
                const uint32_t key = keys[g];
                if (key > threshold) {
                    taken = true;
                } else if (key == threshold) {
                    taken = tie_rank < ties_taken;
                    ++tie_rank;
                }
            }
            if (taken) {
                // densify.rs:196-202: split when the largest log scale is above the threshold.
                const float* ls = params + g * stride + SP_SLOT_LOG_SCALE;
                const float largest = fmaxf(fmaxf(fmaxf(-INFINITY, ls[0]), ls[1]), ls[2]);
                out = largest > c.split_log_scale ? kDensifySplit : kDensifyCloned;
            }
        }
        fate[g] = out;
        copies += out == kDensifyKept || out == kDensifyCloned;
        news += out == kDensifyCloned ? 1u : (out == kDensifySplit ? 2u : 0u);
        splits += out == kDensifySplit;
    }
    block_exclusive(copies, scratch, total);
    if (threadIdx.x == 0) tallies[blockIdx.x].copies = total;
    block_exclusive(news, scratch, total);
    if (threadIdx.x == 0) tallies[blockIdx.x].news = total;
    block_exclusive(splits, scratch, total);
    if (threadIdx.x == 0) tallies[blockIdx.x].splits = total;
}

// SplitMix64 (densify.rs:275-297): the (index + 1)-th draw of the stream seeded with `seed`.
__device__ __forceinline__ uint64_t splitmix64(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1) * 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float uniform_of(uint64_t draw) {
    return ((float)(draw >> 40) + 1.0f) / 16777216.0f;  // (0, 1]
}

// split_child (densify.rs:259-273), positions and log scales only: `out` gets child floats 0..5.
__device__ void split_child_head(const float* gaussian, uint64_t seed, uint64_t index, float log_divisor,
                                 float out[6]) {
    float local[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float scale = exp_rounded(gaussian[3 + k]);
        const float u = uniform_of(splitmix64(seed, index + 2 * k));
        const float v = uniform_of(splitmix64(seed, index + 2 * k + 1));
        const float normal = __fsqrt_rn(-2.0f * log_rounded(u)) * cos_rounded(6.28318530717958647692f * v);
        local[k] = scale * normal;
    }
    // The quaternion (w, x, y, z) normalised as nalgebra's UnitQuaternion (norm of (x, y, z, w)
    // summed as (x^2 + z^2) + (y^2 + w^2)), then v + t w + q x t with t = 2 (q x v).
    const float w0 = gaussian[6], x0 = gaussian[7], y0 = gaussian[8], z0 = gaussian[9];
    const float norm = __fsqrt_rn((x0 * x0 + z0 * z0) + (y0 * y0 + w0 * w0));
    const float w = __fdiv_rn(w0, norm), qx = __fdiv_rn(x0, norm), qy = __fdiv_rn(y0, norm), qz = __fdiv_rn(z0, norm);
    const float t0 = 2.0f * (qy * local[2] - qz * local[1]);
    const float t1 = 2.0f * (qz * local[0] - qx * local[2]);
    const float t2 = 2.0f * (qx * local[1] - qy * local[0]);
    const float c0 = qy * t2 - qz * t1, c1 = qz * t0 - qx * t2, c2 = qx * t1 - qy * t0;
    out[0] = gaussian[0] + (t0 * w + c0 + local[0]);
    out[1] = gaussian[1] + (t1 * w + c1 + local[1]);
    out[2] = gaussian[2] + (t2 * w + c2 + local[2]);
#pragma unroll
    for (int k = 0; k < 3; ++k) out[3 + k] = gaussian[3 + k] - log_divisor;
}

template <int S>
__global__ void __launch_bounds__(kThreads) k_write(const float* __restrict__ params, const float* __restrict__ m1,
                                                    const float* __restrict__ m2, uint64_t n, DensifyConstants c,
                                                    const uint8_t* __restrict__ fate, const DensifyTally* tallies,
                                                    const DensifyState* state, uint64_t seed, uint32_t reset_opacity,
                                                    float* __restrict__ out_params, float* __restrict__ out_m1,
                                                    float* __restrict__ out_m2) {
    __shared__ unsigned long long scratch[2 * (kThreads / 32) + 1];
    __shared__ uint32_t copy_row[kTile];  // output row of the Gaussian's copy, relative to copy_base
    __shared__ uint32_t new_row[kTile];   // output row of its first new Gaussian, relative to new_base
    __shared__ uint8_t fates[kTile];
    const uint64_t tile0 = (uint64_t)blockIdx.x * kTile;
    const uint32_t here = (uint32_t)(n - tile0 < (uint64_t)kTile ? n - tile0 : (uint64_t)kTile);
    const DensifyTally base = tallies[blockIdx.x];
    const unsigned long long copy_base = base.copies;
    const unsigned long long new_base = state->copies + base.news;
    uint32_t copies = 0, news = 0, splits = 0;
    uint8_t f[kPerThread];
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        const uint32_t i = threadIdx.x * kPerThread + j;
        f[j] = i < here ? fate[tile0 + i] : (uint8_t)kDensifyPrunedTransparent;
        copies += f[j] == kDensifyKept || f[j] == kDensifyCloned;
        news += f[j] == kDensifyCloned ? 1u : (f[j] == kDensifySplit ? 2u : 0u);
        splits += f[j] == kDensifySplit;
    }
    unsigned long long total;
    uint32_t copy_at = (uint32_t)block_exclusive(copies, scratch, total);
    uint32_t new_at = (uint32_t)block_exclusive(news, scratch, total);
    unsigned long long split_at = base.splits + block_exclusive(splits, scratch, total);
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        const uint32_t i = threadIdx.x * kPerThread + j;
        if (i >= here) break;
        fates[i] = f[j];
        copy_row[i] = kNone;
        new_row[i] = kNone;
        if (f[j] == kDensifyKept || f[j] == kDensifyCloned) copy_row[i] = copy_at++;
        if (f[j] == kDensifyCloned) {
            new_row[i] = new_at++;
        } else if (f[j] == kDensifySplit) {
            new_row[i] = new_at;
            // The children's positions and log scales; the rest of their rows below.
            const float* gaussian = params + (tile0 + i) * S;
            for (int child = 0; child < 2; ++child) {
                float head[6];
                split_child_head(gaussian, seed, split_at * 12 + child * 6, c.log_split_divisor, head);
                float* row = out_params + (new_base + new_at + child) * S;
#pragma unroll
                for (int k = 0; k < 6; ++k) row[k] = head[k];
            }
            new_at += 2;
            ++split_at;
        }
    }
    __syncthreads();
    // The rows, coalesced: consecutive threads take consecutive floats of the tile.
    const float reset_logit = c.reset_logit;
    for (uint32_t e = threadIdx.x; e < here * S; e += kThreads) {
        const uint32_t i = e / S, k = e - i * S;
        const uint8_t fi = fates[i];
        if (fi == kDensifyPrunedTransparent || fi == kDensifyPrunedOversized) continue;
        const uint64_t src = (tile0 + i) * S + k;
        float p = params[src];
        const bool reset_slot = reset_opacity && k == SP_SLOT_OPACITY;
        if (reset_slot) p = fminf(p, reset_logit);  // f32::min
        if (copy_row[i] != kNone) {
            const uint64_t dst = (copy_base + copy_row[i]) * S + k;
            out_params[dst] = p;
            out_m1[dst] = reset_slot ? 0.0f : m1[src];
            out_m2[dst] = reset_slot ? 0.0f : m2[src];
        }
        if (new_row[i] != kNone) {
            const int rows = fi == kDensifySplit ? 2 : 1;
            for (int r = 0; r < rows; ++r) {
                const uint64_t dst = (new_base + new_row[i] + r) * S + k;
                if (fi != kDensifySplit || k >= 6) out_params[dst] = p;
                out_m1[dst] = 0.0f;
                out_m2[dst] = 0.0f;
            }
        }
    }
}

uint32_t tiles_of(uint64_t n) { return (uint32_t)((n + kTile - 1) / kTile); }

}  // namespace

uint32_t densify_tiles(uint64_t n) { return tiles_of(n); }

cudaError_t launch_densify_plan(const float* params, const float4* stats, uint64_t n, uint32_t stride,
                                const DensifyConstants& c, uint64_t max_count, uint8_t* fate, uint32_t* keys,
                                DensifyTally* tallies, DensifyState* state, uint32_t reset_opacity,
                                cudaStream_t stream) {
    const uint32_t tiles = tiles_of(n);
    cudaError_t err = cudaMemsetAsync(state, 0, sizeof(DensifyState), stream);
    if (err != cudaSuccess) return err;
    k_classify<<<tiles, kThreads, 0, stream>>>(params, stats, n, stride, c, fate, keys, state);
    k_select<<<1, kThreads, 0, stream>>>(state, max_count, 0);
    const uint32_t grid = (uint32_t)std::min<uint64_t>((n + kThreads - 1) / kThreads, 148u * 8u);
    for (int pass = 1; pass < 4; ++pass) {
        k_histogram<<<grid, kThreads, 0, stream>>>(fate, keys, n, state, pass);
        k_select<<<1, kThreads, 0, stream>>>(state, max_count, pass);
    }
    k_ties<<<tiles, kThreads, 0, stream>>>(fate, keys, n, state, tallies);
    k_scan_tallies<<<1, 1024, 0, stream>>>(tallies, tiles, state, 0, n, reset_opacity);
    k_decide<<<tiles, kThreads, 0, stream>>>(params, n, stride, c, fate, keys, state, tallies);
    k_scan_tallies<<<1, 1024, 0, stream>>>(tallies, tiles, state, 1, n, reset_opacity);
    return cudaGetLastError();
}

cudaError_t launch_densify_write(const float* params, const float* first, const float* second, uint64_t n,
                                 uint32_t sh_degree, const DensifyConstants& c, const uint8_t* fate,
                                 const DensifyTally* tallies, const DensifyState* state, uint64_t seed,
                                 uint32_t reset_opacity, float* out_params, float* out_first, float* out_second,
                                 cudaStream_t stream) {
    const uint32_t tiles = tiles_of(n);
#define SP_DENSIFY_WRITE(D)                                                                                     \
    k_write<SP_PARAM_STRIDE(D)><<<tiles, kThreads, 0, stream>>>(params, first, second, n, c, fate, tallies, state, \
                                                               seed, reset_opacity, out_params, out_first,     \
                                                               out_second)
    switch (sh_degree) {
        case 0: SP_DENSIFY_WRITE(0); break;
        case 1: SP_DENSIFY_WRITE(1); break;
        case 2: SP_DENSIFY_WRITE(2); break;
        case 3: SP_DENSIFY_WRITE(3); break;
        default: return cudaErrorInvalidValue;
    }
#undef SP_DENSIFY_WRITE
    return cudaGetLastError();
}

}  // namespace splat
