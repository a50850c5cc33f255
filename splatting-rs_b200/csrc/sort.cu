// Tile binning: key emission (K3), a onesweep LSD radix sort of the (tile, depth) keys
// (K4) and the per-tile ranges (K5).
//
// The order is the reference's: a stable sort of the keys emitted in slot order
// (emit_tile_keys.wgsl:13-36, sort.rs:1-3), so entries with equal keys keep ascending
// Gaussian index. The reference sorts 4 bits a pass over 8 passes with a single-workgroup
// scan between; here each pass moves 8 bits and needs no scan pass: the digit histograms
// of every pass are accumulated while the keys are emitted, and each partition of 4096
// keys finds its output offsets by decoupled look-back on its predecessors (the
// "onesweep" radix sort of Adinets & Merrill, 2022). Passes only cover the significant
// bits of the key (ceil(log2 tiles) + 20).
#include <algorithm>
#include <atomic>

#include <cuda/atomic>

#include "kernels.h"
#include "tile_cull.cuh"

namespace splat {
namespace {

constexpr uint32_t kFlagAggregate = 1u;
constexpr uint32_t kFlagInclusive = 2u;
// Look-back polls that find a predecessor not yet posted before a partition gives up and
// raises SP_ERR_TIMEOUT. Each such poll costs an L2 round trip plus a ~32 ns sleep, so the
// limit is far above any legitimate wait (a predecessor partition takes microseconds) and
// bounds a stuck wait to well under a second.
constexpr uint32_t kLookbackSpinLimit = 1u << 21;
// The limit while the error-path test switch (DeviceMeta::stall_partition) is on.
constexpr uint32_t kLookbackSpinLimitTest = 1u << 12;
constexpr int kLookbackWindow = 8;

// The depth part of a key: the depth's float bits (FULL32), or its 20-bit depth key
// bits >> 12 (the reference's, emit_tile_keys.wgsl:26-29) minus the frame's base (0 unless
// the keys are compressed). The key is (tile << shift) | depth part.
__device__ __forceinline__ uint32_t depth_part(int key_mode, float depth, uint32_t base) {
    const uint32_t bits = __float_as_uint(depth);
    return key_mode == SP_KEYS_FULL32 ? bits : (bits >> (32 - SP_DEPTH_BITS)) - base;
}

template <typename Key>
__device__ __forceinline__ Key compose_key(uint32_t tile, uint32_t shift, uint32_t depth_bits) {
    return (Key)(((unsigned long long)tile << shift) | depth_bits);
}

// Key emission, one warp per 32 Gaussians: the warp's slots are contiguous (the tile
// offsets are an exclusive scan in Gaussian order), so its lanes write them together, key by
// key, whatever the rectangles' sizes: balanced work and coalesced stores. The sort's digit
// histograms are accumulated on the way: per Gaussian (weighted by its tile count) for the
// passes whose digit holds depth bits only, per key for the others.
//
// With CULL the warp walks its rectangles' tile rows 32 at a time: each lane takes one
// (Gaussian, row) and the row's span of reached tiles (tile_cull.cuh, as the projection
// counted them), then the warp writes the 32 rows' keys together; the keys are the
// rectangle's, minus the culled tiles, in the same order.
template <typename Key, bool CULL>
__global__ void __launch_bounds__(kBlock) k_emit(const float4* __restrict__ records, const float4* __restrict__ reach,
                                                 uint32_t* __restrict__ offsets,
                                                 const unsigned long long* __restrict__ block_offsets, uint32_t n,
                                                 uint32_t tiles_x, int key_mode, const DeviceMeta* __restrict__ meta,
                                                 Key* __restrict__ keys0, Key* __restrict__ keys1,
                                                 uint32_t* __restrict__ values0, uint32_t* __restrict__ values1,
                                                 uint32_t* __restrict__ histograms) {
    chain_enter();
    __shared__ uint32_t hist[kSortMaxPasses][kSortRadix];
    const uint32_t t = threadIdx.x, lane = lane_id();
    // This frame's key geometry (k_scan_blocks): the passes it sorts, the tile shift, the
    // depth base, and the ping-pong buffer the keys start in.
    const int passes = (int)meta->passes;
    const uint32_t tile_shift = meta->key_shift, base = meta->key_base;
    Key* __restrict__ keys = meta->first_buffer ? keys1 : keys0;
    uint32_t* __restrict__ values = meta->first_buffer ? values1 : values0;
    for (uint32_t i = t; i < (uint32_t)passes * kSortRadix; i += kBlock) (&hist[0][0])[i] = 0;
    __syncthreads();
    const unsigned long long capacity = meta->capacity;
    const uint32_t g = blockIdx.x * kBlock + t;
    uint32_t x0 = 0, y0 = 0, w = 1, rows = 0, count = 0;
    float depth = 0.0f;
    CullEllipse ellipse{};
    unsigned long long index = 0;
    if (g < n) {
        const float4 r2 = records[(size_t)g * kRecord + 2];
        const uint32_t lo = __float_as_uint(r2.z), hi = __float_as_uint(r2.w);
        x0 = lo & 0xffffu;
        y0 = lo >> 16;
        const uint32_t x1 = hi & 0xffffu, y1 = hi >> 16;
        w = max(x1 - x0, 1u);
        count = (x1 - x0) * (y1 - y0);
        rows = count ? y1 - y0 : 0u;
        if (CULL && count) ellipse = cull_ellipse(records[(size_t)g * kRecord], records[(size_t)g * kRecord + 1]);
        depth = r2.y;
        index = block_offsets[blockIdx.x] + offsets[g];
        offsets[g] = (uint32_t)index;
        // Depth-only digits: the same for every key of the Gaussian (with CULL, per row below).
        const unsigned long long kept = index >= capacity ? 0ull : min((unsigned long long)count, capacity - index);
        if (!CULL && kept) {
            const uint32_t depth_key = depth_part(key_mode, depth, base);
            for (int p = 0; p < passes && 8 * p + 8 <= (int)tile_shift; ++p)
                atomicAdd(&hist[p][(depth_key >> (8 * p)) & 255u], (uint32_t)kept);
        }
    }
    // Exclusive scan over the warp of what it walks: the keys, or with CULL the rows.
    const uint32_t walk = CULL ? rows : count;
    uint32_t inclusive = walk;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t up = __shfl_up_sync(0xffffffffu, inclusive, o);
        if (lane >= (uint32_t)o) inclusive += up;
    }
    const uint32_t exclusive = inclusive - walk;
    const uint32_t total = __shfl_sync(0xffffffffu, inclusive, 31);
    const unsigned long long start = __shfl_sync(0xffffffffu, index, 0);
    const int first_tile_pass = (int)tile_shift / 8;
    // The last lane whose (nondecreasing) exclusive prefix `prefix` is at most e.
    auto holder = [&](uint32_t prefix, uint32_t e) {
        uint32_t h = 0;
#pragma unroll
        for (uint32_t step = 16; step > 0; step >>= 1)
            if (__shfl_sync(0xffffffffu, prefix, h + step) <= e) h += step;
        return h;
    };
    // The key and the value: the Gaussian with the tile's pixel blocks it can reach
    // (common.cuh), given or, without CULL, tested here.
    auto write_key = [&](unsigned long long slot, uint32_t tx, uint32_t ty, float key_depth, uint32_t gaussian,
                         uint32_t blocks) {
        const uint32_t tile = ty * tiles_x + tx;
        const Key key = compose_key<Key>(tile, tile_shift, depth_part(key_mode, key_depth, base));
        keys[slot] = key;
        if (!CULL) {
            const float4* rec = records + (size_t)gaussian * kRecord;
            blocks = block_mask(rec[0], rec[1], reach[gaussian], tx, ty);
        }
        values[slot] = gaussian | (blocks << kGaussianBits);
        for (int p = first_tile_pass; p < passes; ++p) atomicAdd(&hist[p][(uint32_t)(key >> (8 * p)) & 255u], 1u);
    };
    if constexpr (CULL) {
        unsigned long long written = 0;  // keys of the warp's earlier rounds
        for (uint32_t round = 0; round * 32 < total; ++round) {
            // This lane's (Gaussian, row) of the round, and the row's span of tiles.
            const uint32_t p = round * 32 + lane;
            const uint32_t owner = holder(exclusive, p);
            const uint32_t row = __shfl_sync(0xffffffffu, y0, owner) + (p - __shfl_sync(0xffffffffu, exclusive, owner));
            const uint32_t ox0 = __shfl_sync(0xffffffffu, x0, owner), ow = __shfl_sync(0xffffffffu, w, owner);
            const float odepth = __shfl_sync(0xffffffffu, depth, owner);
            const uint32_t og = __shfl_sync(0xffffffffu, g, owner);
            CullEllipse oe;
            oe.mx = __shfl_sync(0xffffffffu, ellipse.mx, owner);
            oe.my = __shfl_sync(0xffffffffu, ellipse.my, owner);
            oe.b = __shfl_sync(0xffffffffu, ellipse.b, owner);
            oe.inv_a = __shfl_sync(0xffffffffu, ellipse.inv_a, owner);
            oe.qa = __shfl_sync(0xffffffffu, ellipse.qa, owner);
            oe.det = __shfl_sync(0xffffffffu, ellipse.det, owner);
            oe.ey = __shfl_sync(0xffffffffu, ellipse.ey, owner);
            oe.stationary = __shfl_sync(0xffffffffu, ellipse.stationary, owner);
            uint2 span = make_uint2(0u, 0u);
            // The ellipse's absolute x-extents over the row's upper and lower 8-pixel bands, from
            // which each key's pixel blocks follow (the blend's 2 x 2 warp blocks of the tile).
            float up_l = INFINITY, up_r = -INFINITY, dn_l = INFINITY, dn_r = -INFINITY;
            if (p < total) {
                span = tile_row_span(oe, row, ox0, ox0 + ow);
                if (!(oe.ey < INFINITY)) {
                    up_l = dn_l = -INFINITY;
                    up_r = dn_r = INFINITY;
                } else if (span.y > span.x) {
                    if (band_extent(oe, row * SP_TILE, SP_TILE / 2, up_l, up_r)) {
                        up_l = __fadd_rn(up_l, oe.mx);
                        up_r = __fadd_rn(up_r, oe.mx);
                    } else {
                        up_l = INFINITY, up_r = -INFINITY;
                    }
                    if (band_extent(oe, row * SP_TILE + SP_TILE / 2, SP_TILE / 2, dn_l, dn_r)) {
                        dn_l = __fadd_rn(dn_l, oe.mx);
                        dn_r = __fadd_rn(dn_r, oe.mx);
                    } else {
                        dn_l = INFINITY, dn_r = -INFINITY;
                    }
                }
            }
            const uint32_t length = span.y - span.x;
            uint32_t row_inclusive = length;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t up = __shfl_up_sync(0xffffffffu, row_inclusive, o);
                if (lane >= (uint32_t)o) row_inclusive += up;
            }
            const uint32_t row_exclusive = row_inclusive - length;
            const uint32_t round_keys = __shfl_sync(0xffffffffu, row_inclusive, 31);
            // Depth-only digits, weighted by the row's keys that fit.
            const unsigned long long row_slot = start + written + row_exclusive;
            const unsigned long long kept =
                row_slot >= capacity ? 0ull : min((unsigned long long)length, capacity - row_slot);
            if (kept) {
                const uint32_t depth_key = depth_part(key_mode, odepth, base);
                for (int q = 0; q < passes && 8 * q + 8 <= (int)tile_shift; ++q)
                    atomicAdd(&hist[q][(depth_key >> (8 * q)) & 255u], (uint32_t)kept);
            }
            // The round's keys, 32 at a time.
            for (uint32_t e0 = 0; e0 < round_keys; e0 += 32) {
                const uint32_t e = e0 + lane;
                const uint32_t src = holder(row_exclusive, e);
                const uint32_t column = __shfl_sync(0xffffffffu, span.x, src) +
                                        (e - __shfl_sync(0xffffffffu, row_exclusive, src));
                const uint32_t key_row = __shfl_sync(0xffffffffu, row, src);
                const float key_depth = __shfl_sync(0xffffffffu, odepth, src);
                const uint32_t key_gaussian = __shfl_sync(0xffffffffu, og, src);
                const float kul = __shfl_sync(0xffffffffu, up_l, src), kur = __shfl_sync(0xffffffffu, up_r, src);
                const float kdl = __shfl_sync(0xffffffffu, dn_l, src), kdr = __shfl_sync(0xffffffffu, dn_r, src);
                const uint32_t blocks = half_columns(kul, kur, column) | (half_columns(kdl, kdr, column) << 2);
                const unsigned long long slot = start + written + e;
                if (e < round_keys && slot < capacity)
                    write_key(slot, column, key_row, key_depth, key_gaussian, blocks);
            }
            written += round_keys;
        }
    } else {
        for (uint32_t round = 0; round * 32 < total; ++round) {
            const uint32_t e = round * 32 + lane;
            const uint32_t owner = holder(exclusive, e);
            const uint32_t local = e - __shfl_sync(0xffffffffu, exclusive, owner);
            const uint32_t ox0 = __shfl_sync(0xffffffffu, x0, owner), oy0 = __shfl_sync(0xffffffffu, y0, owner);
            const uint32_t ow = __shfl_sync(0xffffffffu, w, owner);
            const float odepth = __shfl_sync(0xffffffffu, depth, owner);
            const uint32_t og = __shfl_sync(0xffffffffu, g, owner);
            const uint32_t row = local / ow;
            const unsigned long long slot = start + e;
            if (e < total && slot < capacity)
                write_key(slot, ox0 + (local - row * ow), oy0 + row, odepth, og, 0u);
        }
    }
    __syncthreads();
    for (uint32_t i = t; i < (uint32_t)passes * kSortRadix; i += kBlock) {
        const uint32_t c = (&hist[0][0])[i];
        if (c) atomicAdd(histograms + i, c);
    }
}

// One pass of the onesweep sort. A persistent grid: each block takes partitions of
// kSortPartition keys in ticket order, ranks its keys stably by digit, publishes its digit
// counts, sums its predecessors' (decoupled look-back) and scatters, digit-sorted through
// shared memory so that the global writes of each digit are contiguous.
template <typename Key>
__global__ void __launch_bounds__(kSortThreads, kSortBlocksPerSM)
    k_sort_pass(int pass, uint32_t sequence, Key* keys0, uint32_t* values0, Key* keys1, uint32_t* values1,
                const uint32_t* __restrict__ histogram, uint32_t* ticket, unsigned long long* lookback,
                DeviceMeta* meta) {
    chain_enter();
    // Passes past the ones this frame's keys need do nothing; the others ping-pong from the
    // buffer the emission started in.
    if (pass >= (int)meta->passes) return;
    const int shift = 8 * pass;
    const bool from1 = (meta->first_buffer ^ (uint32_t)pass) & 1u;
    const Key* __restrict__ keys_in = from1 ? keys1 : keys0;
    const uint32_t* __restrict__ values_in = from1 ? values1 : values0;
    Key* __restrict__ keys_out = from1 ? keys0 : keys1;
    uint32_t* __restrict__ values_out = from1 ? values0 : values1;
    extern __shared__ float4 smem4[];
    Key* s_keys = reinterpret_cast<Key*>(smem4);
    uint32_t* s_values = reinterpret_cast<uint32_t*>(s_keys + kSortPartition);
    __shared__ uint32_t s_warp[kSortThreads / 32][kSortRadix];
    __shared__ uint32_t s_global_base[kSortRadix];
    __shared__ uint32_t s_block_start[kSortRadix];
    __shared__ uint32_t s_out_base[kSortRadix];
    __shared__ uint32_t s_scan_warp[kSortThreads / 32];
    __shared__ uint32_t s_partition;

    const uint32_t t = threadIdx.x, lane = lane_id(), warp = t / 32;
    const uint32_t count = meta->count;
    const uint32_t partitions = meta->partitions;
    const uint32_t lanes_below = (1u << lane) - 1u;
    // Error-path test switch: the partition that never posts (none when 0) and the short limit.
    const uint32_t stalled = meta->stall_partition;
    const uint32_t spin_limit = stalled ? kLookbackSpinLimitTest : kLookbackSpinLimit;

    // Exclusive scan over the digits of this pass's global histogram (thread t = digit t).
    auto block_exclusive = [&](uint32_t v) -> uint32_t {
        uint32_t inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t up = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= (uint32_t)o) inc += up;
        }
        if (lane == 31) s_scan_warp[warp] = inc;
        __syncthreads();
        uint32_t before = 0;
#pragma unroll
        for (int w = 0; w < kSortThreads / 32; ++w)
            if ((uint32_t)w < warp) before += s_scan_warp[w];
        __syncthreads();
        return before + inc - v;
    };
    s_global_base[t] = block_exclusive(histogram[t]);

    for (;;) {
        if (t == 0) s_partition = atomicAdd(ticket, 1u);
#pragma unroll
        for (int w = 0; w < kSortThreads / 32; ++w) s_warp[w][t] = 0;
        __syncthreads();
        const uint32_t part = s_partition;
        if (part >= partitions) break;
        const uint32_t base = part * kSortPartition;

        // Load: warp w holds keys [base + 32 kSortItems w, base + 32 kSortItems (w + 1)), item k at lane + 32 k,
        // so (warp, item, lane) order is the keys' original order.
        Key key[kSortItems];
        uint32_t value[kSortItems], digit[kSortItems], rank[kSortItems];
#pragma unroll
        for (int k = 0; k < kSortItems; ++k) {
            const uint32_t i = base + warp * (32 * kSortItems) + k * 32 + lane;
            const bool valid = i < count;
            key[k] = valid ? keys_in[i] : (Key)0;
            value[k] = valid ? values_in[i] : 0u;
            digit[k] = valid ? ((uint32_t)(key[k] >> shift) & 255u) : 0xffffu;
        }
        // Stable rank within the warp, item by item.
#pragma unroll
        for (int k = 0; k < kSortItems; ++k) {
            const uint32_t peers = __match_any_sync(0xffffffffu, digit[k]);
            const bool valid = digit[k] < 256u;
            uint32_t before = 0;
            if (valid) before = s_warp[warp][digit[k]];
            rank[k] = before + __popc(peers & lanes_below);
            __syncwarp();
            if (valid && (__ffs(peers) - 1) == (int)lane) s_warp[warp][digit[k]] = before + __popc(peers);
            __syncwarp();
        }
        __syncthreads();
        // Thread t = digit t: the warps' offsets within the partition and its total.
        uint32_t total = 0;
#pragma unroll
        for (int w = 0; w < kSortThreads / 32; ++w) {
            const uint32_t c = s_warp[w][t];
            s_warp[w][t] = total;
            total += c;
        }
        // Decoupled look-back for digit t.
        {
            cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> mine(
                lookback[(size_t)part * kSortRadix + t]);
            const unsigned long long tag = (unsigned long long)sequence << 32;
            uint32_t prefix = 0;
            const bool posts = stalled == 0 || part != stalled - 1;
            if (part == 0) {
                if (posts)
                    mine.store(tag | ((unsigned long long)kFlagInclusive << 30) | total, cuda::memory_order_relaxed);
            } else {
                if (posts)
                    mine.store(tag | ((unsigned long long)kFlagAggregate << 30) | total, cuda::memory_order_relaxed);
                // Walk back kLookbackWindow predecessors per round trip: read them all, then
                // add in order up to the first inclusive prefix or the first not yet posted.
                uint32_t spins = 0;
                int64_t k = (int64_t)part - 1;
                for (;;) {
                    unsigned long long e[kLookbackWindow];
#pragma unroll
                    for (int w = 0; w < kLookbackWindow; ++w) {
                        e[w] = 0ull;
                        if (k - w >= 0) {
                            cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> other(
                                lookback[(size_t)(k - w) * kSortRadix + t]);
                            e[w] = other.load(cuda::memory_order_relaxed);
                        }
                    }
                    int taken = 0;
                    bool inclusive = false, waiting = false;
#pragma unroll
                    for (int w = 0; w < kLookbackWindow; ++w) {
                        if (inclusive || waiting) continue;
                        const uint32_t flag = (uint32_t)(e[w] >> 30) & 3u;
                        if (k - w < 0 || (uint32_t)(e[w] >> 32) != sequence || flag == 0u) {
                            waiting = true;
                            continue;
                        }
                        prefix += (uint32_t)(e[w] & 0x3fffffffull);
                        ++taken;
                        inclusive = flag == kFlagInclusive;
                    }
                    if (inclusive) break;
                    k -= taken;
                    if (waiting) {
                        if (++spins > spin_limit) {
                            raise_status(meta, SP_ERR_TIMEOUT);
                            break;
                        }
                        __nanosleep(32);
                    }
                }
                if (posts)
                    mine.store(tag | ((unsigned long long)kFlagInclusive << 30) | (prefix + total),
                               cuda::memory_order_relaxed);
            }
            s_out_base[t] = s_global_base[t] + prefix;
        }
        s_block_start[t] = block_exclusive(total);
        __syncthreads();
        // Digit-sorted order in shared memory.
#pragma unroll
        for (int k = 0; k < kSortItems; ++k)
            if (digit[k] < 256u) {
                const uint32_t pos = s_block_start[digit[k]] + s_warp[warp][digit[k]] + rank[k];
                s_keys[pos] = key[k];
                s_values[pos] = value[k];
            }
        __syncthreads();
        const uint32_t valid_here = min((uint32_t)kSortPartition, count - base);
        for (uint32_t i = t; i < valid_here; i += kSortThreads) {
            const Key k = s_keys[i];
            const uint32_t d = (uint32_t)(k >> shift) & 255u;
            const uint32_t dst = s_out_base[d] + (i - s_block_start[d]);
            keys_out[dst] = k;
            values_out[dst] = s_values[i];
        }
        __syncthreads();
    }
}

// tile_ranges.wgsl:9-22 without the zeroed array: each thread takes kRangeItems consecutive
// sorted keys; where the tile changes between two neighbours it writes the end of the one
// and the start of the other, and (0, 0) for the tiles in between, which hold no key (so do
// the tiles before the first key and after the last). Every tile is written exactly once.
constexpr uint32_t kRangeItems = 4;

template <typename Key>
__global__ void __launch_bounds__(kBlock) k_ranges(const Key* __restrict__ keys, const DeviceMeta* __restrict__ meta,
                                                   uint32_t tiles, uint2* __restrict__ ranges) {
    chain_enter();
    // A frame whose sort gave up (a look-back wait ran out) holds keys out of order: its tiles
    // are all left empty, so that the blend kernels read nothing of it.
    const uint32_t count = meta->status != 0 ? 0u : meta->count;
    const uint32_t tile_shift = meta->key_shift;
    const uint32_t threads = gridDim.x * blockDim.x;
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (count == 0) {
        for (uint32_t tile = t; tile < tiles; tile += threads) ranges[tile] = make_uint2(0u, 0u);
        return;
    }
    auto tile_at = [&](uint32_t i) { return min((uint32_t)(keys[i] >> tile_shift), tiles); };
    for (uint32_t i0 = t * kRangeItems; i0 < count; i0 += threads * kRangeItems) {
        // The tile before this thread's first key (`tiles` plays "none" past the end, and the
        // first key's predecessor is tile -1, as an unsigned wrap below).
        uint32_t previous = i0 == 0 ? 0xFFFFFFFFu : tile_at(i0 - 1);
        const uint32_t last = min(i0 + kRangeItems, count);
        for (uint32_t i = i0; i < last; ++i) {
            const uint32_t tile = tile_at(i);
            if (tile != previous) {
                if (previous != 0xFFFFFFFFu && previous < tiles) ranges[previous].y = i;
                if (tile < tiles) ranges[tile].x = i;
                for (uint32_t empty = previous + 1; empty < tile; ++empty) ranges[empty] = make_uint2(0u, 0u);
            }
            previous = tile;
        }
        if (last == count) {
            if (previous < tiles) ranges[previous].y = count;
            for (uint32_t empty = previous + 1; empty < tiles; ++empty) ranges[empty] = make_uint2(0u, 0u);
        }
    }
}

// The persistent grid of the current device (SM count x blocks per SM), looked up once per
// device: a process may drive GPUs of different SM counts.
int sort_grid() {
    constexpr int kDevices = 64;
    static std::atomic<int> grids[kDevices];
    int device = 0;
    cudaGetDevice(&device);
    if (device < 0 || device >= kDevices) device = 0;
    int grid = grids[device].load(std::memory_order_relaxed);
    if (grid == 0) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        grid = (sms > 0 ? sms : 148) * kSortBlocksPerSM;
        grids[device].store(grid, std::memory_order_relaxed);
    }
    return grid;
}

}  // namespace

cudaError_t launch_emit(const float4* records, const float4* reach, uint32_t* offsets,
                        const unsigned long long* block_offsets, uint64_t n,
                        const sp_camera_uniform& cam, int key_mode, int tile_culling, const SortPlan& plan,
                        const DeviceMeta* meta, void* keys0, void* keys1, uint32_t* values0, uint32_t* values1,
                        uint32_t* sort_histograms, cudaStream_t stream) {
    const unsigned grid = grid_for(n, kBlock);
#define SPLAT_EMIT(K, C)                                                                                          \
    launch_chained(k_emit<K, C>, grid, kBlock, 0, stream, records, reach, offsets, block_offsets, (uint32_t)n,         \
                                              cam.tiles_x, key_mode,                                              \
                                              meta, static_cast<K*>(keys0), static_cast<K*>(keys1), values0,      \
                                              values1, sort_histograms)
    if (plan.key64) {
        if (tile_culling) SPLAT_EMIT(unsigned long long, true);
        else SPLAT_EMIT(unsigned long long, false);
    } else {
        if (tile_culling) SPLAT_EMIT(uint32_t, true);
        else SPLAT_EMIT(uint32_t, false);
    }
#undef SPLAT_EMIT
    return cudaGetLastError();
}

cudaError_t launch_sort_pass(const SortPlan& plan, int pass, uint32_t sequence, void* keys0, uint32_t* values0,
                             void* keys1, uint32_t* values1, const uint32_t* sort_histograms, uint32_t* sort_tickets,
                             unsigned long long* lookback, uint32_t max_partitions, DeviceMeta* meta,
                             cudaStream_t stream) {
    const unsigned grid = (unsigned)std::min<int>(sort_grid(), (int)std::max<uint32_t>(max_partitions, 1u));
    const uint32_t* hist = sort_histograms + pass * kSortRadix;
    if (plan.key64) {
        using K = unsigned long long;
        const size_t smem = kSortPartition * (sizeof(K) + sizeof(uint32_t));
        static std::atomic<unsigned long long> configured{0};
        const cudaError_t err = allow_smem_once(k_sort_pass<K>, smem, configured);
        if (err != cudaSuccess) return err;
        launch_chained(k_sort_pass<K>, grid, kSortThreads, smem, stream, pass, sequence, static_cast<K*>(keys0), values0,
                                                             static_cast<K*>(keys1), values1, hist,
                                                             sort_tickets + pass, lookback, meta);
    } else {
        using K = uint32_t;
        const size_t smem = kSortPartition * (sizeof(K) + sizeof(uint32_t));
        static std::atomic<unsigned long long> configured{0};
        const cudaError_t err = allow_smem_once(k_sort_pass<K>, smem, configured);
        if (err != cudaSuccess) return err;
        launch_chained(k_sort_pass<K>, grid, kSortThreads, smem, stream, pass, sequence, static_cast<K*>(keys0), values0,
                                                             static_cast<K*>(keys1), values1, hist,
                                                             sort_tickets + pass, lookback, meta);
    }
    return cudaGetLastError();
}

cudaError_t launch_ranges(const SortPlan& plan, const void* keys, const DeviceMeta* meta, uint64_t capacity,
                          uint2* ranges, uint32_t tiles, cudaStream_t stream) {
    const unsigned grid = (unsigned)std::min<uint64_t>(
        std::max<uint64_t>(grid_for((capacity + kRangeItems - 1) / kRangeItems, kBlock), 1), 148 * 8);
    if (plan.key64)
        launch_chained(k_ranges<unsigned long long>, grid, kBlock, 0, stream, static_cast<const unsigned long long*>(keys), meta,
                                                                   tiles, ranges);
    else
        launch_chained(k_ranges<uint32_t>, grid, kBlock, 0, stream, static_cast<const uint32_t*>(keys), meta, tiles, ranges);
    return cudaGetLastError();
}

}  // namespace splat
