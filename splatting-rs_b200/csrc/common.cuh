// Shared device-side declarations of libsplat_b200: record layouts, launch helpers and
// the small warp primitives the kernels use. Written for sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "../../include/splat.h"
#include "../../include/splat_constants.h"
#include "../../include/splat_math.h"

namespace splat {

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device, once per
// device and call site: `done` holds one bit per device, because function attributes are set
// per device and a process may drive several GPUs (devices past 63 are set at every call).
template <typename Kernel>
inline cudaError_t allow_smem_once(Kernel kernel, size_t bytes, std::atomic<unsigned long long>& done) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return err;
    const unsigned long long bit = device < 64 ? 1ull << device : 0ull;
    if (bit && (done.load(std::memory_order_relaxed) & bit)) return cudaSuccess;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err == cudaSuccess) done.fetch_or(bit, std::memory_order_relaxed);
    return err;
}

constexpr int kBlock = 256;                 // threads of every 1-D kernel
constexpr int kTilePixels = SP_TILE * SP_TILE;

// Per-Gaussian blend record written by the projection, 4 float4 (64 B: each record is two
// whole 32-B L2 sectors):
//   [0] mean.x, mean.y, conic.a, conic.b
//   [1] conic.c, opacity, colour.r, colour.g
//   [2] colour.b, depth, tile_min (x | y << 16), tile_max (x | y << 16)  (bit patterns)
//   [3] take_from, clamp_from, 0, 0: the blend's alpha decisions as thresholds on the
//       falloff's power (alpha_thresholds in project.cu): a pixel takes the Gaussian exactly
//       when power >= take_from (opacity * e^power >= 1/255, rasterize_forward.wgsl:66-68)
//       and its alpha is clamped to 0.99 exactly when power >= clamp_from (opacity * e^power
//       >= 0.99); +inf where never.
// The fields of the reference's 80-B `Projected` (common.wgsl:49-61) that the blend and
// binning read, without its padding; the radius lives in its own array. A culled Gaussian
// has an all-zero record and radius 0, as the reference's zeroed `Projected`.
constexpr int kRecord = 4;

// A sorted intersection's value: the Gaussian's index in the low 28 bits and, in the high 4,
// which of the tile's four 8 x 8 pixel blocks (block w at x offset 8 (w & 1), y offset
// 8 (w >> 1)) the Gaussian can reach (tile_cull.cuh, reaches), decided once per key at emission
// so that the blend kernels' warps gather only the records that reach their block. Hence at
// most 2^28 Gaussians.
constexpr uint32_t kGaussianBits = 28;
constexpr uint32_t kGaussianMask = (1u << kGaussianBits) - 1u;

// Device-side bookkeeping of one forward pass (the reference's IntersectionMeta and
// ScanControl, rasterizer.rs:29-44), plus the status word device code raises errors in.
struct DeviceMeta {
    uint32_t count;             // entries in the intersection list: min(total, capacity)
    uint32_t sort_blocks;       // ceil(count / 1024), as the reference reports it
    uint32_t histogram_length;  // 16 * sort_blocks, as the reference reports it
    uint32_t overflow;          // total > capacity
    uint32_t capacity;
    uint32_t partitions;        // sort partitions of this forward pass
    uint32_t status;            // SP_ERR_* raised on the device, 0 when fine
    uint32_t total_hi;          // high word of the uncapped total
    uint32_t total_lo;
    // Compressed keys (SortPlan::compressed): the projection accumulates the range of the
    // visible Gaussians' depth keys (bits(depth) >> 12) in depth_lo / depth_hi; the scan
    // turns it into key = (tile << key_shift) | (depth key - key_base), a key as wide as the
    // frame needs and ordered as the reference's (tile << 20) | depth key.
    uint32_t depth_lo, depth_hi;
    uint32_t key_shift;         // key >> key_shift = tile
    uint32_t key_base;          // depth key of the nearest visible Gaussian
    uint32_t passes;            // sort passes this frame needs (<= SortPlan::passes)
    uint32_t first_buffer;      // the emission's ping-pong buffer, so that the last pass
                                // lands in buffer SortPlan::passes & 1
    // Error-path test switch (sp_debug_stall_sort_partition): partition stall_partition - 1 of
    // every sort pass never posts its look-back record, and waits give up after a short limit;
    // 0 (the default) is off. Set by the host only; no kernel writes it.
    uint32_t stall_partition;
};

// Sort geometry decided on the host from the tile grid.
struct SortPlan {
    int key_bits;      // significant bits of the keys (an upper bound when compressed)
    int key64;         // keys need 64 bits
    int passes;        // ceil(key_bits / 8): the passes launched
    int tile_shift;    // key >> tile_shift = tile index (uncompressed keys)
    int compressed;    // REF20 order in 32-bit keys whose width follows the frame's depth range
    int tile_bits;     // ceil(log2 tiles)
};

// bits(0.01f) >> 12 and the largest depth key (NaN included) a visible Gaussian can have:
// a frame's depth-key range is below 2^19, so compressed keys fit 32 bits up to 2^13 tiles.
constexpr uint32_t kMinDepthKey = 0x3C23Du;
constexpr int kMaxDepthRangeBits = 19;

constexpr int kSortThreads = 256;
constexpr int kSortItems = 24;  // measured best of 8-40 keys per thread and 1-4 blocks per SM
constexpr int kSortBlocksPerSM = 2;
constexpr int kSortPartition = kSortThreads * kSortItems;  // 6144 keys per partition
constexpr int kSortMaxPasses = 8;
constexpr int kSortRadix = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

// Asks the bulk-copy engine to bring [ptr, ptr + bytes) into L2 (cp.async.bulk.prefetch.L2,
// sm_90+): a hint with nothing to wait for. The range must lie inside one allocation; it is
// skipped unless ptr is 16-B aligned, and bytes is rounded down to a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void* ptr, uint32_t bytes) {
    bytes &= ~15u;
    if (bytes == 0 || (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

__device__ __forceinline__ void raise_status(DeviceMeta* meta, uint32_t status) {
    atomicCAS(&meta->status, 0u, status);
}

// Programmatic dependent launch along the training step's chain of kernels (projection, scan,
// emission, sort passes, ranges, tile order, blend forward, SSIM, loss, loss sums, blend
// backward, projection backward). Each of them is launched by launch_chained and calls
// chain_enter first, before any memory access: griddepcontrol.wait returns once the previous
// grid of the stream has completed and its writes are visible (the ordering of a plain launch),
// and launch_dependents then lets the next grid be launched as soon as every block of this one
// has started, so its blocks take the SMs this grid's last wave leaves and the launch latency
// between the two is hidden (config 2: 1014 -> 1040 views/s). A memset, copy or event between
// two launches orders them as usual; a kernel outside the chain is launched plainly.
__device__ __forceinline__ void chain_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Params, typename... Args>
inline cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

inline unsigned grid_for(uint64_t items, unsigned per_block) {
    return (unsigned)((items + per_block - 1) / per_block);
}

}  // namespace splat
