// Host-side launchers of the kernels of libsplat_b200 (one .cu file each group). The
// C ABI (api.cu) calls only these. Every launcher enqueues on `stream` and returns the
// launch error, if any.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace splat {

// ---- project.cu (compiled with -fmad=false: the tile decisions match the oracle's bits)

// project_forward.wgsl:19-93 with the scan's first level (scan.wgsl:27-62) fused: per
// block of 256 Gaussians the exclusive prefix of the tile counts and the block total.
// The camera is `cam`, or when `cam_device` is non-null the 80 B there (written on the device).
// With `depth_range` non-null (compressed keys) the depth keys' range of the Gaussians that
// emit keys is accumulated into its depth_lo / depth_hi.
// With `tile_culling` the tile counts are those of tile_cull.cuh (the rectangle's tiles the
// ellipse reaches) instead of the rectangle's area.
cudaError_t launch_project(const float* params, uint64_t n, int sh_degree, const sp_camera_uniform& cam,
                           const sp_camera_uniform* cam_device, float4* records, uint32_t* radii,
                           uint32_t* local_offsets, uint32_t* block_totals, DeviceMeta* depth_range,
                           float4* reach, int tile_culling, cudaStream_t stream);
// scan_tile_counts (scan.wgsl:64-81): scans the block totals into 64-bit block offsets,
// fills the meta (count, overflow, sort partitions, this frame's key geometry) and zeroes
// the sort's histograms and partition tickets for this forward pass.
cudaError_t launch_scan_blocks(const uint32_t* block_totals, unsigned long long* block_offsets, uint32_t blocks,
                               uint64_t capacity, DeviceMeta* meta, uint32_t* sort_histograms, uint32_t* sort_tickets,
                               const SortPlan& plan, cudaStream_t stream);
// project_backward.wgsl:30-227 + reduce_camera_gradient.wgsl:10-34, fused (last block
// done). Blend sums come per Gaussian (atomic mode) or per slot (deterministic mode).
// One Adam step for the projection backward to apply in place of writing the parameter
// gradients (the parameters are the projection's own).
struct AdamLaunch {
    float* params;
    float* first_moment;
    float* second_moment;
    const float* lr_by_slot;  // host, one rate per parameter slot
    float bias1, bias2, max_log_scale, max_log_anisotropy;
};
// project_backward.wgsl plus reduce_camera_gradient.wgsl over the Gaussians
// [first, first + count) (first a multiple of 256; ranges that cover all n, launched in order
// on one stream, the last block of all reducing the camera gradient); with `adam` non-null
// the parameter gradients are not written but consumed by that Adam step (adam.wgsl,
// clamp_scales.wgsl) in the same kernel.
cudaError_t launch_project_backward(const float* params, uint64_t n, int sh_degree, int mode,
                                    const sp_camera_uniform& cam, const sp_camera_uniform* cam_device,
                                    const float4* records, const uint32_t* radii, const uint32_t* offsets,
                                    const float* slot_gradients, uint64_t capacity, const float4* gaussian_gradients,
                                    float* param_gradients, int accumulate, float* camera_partials,
                                    uint32_t* camera_done, float* camera_gradient, float4* densify_stats,
                                    const AdamLaunch* adam, uint64_t first, uint64_t count, cudaStream_t stream);
// The reference's 80-B Projected records (diagnostics).
cudaError_t launch_to_projected(const float4* records, const uint32_t* radii, uint64_t n, sp_projected* out,
                                cudaStream_t stream);

// ---- sort.cu

// emit_tile_keys.wgsl:13-36: adds the block offsets into the tile offsets, writes one key
// and value per covered tile (the Gaussian index with its block bits, common.cuh; `reach`:
// the projection's culling constants), and accumulates every sort pass's digit histogram.
// Keys and values go to ping-pong buffer meta->first_buffer, so that the frame's last sort
// pass lands in buffer plan.passes & 1.
// With `tile_culling`, only the tiles of tile_cull.cuh get keys (the counts of launch_project
// with the same flag).
cudaError_t launch_emit(const float4* records, const float4* reach, uint32_t* offsets,
                        const unsigned long long* block_offsets, uint64_t n,
                        const sp_camera_uniform& cam, int key_mode, int tile_culling, const SortPlan& plan,
                        const DeviceMeta* meta, void* keys0, void* keys1, uint32_t* values0, uint32_t* values1,
                        uint32_t* sort_histograms, cudaStream_t stream);
// One onesweep pass (stable, 8-bit digit `pass`) between the two ping-pong buffers; a pass at
// or past the frame's meta->passes does nothing.
cudaError_t launch_sort_pass(const SortPlan& plan, int pass, uint32_t sequence, void* keys0, uint32_t* values0,
                             void* keys1, uint32_t* values1, const uint32_t* sort_histograms, uint32_t* sort_tickets,
                             unsigned long long* lookback, uint32_t max_partitions, DeviceMeta* meta,
                             cudaStream_t stream);
// tile_ranges.wgsl:9-22: every tile's [start, end) in the sorted keys, (0, 0) for tiles
// without keys (the reference zeroes the array first; here each tile is written once).
cudaError_t launch_ranges(const SortPlan& plan, const void* keys, const DeviceMeta* meta, uint64_t capacity,
                          uint2* ranges, uint32_t tiles, cudaStream_t stream);

// ---- blend.cu

// The blend kernels' schedule: the tiles in decreasing order of list length (to a quarter
// octave), so that the longest tiles start first and the short ones fill the last wave.
cudaError_t launch_tile_order(const uint2* ranges, uint32_t tiles, uint32_t* order, cudaStream_t stream);
// rasterize_forward.wgsl:22-88; block b blends tile order[b].
cudaError_t launch_blend_forward(const float4* records, const uint32_t* sorted_gaussians, const uint2* ranges,
                                 const uint32_t* order, const sp_camera_uniform& cam, float4* image,
                                 uint32_t* contributions, cudaStream_t stream);
// rasterize_backward.wgsl:30-133. mode SP_BWD_*: slot sums (deterministic) or atomics
// into gaussian_gradients (3 float4 per Gaussian, zeroed by the caller).
cudaError_t launch_blend_backward(int mode, const float4* records, const uint32_t* sorted_gaussians,
                                  const uint2* ranges, const uint32_t* order, const uint32_t* offsets,
                                  const sp_camera_uniform& cam, const float4* image, const uint32_t* contributions,
                                  const float4* loss_gradient, float* slot_gradients, float4* gaussian_gradients,
                                  cudaStream_t stream);

// The work the blend kernels do for the current state: counts[0] += entries the forward
// visits per pixel (through the terminating one), counts[1] += contributors per pixel.
cudaError_t launch_count_blend(const float4* records, const uint32_t* sorted_gaussians, const uint2* ranges,
                               const sp_camera_uniform& cam, const uint32_t* contributions,
                               unsigned long long* counts, cudaStream_t stream);

// ---- loss.cu

// ssim_forward.wgsl:34-91 (separable window sums in shared memory).
cudaError_t launch_ssim(const float4* image, const float4* ground_truth, uint32_t width, uint32_t height,
                        float4* partials, cudaStream_t stream);
// loss.wgsl:35-97. When `clear` is given it also zeroes its first `clear_count` float4s (the
// atomic backward's blend sums for this view).
cudaError_t launch_loss(const float4* image, const float4* ground_truth, const float4* partials, uint32_t width,
                        uint32_t height, const sp_loss_weights& weights, float4* loss_gradient, float4* pixel_loss,
                        float4* clear, uint64_t clear_count, cudaStream_t stream);

// ---- adam.cu

// adam.wgsl:20-37 + clamp_scales.wgsl:15-29, fused, over Gaussians [first, first + count).
cudaError_t launch_adam(float* params, const float* gradients, float* first_moment, float* second_moment,
                        uint64_t first, uint64_t count, int stride, const float* lr_by_slot_host, float bias1,
                        float bias2, float max_log_scale, float max_log_anisotropy, cudaStream_t stream);

// The peer-memory exchange with Adam (sp_peer_exchange_step): per Gaussian of this rank's
// share [first, first + count), the gradients summed over the ranks' buffers in rank order
// (peer loads), the Adam step and scale clamp on this rank's parameters and moments, and the
// updated parameters stored into every rank's parameter buffer (peer stores).
constexpr int kMaxPeers = 8;
struct PeerBuffers {
    const float* gradients[kMaxPeers];
    float* params[kMaxPeers];
    uint32_t world, rank;
};
cudaError_t launch_adam_peer(const PeerBuffers& peers, float* first_moment, float* second_moment, uint64_t first,
                             uint64_t count, int stride, const float* lr_by_slot_host, float bias1, float bias2,
                             float max_log_scale, float max_log_anisotropy, cudaStream_t stream);

// Reads `count` float4 of `src` (another GPU's memory mapped into this one) with `blocks`
// blocks and stores one sum per block into sink[blocks]: the peer-read probe of the exchange.
cudaError_t launch_peer_read(const float4* src, uint64_t count, float4* sink, unsigned blocks, cudaStream_t stream);

// ---- pose_device.cu

namespace pose {
struct ViewState;
struct SharedState;
}  // namespace pose
// The device pose refinement: if view < views, the refinement step of `view` from the
// camera gradient (14 floats); then, if next_view < views, the camera uniform of next_view
// into camera_out. One thread.
cudaError_t launch_pose_step(const sp_pinhole_camera* initial, pose::ViewState* states, pose::SharedState* shared,
                             const float* camera_gradient, uint32_t views, uint32_t view, uint32_t next_view,
                             double factor, sp_camera_uniform* camera_out, cudaStream_t stream);

}  // namespace splat
