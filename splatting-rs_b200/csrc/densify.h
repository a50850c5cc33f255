// Device densification (densify.cu): the state the plan's kernels share and their launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace splat {

// densify.rs:138-145 (Fate).
enum DensifyFate : uint8_t {
    kDensifyKept = 0,
    kDensifyCloned = 1,
    kDensifySplit = 2,
    kDensifyPrunedTransparent = 3,
    kDensifyPrunedOversized = 4,
};

// How the candidates are taken: all of them (the budget covers them), none (no room), or
// those above the selected key plus the first ties in index order.
enum DensifySelect : uint32_t { kSelectAll = 0, kSelectNone = 1, kSelectByKey = 2 };

// The settings' thresholds as the kernels compare them; the logarithms are computed on the
// host (f32 ln of the reference's f32 operands).
struct DensifyConstants {
    float prune_opacity;
    float max_screen_radius;
    float gradient_threshold;
    float split_log_scale;    // ln(split_scale_fraction * extent)
    float log_split_divisor;  // ln(SPLIT_SCALE_DIVISOR) = ln(1.6)
    float reset_logit;        // logit(RESET_OPACITY) = ln(0.01 / 0.99)
};

// Device-resident state of one plan (zeroed by the plan's first launch).
struct DensifyState {
    unsigned long long kept, candidates, pruned_transparent, pruned_oversized;
    unsigned long long budget;
    uint32_t mode;    // DensifySelect
    uint32_t prefix;  // the selected key, one byte per select pass
    unsigned long long remaining;  // after the last pass: the ties to take, in index order
    unsigned long long histogram[4][256];
    unsigned long long ties;
    unsigned long long copies, news, splits;  // totals (contiguous, in this order)
    sp_densify_report report;
};

// One tile's counts, scanned in place into its exclusive offsets.
struct DensifyTally {
    unsigned long long copies, news, splits, ties;
};

// Tiles (of 1024 Gaussians) the kernels cut n Gaussians into: the length of the tally array.
uint32_t densify_tiles(uint64_t n);

// Classify, select, decide and scan (densify.rs:167-202): fills `state` (report included),
// `fate` (n bytes) and `tallies`; reads `keys` scratch of n words.
cudaError_t launch_densify_plan(const float* params, const float4* stats, uint64_t n, uint32_t stride,
                                const DensifyConstants& c, uint64_t max_count, uint8_t* fate, uint32_t* keys,
                                DensifyTally* tallies, DensifyState* state, uint32_t reset_opacity,
                                cudaStream_t stream);
// densify.rs:204-255 for a plan: writes state->report.after Gaussians and their moments.
cudaError_t launch_densify_write(const float* params, const float* first, const float* second, uint64_t n,
                                 uint32_t sh_degree, const DensifyConstants& c, const uint8_t* fate,
                                 const DensifyTally* tallies, const DensifyState* state, uint64_t seed,
                                 uint32_t reset_opacity, float* out_params, float* out_first, float* out_second,
                                 cudaStream_t stream);

}  // namespace splat
