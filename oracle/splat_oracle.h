/* CPU oracle of the differentiable Gaussian-splatting path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain C++ restatement of the reference's WGSL kernels and Rust host arithmetic
 * (the .wgsl files of instantsplat-rs/src/shaders, optimizer.rs, prune.rs, loss.rs), each function
 * citing the file:line it follows. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it, as the checker or as the timed CPU
 * baseline; the product path (libsplat_b200.so) never calls it.
 *
 * Parity status: the reference is Rust + WGSL on wgpu (Metal/WebGPU only) and cannot be
 * built or run here, so this restatement is pinned by the known-answer tests the
 * reference's own tests hold (tests/golden/reference_known_answers.json), by
 * finite-difference checks, and by an independent per-pixel f64 renderer — not by
 * outputs of the reference itself.
 *
 * The arithmetic that decides tile lists (projection to depth, radius and tile rectangle)
 * uses the same operation order and the same exp (include/splat_math.h) as the CUDA
 * kernels, so tile lists and sort order are comparable bit for bit.
 */
#ifndef SPLAT_ORACLE_H
#define SPLAT_ORACLE_H

#include <stdint.h>

#include "../include/splat.h"

#ifdef __cplusplus
extern "C" {
#endif

/* project_forward.wgsl:19-93 (+ SH degree 1-3 colour). counts: tiles per Gaussian. */
void or_project(const float* params, uint64_t n, uint32_t sh_degree, const sp_camera_uniform* cam,
                sp_projected* out, uint32_t* tile_counts);

/* scan_tile_counts (scan.wgsl:27-81): exclusive prefix of the counts; meta filled as the
 * kernel does with `capacity`. Returns the uncapped total. */
uint64_t or_scan(const uint32_t* counts, uint64_t n, uint64_t capacity, uint32_t* offsets,
                 sp_intersection_meta* meta);

/* emit_tile_keys.wgsl:13-36, the stable radix sort (sort.rs:92-98) and tile_ranges.wgsl:9-22.
 * Outputs `count` sorted keys (64-bit values of the key layout), the Gaussian of each entry,
 * its emission slot, and 2 * tiles range entries. Returns count. */
uint64_t or_bin(const sp_projected* proj, const uint32_t* offsets, uint64_t n, const sp_camera_uniform* cam,
                uint64_t capacity, int key_mode, uint64_t* sorted_keys, uint32_t* sorted_gaussians,
                uint32_t* sorted_slots, uint32_t* ranges);

/* rasterize_forward.wgsl:22-88. image: P * 4 (premultiplied rgb, transmittance). */
void or_blend_forward(const sp_projected* proj, const uint32_t* sorted_gaussians, const uint32_t* ranges,
                      const sp_camera_uniform* cam, float* image, uint32_t* contributions);

/* ssim_forward.wgsl:34-91 on one view's ground truth (P * 4). partials: P * 3 * 4. */
void or_ssim(const float* image, const float* ground_truth, uint32_t width, uint32_t height, float* partials);

/* loss.wgsl:35-97. loss_gradient, pixel_loss: P * 4. */
void or_loss(const float* image, const float* ground_truth, const float* partials, uint32_t width,
             uint32_t height, const sp_loss_weights* weights, float* loss_gradient, float* pixel_loss);

/* rasterize_backward.wgsl:30-133: one SP_GRAD_STRIDE slot per (Gaussian, tile) entry,
 * indexed by emission slot; intersection_gradients holds capacity * 10 floats. */
void or_blend_backward(const sp_projected* proj, const uint32_t* sorted_gaussians, const uint32_t* sorted_slots,
                       const uint32_t* ranges, const sp_camera_uniform* cam, const float* image,
                       const uint32_t* contributions, const float* loss_gradient, float* intersection_gradients);

/* or_blend_backward, and into `magnitudes` (capacity * 10 doubles) per slot the sums of the
 * absolute values of the same per-pixel terms: the scale of the rounding error any other
 * order of summing them can carry (for the tests' element-wise bars). */
void or_blend_backward_magnitudes(const sp_projected* proj, const uint32_t* sorted_gaussians,
                                  const uint32_t* sorted_slots, const uint32_t* ranges, const sp_camera_uniform* cam,
                                  const float* image, const uint32_t* contributions, const float* loss_gradient,
                                  float* intersection_gradients, double* magnitudes);

/* project_backward.wgsl:30-227 + reduce_camera_gradient.wgsl:10-34 (+ SH degree 1-3).
 * param_gradients: n * stride (overwritten); camera_gradient: 14; stats: n (added to). */
void or_project_backward(const float* params, uint64_t n, uint32_t sh_degree, const sp_camera_uniform* cam,
                         const sp_projected* proj, const uint32_t* offsets, const float* intersection_gradients,
                         uint64_t capacity, float* param_gradients, float* camera_gradient,
                         sp_densify_stats* stats);

/* adam.wgsl:20-37 then clamp_scales.wgsl:15-29. lr_by_slot: one rate per parameter slot
 * (stride entries); bias1 = 1 - beta1^step, bias2 = 1 - beta2^step. */
void or_adam_step(float* params, const float* gradients, float* first_moment, float* second_moment, uint64_t n,
                  uint32_t stride, const float* lr_by_slot, float bias1, float bias2, float max_log_scale,
                  float max_log_anisotropy);

/* The per-slot learning rates (LearningRates::by_slot, optimizer.rs:82-100, with the SH
 * degree 1-3 slots at `sh_rest`). */
void or_learning_rates_by_slot(const sp_learning_rates* rates, float position_scale, uint32_t stride, float* out);

/* 1 - beta^step as the host computes it for the kernels (adam.wgsl:31-32). */
float or_bias_correction(float beta, uint32_t step);

/* The libm exp, for checking the shared exps (include/splat_math.h). */
float or_libm_expf(float x);
float or_sp_expf(float x);
float or_sp_expf_exact(float x);

/* One full training step of one view (training.rs:197-209 with fixed poses): forward,
 * loss against view `view`, backward, Adam. Scratch buffers are allocated inside. The
 * timed CPU baseline. Returns the mean total loss; intersections written to *count. */
double or_train_step(float* params, uint64_t n, uint32_t sh_degree, const sp_camera_uniform* cam,
                     const float* ground_truth_view, float* first_moment, float* second_moment,
                     const float* lr_by_slot, uint32_t step, float max_log_scale, float max_log_anisotropy,
                     uint64_t* count);

/* densify.rs:147-257 (densify) with split_child (259-273) and SplitMix64 (275-297): the
 * Gaussians and moments after one densification, `stride` floats per Gaussian. Fills
 * `report`; writes the outputs when out_capacity >= report->after. Returns 0, 1 when every
 * Gaussian was pruned (the reference panics), 2 when the outputs did not fit. */
int or_densify(const float* params, const float* first_moment, const float* second_moment,
               const sp_densify_stats* stats, uint64_t n, uint32_t stride, float extent, uint64_t max_count,
               const sp_densify_settings* settings, int reset_opacity, uint64_t seed, float* out_params,
               float* out_first, float* out_second, uint64_t out_capacity, sp_densify_report* report);
/* One draw of the SplitMix64 stream seeded with `seed`: the (index + 1)-th next_u64. */
uint64_t or_splitmix64(uint64_t seed, uint64_t index);
/* f32::total_cmp order as an unsigned key (the densify candidates' sort order). */
uint32_t or_total_order_key(float value);

/* Threads the oracle's OpenMP loops use (0 = all). */
void or_set_threads(int threads);
int or_get_threads(void);

#ifdef __cplusplus
}
#endif

#endif
