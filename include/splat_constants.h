/* Constants of the differentiable Gaussian-splatting path, shared by the CUDA kernels
 * (splatting-rs_b200/csrc) and the CPU oracle (oracle/).
 *
 * Values follow instantsplat-rs/src/shaders/common.wgsl:7-36 (mirrored on the Rust side in
 * instantsplat-rs/src/shaders.rs:28-48) and the host constants they depend on
 * (instantsplat-rs/src/rasterizer.rs:24-27, optimizer.rs:64-66, loss.rs:32-36,
 * prune.rs:23-26). The SH degree 1-3 extension (stride 59) has no reference counterpart.
 */
#ifndef SPLAT_CONSTANTS_H
#define SPLAT_CONSTANTS_H

/* Pixels per tile side (common.wgsl:7). */
#define SP_TILE 16
/* Floats per Gaussian at SH degree 0 (common.wgsl:8): position xyz, log scale xyz,
 * rotation wxyz, opacity logit, SH dc rgb. */
#define SP_PARAM_STRIDE_SH0 14
#define SP_SLOT_POSITION 0
#define SP_SLOT_LOG_SCALE 3
#define SP_SLOT_ROTATION 6
#define SP_SLOT_OPACITY 10
/* First SH coefficient; coefficient k of channel c sits at SP_SLOT_SH + 3k + c, so
 * degree 0 is exactly the reference layout (common.wgsl:13). */
#define SP_SLOT_SH 11
/* Floats per (Gaussian, tile) gradient slot: mean xy, conic abc, colour rgb, opacity,
 * one unused (common.wgsl:14-15). */
#define SP_GRAD_STRIDE 10
/* Per-view camera gradient: 9 rotation entries (rows), translation, 2 focals
 * (common.wgsl:16-18). */
#define SP_CAMERA_GRAD_STRIDE 14
/* Bits of the sort key below the tile index (common.wgsl:19-20). */
#define SP_DEPTH_BITS 20
#define SP_SH_C0 0.28209479f
#define SP_COVARIANCE_BLUR 0.3f
#define SP_NEAR_Z 0.01f
#define SP_VIEW_LIMIT_FACTOR 1.3f
#define SP_MIN_ALPHA (1.0f / 255.0f)
#define SP_MAX_ALPHA 0.99f
#define SP_MIN_TRANSMITTANCE 1e-4f
/* SSIM: 11x11 Gaussian window of sigma 1.5, zero padded (common.wgsl:31-36). */
#define SP_SSIM_RADIUS 5
#define SP_SSIM_SIGMA 1.5f
#define SP_SSIM_C1 0.0001f
#define SP_SSIM_C2 0.0009f
/* Floats per pixel of the ground truth: rgb premultiplied by the mask, then the mask
 * (loss.rs:91-92). */
#define SP_GROUND_TRUTH_STRIDE 4
/* Intersection list capacity per Gaussian under the fixed policy (rasterizer.rs:27). */
#define SP_INTERSECTIONS_PER_GAUSSIAN 24
/* Tiles the 32-bit (tile << 20 | depth >> 12) key can hold (rasterizer.rs:24-25). */
#define SP_MAX_TILES_KEY32 4096u
/* Adam (optimizer.rs:64-66). */
#define SP_ADAM_BETA1 0.9f
#define SP_ADAM_BETA2 0.999f
#define SP_ADAM_EPSILON 1e-15f
/* Scale limits (prune.rs:23-26). */
#define SP_SCALE_MAX_ANISOTROPY 10.0f
#define SP_SCALE_MAX_EXTENT_FRACTION 0.02f
/* Loss weights (loss.rs:32-36). */
#define SP_LOSS_L1 0.8f
#define SP_LOSS_DSSIM 0.2f
#define SP_LOSS_ALPHA 1.0f
/* Position learning-rate decay over a run (optimizer.rs:56). */
#define SP_POSITION_RATE_FINAL_OVER_INITIAL 0.01f

/* Real spherical-harmonic basis normalisation constants for degrees 1-3 (the
 * standard orthonormal real SH of the 3DGS colour model). Degree 0 is SP_SH_C0. */
#define SP_SH_C1 0.4886025119029199f
#define SP_SH_C2_0 1.0925484305920792f
#define SP_SH_C2_1 (-1.0925484305920792f)
#define SP_SH_C2_2 0.31539156525252005f
#define SP_SH_C2_3 (-1.0925484305920792f)
#define SP_SH_C2_4 0.5462742152960396f
#define SP_SH_C3_0 (-0.5900435899266435f)
#define SP_SH_C3_1 2.890611442640554f
#define SP_SH_C3_2 (-0.4570457994644658f)
#define SP_SH_C3_3 0.3731763325901154f
#define SP_SH_C3_4 (-0.4570457994644658f)
#define SP_SH_C3_5 1.445305721320277f
#define SP_SH_C3_6 (-0.5900435899266435f)

/* Floats per Gaussian at SH degree d: 11 geometry/opacity floats plus 3 per basis
 * function ((d + 1)^2 of them). */
#define SP_PARAM_STRIDE(d) (11 + 3 * ((d) + 1) * ((d) + 1))

#endif
