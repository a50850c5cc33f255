/* splat.h — C ABI of the B200-native differentiable Gaussian-splatting rasterizer and
 * optimiser step (libsplat_b200.so).
 *
 * The entry points mirror the Rust API of instantsplat-rs, so that its `Trainer`
 * (instantsplat-rs/src/training.rs) can hold an sp_rasterizer / sp_adam instead of a
 * `Rasterizer` / `Adam`:
 *   Rasterizer  — instantsplat-rs/src/rasterizer.rs:134-565
 *   Adam        — instantsplat-rs/src/optimizer.rs:118-276
 *   camera      — instantsplat-rs/src/camera.rs:8-70
 *   pose chain  — instantsplat-rs/src/camera_pose.rs:39-99, pose_refinement.rs:113-163
 * Each declaration names the reference item it replaces.
 *
 * Conventions.
 *  - Every call returns an sp_status; SP_OK is 0. Where the reference panics (an assert!
 *    or expect), the matching call returns an error status instead and leaves its
 *    outputs untouched; sp_last_error() gives the message.
 *  - Device pointers passed in (parameters, ground truth) are borrowed: the caller owns
 *    them and they must outlive the object that holds them (rasterizer.rs:176-184 takes
 *    them as &wgpu::Buffer the same way). The library never frees them.
 *  - All device work of a context is enqueued, in call order, on the context's CUDA
 *    stream (its own, or one the caller lends). sp_read_* calls copy to host memory and
 *    synchronise that stream, like the reference's blocking read_* wrappers.
 *  - A context and everything made from it is used from one host thread at a time (the
 *    reference runs one GPU job at a time, web/src/lib.rs:1-5). One context per GPU.
 *  - Structures are #[repr(C)] compatible with the reference's Pod types: sizes are
 *    checked by tests/test_abi.py (CameraUniform 80 B, CameraGradient 56 B,
 *    IntersectionMeta 20 B, DensifyStats 16 B, Projected 80 B).
 */
#ifndef SPLAT_H
#define SPLAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SP_ABI_VERSION 1

typedef enum sp_status {
    SP_OK = 0,
    /* A size or argument check failed: every assert! of rasterizer.rs:185-199, 399, 447,
     * 454 and optimizer.rs:272-273, 302-303, 348-351. */
    SP_ERR_INVALID = 1,
    /* The tile grid is larger than the library holds (over 65535 tiles on a side). The
     * reference stops at 4096 tiles in all (rasterizer.rs:188-192); this library moves to
     * 64-bit keys there instead, keeping the same order. */
    SP_ERR_TOO_MANY_TILES = 2,
    /* The last forward pass had more (Gaussian, tile) pairs than the intersection list
     * holds (the panic of read_intersections_async, rasterizer.rs:536-544). */
    SP_ERR_OVERFLOW = 3,
    /* A device-side wait gave up after its iteration limit (sort look-back). */
    SP_ERR_TIMEOUT = 4,
    SP_ERR_CUDA = 5,
    SP_ERR_NCCL = 6,
    /* A pose gradient was not finite (pose_refinement.rs:113-125). */
    SP_ERR_NONFINITE = 7,
    SP_ERR_NO_DEVICE = 8,
    SP_ERR_OUT_OF_MEMORY = 9
} sp_status;

/* World-to-camera rows (r0, r1, r2, t), intrinsics and tile grid: CameraUniform,
 * camera.rs:23-31 / common.wgsl:38-47. 80 bytes. */
typedef struct sp_camera_uniform {
    float world_to_camera_rows[3][4];
    float focal[2];
    float principal_point[2];
    uint32_t width;
    uint32_t height;
    uint32_t tiles_x;
    uint32_t tiles_y;
} sp_camera_uniform;

/* dL/d(world-to-camera rotation rows, translation, focal): CameraGradient,
 * camera.rs:39-43. 56 bytes. */
typedef struct sp_camera_gradient {
    float world_to_camera_rotation_rows[3][3];
    float world_to_camera_translation[3];
    float focal[2];
} sp_camera_gradient;

/* IntersectionMeta, rasterizer.rs:29-37. 20 bytes. */
typedef struct sp_intersection_meta {
    uint32_t count;
    uint32_t sort_blocks;
    uint32_t histogram_length;
    uint32_t overflow;
    uint32_t capacity;
} sp_intersection_meta;

/* DensifyStats, rasterizer.rs:63-75. 16 bytes. */
typedef struct sp_densify_stats {
    float mean_gradient_sum;
    float visible_count;
    float max_radius;
    float _pad;
} sp_densify_stats;

/* DensifySettings (densify.rs:19-45): when and how strongly the Gaussians are densified and
 * pruned. opacity_reset_interval 0 is None. */
typedef struct sp_densify_settings {
    uint32_t interval;
    uint32_t start;
    float stop_fraction;
    float gradient_threshold;
    float split_scale_fraction;
    float prune_opacity;
    float max_screen_radius;
    float max_growth;
    uint32_t opacity_reset_interval;
    uint32_t _pad;
} sp_densify_settings;

/* DensifyReport (densify.rs:97-111). */
typedef struct sp_densify_report {
    uint64_t before;
    uint64_t cloned;
    uint64_t split;
    uint64_t pruned_transparent;
    uint64_t pruned_oversized;
    uint64_t over_budget;
    uint64_t after;
    uint32_t opacity_reset;
    uint32_t _pad;
} sp_densify_report;

/* Projected, rasterizer.rs:46-61 / common.wgsl:49-61 (the diagnostics mirror). 80 bytes. */
typedef struct sp_projected {
    float mean[2];
    float _pad0[2];
    float conic[3];
    float depth;
    float color[3];
    float opacity;
    uint32_t radius;
    uint32_t _pad1;
    uint32_t tile_min[2];
    uint32_t tile_max[2];
    uint32_t _pad2[2];
} sp_projected;

/* LossWeights, loss.rs:20-36. */
typedef struct sp_loss_weights {
    float l1;
    float dssim;
    float alpha;
} sp_loss_weights;

/* LossTerms, loss.rs:38-64: means over the pixels (summed in double). */
typedef struct sp_loss_terms {
    float l1;
    float alpha;
    float dssim;
    float total;
} sp_loss_terms;

/* LearningRates, optimizer.rs:17-26, plus the rate of the SH coefficients of degree 1-3
 * (an extension; the reference has degree 0 only). */
typedef struct sp_learning_rates {
    float position;
    float log_scale;
    float rotation;
    float opacity;
    float sh_dc;
    float camera_rotation;
    float camera_translation;
    float camera_focal;
    float sh_rest;
} sp_learning_rates;

/* Sort key layouts. */
enum {
    /* (tile << 20) | (bits(depth) >> 12): the reference's order (emit_tile_keys.wgsl:24-29),
     * held in 32 bits while tiles <= 4096 and in 64 bits above (the reference refuses
     * those images; the order stays (tile, depth >> 12, Gaussian index)). */
    SP_KEYS_REF20 = 0,
    /* (tile << 32) | bits(depth): the full-precision depth order, 64-bit keys. */
    SP_KEYS_FULL32 = 1
};

/* Which tiles of a Gaussian get a key. */
enum {
    /* Every tile of its bounding rectangle (project_forward.wgsl:76-83): the reference's
     * intersection lists. */
    SP_TILES_RECTANGLE = 0,
    /* Only the rectangle's tiles where its alpha can reach 1/255 at a pixel centre (its
     * ellipse at that level, padded, meets the tile): shorter lists, fewer keys to sort. The
     * dropped pairs are ones the blend skips at every pixel, so images, losses, gradients
     * and parameters are those of SP_TILES_RECTANGLE; intersection counts, list indices and
     * contribution counts are of the shorter lists. Needs SP_BWD_ATOMIC (the deterministic
     * backward addresses its slots by the tile's place in the rectangle). */
    SP_TILES_ELLIPSE = 1
};

/* How the blend backward sums each Gaussian's gradient over the pixels of a tile. */
enum {
    /* One write per (Gaussian, tile) slot, summed per Gaussian afterwards in slot order,
     * as rasterize_backward.wgsl:1-7 and project_backward.wgsl:38-55: bit-stable. */
    SP_BWD_DETERMINISTIC = 0,
    /* Warp-shuffle pre-reduction, then vector float atomics into per-Gaussian sums. */
    SP_BWD_ATOMIC = 1
};

typedef struct sp_options {
    uint32_t key_mode;                   /* SP_KEYS_* (default SP_KEYS_REF20) */
    uint32_t backward_mode;              /* SP_BWD_* (default SP_BWD_ATOMIC) */
    uint32_t sh_degree;                  /* 0 (stride 14, the reference) .. 3 (stride 59) */
    uint32_t intersections_per_gaussian; /* capacity = this * N (default 24, rasterizer.rs:27) */
    /* 0: each backward overwrites the parameter gradients (the reference). 1: it adds to
     * them, for batches of views summed before one Adam step; clear with
     * sp_zero_param_gradients. */
    uint32_t accumulate_gradients;
    sp_loss_weights loss_weights;        /* default LOSS_WEIGHTS (loss.rs:32-36) */
    /* SP_TILES_* (default SP_TILES_RECTANGLE). */
    uint32_t tile_culling;
} sp_options;

typedef struct sp_context sp_context;
typedef struct sp_rasterizer sp_rasterizer;
typedef struct sp_adam sp_adam;

/* ---------------------------------------------------------------- context / runtime */

/* Library version string. */
const char* sp_version(void);
/* Human-readable name of a status. */
const char* sp_status_string(sp_status status);
/* Replaces Gpu::request / request_async (gpu.rs:29-66): device `device`, its own stream. */
sp_status sp_context_create(int device, sp_context** out);
/* As sp_context_create, but enqueues on `stream` (a cudaStream_t the caller keeps alive),
 * so that the work orders with the caller's own (e.g. a torch stream). NULL gives the
 * context a stream of its own, as sp_context_create; the legacy default stream is passed
 * as cudaStreamLegacy. */
sp_status sp_context_create_on_stream(int device, void* stream, sp_context** out);
void sp_context_destroy(sp_context* ctx);
/* Waits for every call enqueued on the context's stream (Gpu::submit + poll). */
sp_status sp_context_sync(sp_context* ctx);
/* The cudaStream_t the context enqueues on. */
void* sp_context_stream(sp_context* ctx);
/* Message of the last error status a call on this context returned. */
const char* sp_last_error(const sp_context* ctx);

/* --------------------------------------------------------------------------- camera */

/* PinholeCamera::uniform (camera.rs:51-70): camera-to-world rotation (row-major 3x3) and
 * centre in f64, focal and principal point in pixels; tiles of SP_TILE pixels. */
sp_status sp_camera_uniform_from_pinhole(const double rotation_c2w[9], const double translation[3],
                                         const double focal[2], const double principal_point[2],
                                         uint32_t width, uint32_t height, sp_camera_uniform* out);

/* ----------------------------------------------------------------------- rasterizer */

/* Fills `out` with the defaults (reference behaviour, SH degree 0). */
void sp_options_default(sp_options* out);

/* Rasterizer::new (rasterizer.rs:176-391). `d_params` holds gaussian_count * stride floats
 * (stride 14 at SH degree 0); `d_ground_truth` holds view_count images of
 * width * height * 4 floats (loss::ground_truth_rgba, loss.rs:95-104). Both are device
 * pointers the caller keeps alive. `options` may be NULL for the defaults. */
sp_status sp_rasterizer_create(sp_context* ctx, const float* d_params, uint64_t gaussian_count,
                               uint32_t width, uint32_t height, const float* d_ground_truth,
                               uint32_t view_count, const sp_options* options, sp_rasterizer** out);
void sp_rasterizer_destroy(sp_rasterizer* r);
/* The parameter floats per Gaussian this rasterizer reads. */
uint32_t sp_rasterizer_param_stride(const sp_rasterizer* r);
/* Rasterizer::set_camera (rasterizer.rs:398-401). Takes effect at the next sp_forward /
 * sp_backward. SP_ERR_INVALID when the image size differs. */
sp_status sp_set_camera(sp_rasterizer* r, const sp_camera_uniform* camera);
/* Rasterizer::encode_forward (rasterizer.rs:404-416): projection, binning, sort, blend. */
sp_status sp_forward(sp_rasterizer* r);
/* Rasterizer::encode_loss (rasterizer.rs:420-425): loss of the image against view `view`. */
sp_status sp_loss(sp_rasterizer* r, uint32_t view);
/* Rasterizer::encode_backward (rasterizer.rs:429-442). */
sp_status sp_backward(sp_rasterizer* r);
/* sp_backward in parts (no counterpart in the reference), so that a collective on the
 * gradients of some Gaussians can overlap the backward of the others: the blend backward
 * (K8) once, then the projection backward (K9-K10) over ranges [first, first + count) of the
 * Gaussians, first a multiple of 256, the ranges covering all of them once, in order; the
 * camera gradient is complete after the last range. */
sp_status sp_backward_blend(sp_rasterizer* r);
sp_status sp_backward_project(sp_rasterizer* r, uint64_t first, uint64_t count);
/* write_loss_gradient / write_image (rasterizer.rs:446-456): width*height*4 floats from
 * host memory (src_is_device = 0) or device memory (1). */
sp_status sp_write_loss_gradient(sp_rasterizer* r, const float* src, int src_is_device);
sp_status sp_write_image(sp_rasterizer* r, const float* src, int src_is_device);
/* Overwrites the accumulated densify statistics with N sp_densify_stats from host memory
 * (diagnostics and tests; the backward passes accumulate them otherwise). */
sp_status sp_write_densify_stats(sp_rasterizer* r, const sp_densify_stats* host);
/* Rasterizer::param_gradients (rasterizer.rs:467-469): device pointer to N * stride floats. */
float* sp_param_gradients(sp_rasterizer* r);
/* Zeroes the parameter gradients (for accumulate_gradients batches). */
sp_status sp_zero_param_gradients(sp_rasterizer* r);
/* Device pointer to the 14-float camera gradient of the last backward. */
float* sp_camera_gradient_device(sp_rasterizer* r);
/* Device pointer to the N accumulated densify statistics (read and written by the
 * multi-GPU merge of several ranks' statistics before a densification). */
sp_densify_stats* sp_densify_stats_device(sp_rasterizer* r);
/* The read_* calls of rasterizer.rs:458-549, into host memory. */
sp_status sp_read_loss_gradient(sp_rasterizer* r, float* host);      /* P * 4 */
sp_status sp_read_param_gradients(sp_rasterizer* r, float* host);    /* N * stride */
sp_status sp_read_densify_stats(sp_rasterizer* r, sp_densify_stats* host); /* N */
sp_status sp_read_camera_gradient(sp_rasterizer* r, sp_camera_gradient* host);
sp_status sp_read_image(sp_rasterizer* r, float* host_rgbt);         /* P * 4 */
sp_status sp_read_pixel_loss(sp_rasterizer* r, float* host);         /* P * 4 */
/* read_loss; `out` is filled, and SP_ERR_OVERFLOW (or the device status) returned, when the
 * frame was rendered from truncated lists. */
sp_status sp_read_loss(sp_rasterizer* r, sp_loss_terms* out);

/* Largest pixel_count sp_loss_sums_noalloc accepts: 1024 blocks of 4096 pixels. */
#define SP_NOALLOC_MAX_PIXELS 4194304ull
/* No counterpart in the reference. The sums over pixels of the 4 per-pixel loss terms
 * (L1, alpha error, 1 - SSIM, weighted total: what sp_read_loss divides by the pixel count)
 * of `d_pixel_loss` (pixel_count x 4 floats, device) into `d_sums` (4 doubles, device), on
 * `stream` of device `device`, without allocating anything: for callers whose device memory
 * is owned by their own allocator or who cannot afford the device-wide synchronisation of a
 * cudaMalloc / cudaFree. Its scratch is a fixed array in the library of 4 * 1024 + 1 doubles
 * (32,776 bytes, about 32 KiB) that every GPU loading the library keeps until exit; hence the
 * limit: SP_ERR_INVALID for pixel_count 0 or above SP_NOALLOC_MAX_PIXELS. `d_pixel_loss` must
 * be 16-byte aligned and `d_sums` 8-byte aligned (SP_ERR_INVALID otherwise, checked before
 * anything is enqueued). The first call on a device looks the array's device
 * address up (cudaGetSymbolAddress); make that first call before any stream capture. Every
 * call shares the array, so calls that overlap on the GPU race: order them on one stream.
 * Enqueues only; the sums are ready when the stream reaches them. */
sp_status sp_loss_sums_noalloc(int device, const float* d_pixel_loss, uint64_t pixel_count, double* d_sums,
                               void* stream);
/* read_intersections (rasterizer.rs:536-544): fills `out` and returns SP_ERR_OVERFLOW when
 * the list overflowed (where the reference panics). */
sp_status sp_read_intersections(sp_rasterizer* r, sp_intersection_meta* out);
/* The intersection capacity sized from the scan (no counterpart in the reference, whose
 * capacity is fixed at 24 N, rasterizer.rs:27, and which panics on overflow): the number of
 * (Gaussian, tile) pairs the last forward pass's scan counted, before truncation at the
 * capacity. A caller that met SP_ERR_OVERFLOW reserves that many (with a margin) and
 * renders again. */
sp_status sp_intersections_needed(sp_rasterizer* r, uint64_t* total);
/* Grows the intersection buffers (keys, values, the sort's look-back words and, in the
 * deterministic backward, the per-slot gradients) to `capacity` pairs, below 2^32. Never
 * shrinks. Synchronises the context's stream; the last forward pass's lists are dropped, so
 * the next backward needs a forward first. On an allocation failure the rasterizer is left
 * as it was and SP_ERR_CUDA is returned. */
sp_status sp_reserve_intersections(sp_rasterizer* r, uint64_t capacity);
/* sp_backward then sp_adam_step(adam, position_rate_factor) in one pass over the
 * parameters: the projection backward applies the Adam update and the scale clamp to each
 * Gaussian as soon as its gradient is complete, so the parameter gradients are not written
 * (sp_param_gradients / sp_read_param_gradients then hold stale values). The camera
 * gradient, densify statistics and blend sums are produced as by sp_backward. `adam` must
 * be over this rasterizer's own parameters and gradient buffer, and the rasterizer must not
 * accumulate gradients. Parameters and moments equal those of the two separate calls bit for
 * bit. No counterpart in the reference, whose Trainer::step_async (training.rs:203-204)
 * encodes the two passes one after the other. */
sp_status sp_backward_adam(sp_rasterizer* r, sp_adam* adam, float position_rate_factor);
/* Trainer::step_async (training.rs:197-209) in one call: set the camera, forward, loss
 * against `view`, backward, one Adam step at `position_rate_factor` (the last two fused as
 * by sp_backward_adam unless the rasterizer accumulates gradients or `adam` is over other
 * buffers); then, if either
 * output is non-NULL, the camera gradient (56 B) and the loss terms (32 B) are copied to
 * pinned host memory and the stream is synchronised once — the per-step read-back the
 * reference's pose refinement does (training.rs:205-208). With that read-back the step's
 * errors are reported: SP_ERR_TIMEOUT when a device wait gave up, SP_ERR_OVERFLOW when the
 * forward pass had more (Gaussian, tile) pairs than the intersection list holds (the step
 * ran on the truncated list; the reference's read_step_async panics there, training.rs:271
 * and rasterizer.rs:536-544). */
sp_status sp_train_step(sp_rasterizer* r, sp_adam* adam, const sp_camera_uniform* camera, uint32_t view,
                        float position_rate_factor, sp_camera_gradient* camera_gradient_out, sp_loss_terms* loss_out);
/* Rasterizer::render (rasterizer.rs:552-564): set_camera, forward, overflow check, image. */
sp_status sp_render(sp_rasterizer* r, const sp_camera_uniform* camera, float* host_rgbt);
/* Diagnostics, as the reference's `Projected` mirror "for tests and diagnostics"
 * (rasterizer.rs:46-61): the per-Gaussian projection of the last forward pass. */
sp_status sp_read_projected(sp_rasterizer* r, sp_projected* host);   /* N */
/* The intersection list of the last forward pass in sorted order: `count` keys (as 64-bit
 * values of the key layout) and the Gaussian index of each entry. */
sp_status sp_read_sorted_intersections(sp_rasterizer* r, uint64_t* keys_host, uint32_t* gaussians_host);
/* Per tile [start, end) of the sorted list, 2 * tiles entries (tile_ranges.wgsl:9-22). */
sp_status sp_read_tile_ranges(sp_rasterizer* r, uint32_t* host);
/* Per pixel, how many of the tile's entries contributed (rasterize_forward.wgsl:72). */
sp_status sp_read_contributions(sp_rasterizer* r, uint32_t* host);
/* Per Gaussian, the exclusive prefix sum of the tile counts (scan.wgsl:64-81). */
sp_status sp_read_tile_offsets(sp_rasterizer* r, uint32_t* host);
/* Per-Gaussian sums of the blend backward (mean xy, conic abc, colour rgb, opacity, 0)
 * of the last sp_backward: SP_GRAD_STRIDE floats per Gaussian. */
sp_status sp_read_gaussian_blend_gradients(sp_rasterizer* r, float* host);
/* Resets the densification statistics to zero (a fresh rasterizer starts at zero). */
sp_status sp_clear_densify_stats(sp_rasterizer* r);
/* Work of the blend kernels for the current camera and parameters (replays the forward
 * pass's per-pixel decisions; no reference counterpart, used for roofline accounting):
 * forward_pairs = sum over pixels of the tile-list entries the forward visits, up to and
 * including the one that terminates the pixel; backward_pairs = sum over pixels of the
 * contributor count (the entries the backward replays); taken_pairs (may be NULL) = sum over
 * pixels of the entries actually blended (alpha at least 1/255, before the termination). */
sp_status sp_count_blend_work(sp_rasterizer* r, uint64_t* forward_pairs, uint64_t* backward_pairs,
                              uint64_t* taken_pairs);

/* Error-path test switch (no counterpart in the reference): from the next forward pass on,
 * sort partition `partition` of every sort pass never posts its digit counts, and its
 * successors' look-back waits give up after a short limit (a few thousand polls) instead of
 * the normal one, raising SP_ERR_TIMEOUT, which the next sp_read_intersections or
 * sp_train_step returns; the scatter stays inside the key buffers (its order is then
 * wrong). UINT32_MAX switches it off. For tests of the bounded device wait only. */
sp_status sp_debug_stall_sort_partition(sp_rasterizer* r, uint32_t partition);

/* Parity test support (no counterpart in the reference): the falloff power
 * -1/2 (a dx^2 + c dy^2) - b dx dy (rasterize_forward.wgsl:60-63) exactly as the forward and
 * atomic backward blend kernels compute it, for `count` items of 12 floats each in device
 * memory (16-byte aligned): a blend record's words [0] (mean.x, mean.y, conic.a, conic.b) and
 * [1] (conic.c, ...), then the pixel column x and two pixel rows y0, y1 (and one unused float).
 * Writes 2 floats per item (the power at (x, y0) and at (x, y1)) to d_powers, on `stream` of
 * the current device. */
sp_status sp_debug_falloff_powers(const float* d_items, uint64_t count, float* d_powers, void* stream);

/* Parity test support (no counterpart in the reference): the divisions of the Adam step and
 * the projection as their kernels compute them, for `count` operand pairs x, y in device
 * memory. Writes 3 floats per pair to d_quotients: x / y as the division by a bias correction
 * 1 - beta^t (y in (0, 1], else 0 is written), x / y as Adam's division by
 * sqrt(v_hat) + epsilon (y in [2^-126, 2^126] or +inf, else 0 is written), and x / y as the
 * projection divides (any y). Each must equal the IEEE single-precision quotient. On
 * `stream` of the current device. */
sp_status sp_debug_adam_quotients(const float* d_x, const float* d_y, uint64_t count, float* d_quotients,
                                  void* stream);

/* ------------------------------------------------------------- per-kernel device timing */

/* Kernels timed by the profiler (CUDA events on the context's stream around each launch;
 * the reference has only wall-clock timing, training.rs:104,147,303). */
enum {
    SP_K_PROJECT = 0,
    SP_K_SCAN = 1,
    SP_K_EMIT = 2,
    SP_K_SORT = 3,
    SP_K_RANGES = 4,
    SP_K_BLEND_FORWARD = 5,
    SP_K_SSIM = 6,
    SP_K_LOSS = 7,
    SP_K_BLEND_BACKWARD = 8,
    SP_K_PROJECT_BACKWARD = 9,
    SP_K_ADAM = 10,
    SP_K_TILE_ORDER = 11, /* the blend kernels' tile schedule (no counterpart in the reference) */
    SP_K_BACKWARD_ADAM = 12, /* projection backward with the Adam step fused (sp_backward_adam) */
    SP_K_DENSIFY = 13,       /* the densification's kernels (sp_densify_plan, sp_densify_apply) */
    SP_K_PEER_ADAM = 14,     /* the peer-memory exchange with the Adam step (sp_peer_exchange_step) */
    SP_K_COUNT = 15
};
/* Starts (1) or stops (0) recording events around every kernel launch of the context. */
sp_status sp_profile_enable(sp_context* ctx, int enable);
/* Waits for the recorded launches and adds their device milliseconds and launch counts
 * per kernel into ms[SP_K_COUNT] and launches[SP_K_COUNT]; then forgets them. */
sp_status sp_profile_read(sp_context* ctx, double* ms, uint64_t* launches);

/* ---------------------------------------------------------------------------- Adam */

/* Adam::new (optimizer.rs:137-159): moments zeroed, `position_scale` = camera extent
 * (multiplies the position rate, sets the log-scale cap ln(0.02 * extent)). `d_params`
 * is updated in place; `d_gradients` is read (typically sp_param_gradients). */
sp_status sp_adam_create(sp_context* ctx, float* d_params, const float* d_gradients, uint64_t gaussian_count,
                         uint32_t sh_degree, const sp_learning_rates* rates, float position_scale, sp_adam** out);
/* Adam::resumed (optimizer.rs:164-188): the optimiser `from`'s rates, scale and step count
 * over new buffers, starting from host moments of gaussian_count * stride floats each. */
sp_status sp_adam_resume(const sp_adam* from, float* d_params, const float* d_gradients, uint64_t gaussian_count,
                         const float* host_first_moment, const float* host_second_moment, sp_adam** out);
void sp_adam_destroy(sp_adam* adam);
/* Adam::encode_step (optimizer.rs:248-264): one update with the position rate times
 * `position_rate_factor` in (0, 1], then the scale clamp (clamp_scales.wgsl), fused. */
sp_status sp_adam_step(sp_adam* adam, float position_rate_factor);
/* As sp_adam_step, restricted to Gaussians [first, first + count): the shard of a
 * view-sharded multi-GPU step. Every shard of one step must pass the same
 * position_rate_factor; call sp_adam_advance once per step before the shards. */
sp_status sp_adam_advance(sp_adam* adam, float position_rate_factor);
sp_status sp_adam_step_range(sp_adam* adam, uint64_t first, uint64_t count);
/* Adam::steps_taken (optimizer.rs:266-268). */
uint32_t sp_adam_steps_taken(const sp_adam* adam);
/* Adam::read_moments_async (optimizer.rs:270-275), into host memory. */
sp_status sp_adam_read_moments(sp_adam* adam, float* host_first, float* host_second);
/* Device pointers to the first and second moments (N * stride floats each), for the
 * multi-GPU gather of the ranks' moment shards. */
float* sp_adam_first_moment_device(sp_adam* adam);
float* sp_adam_second_moment_device(sp_adam* adam);

/* ------------------------------------------------- multi-GPU exchange over peer memory */

/* The view-sharded step of several GPUs (one process each, one node) without a library
 * collective: each rank sums the parameter gradients of its share of the Gaussians over
 * every rank's gradient buffer (peer loads over NVLink, in rank order: the sum one GPU
 * accumulating the ranks' views in order would form), takes the Adam step and the scale clamp
 * on that share, and stores the updated parameters into its own and every peer's parameter
 * buffer (peer stores), in one kernel. Shares are [rank n / world, (rank + 1) n / world), n a
 * multiple of world; each rank's moments are current on its share only.
 *
 * Set-up: every rank calls sp_peer_export and gives all ranks' handles (in rank order) to
 * sp_peer_exchange_create, which maps the peers' buffers (CUDA IPC). Each step: every rank
 * must have finished its backward before any rank calls sp_peer_exchange_step, and every
 * rank's call must have finished before any rank's next forward (the caller orders both,
 * e.g. with a one-element collective on the context's stream before and after). */
typedef struct sp_peer_handle {
    uint8_t params[64];         /* cudaIpcMemHandle_t of the allocation holding the parameters */
    uint8_t gradients[64];      /* ... and of the one holding the parameter gradients */
    uint64_t params_offset;     /* byte offsets of the two buffers in those allocations */
    uint64_t gradients_offset;
    uint64_t gaussian_count;
    uint32_t stride;
    int32_t device;
} sp_peer_handle;
sp_status sp_peer_export(const sp_adam* adam, sp_peer_handle* out);
typedef struct sp_peer_exchange sp_peer_exchange;
/* At most 8 ranks; every rank's optimiser over the same count and stride. */
sp_status sp_peer_exchange_create(sp_adam* adam, uint32_t rank, uint32_t world, const sp_peer_handle* handles,
                                  sp_peer_exchange** out);
/* Enqueues the exchange and the Adam step (position_rate_factor as sp_adam_step). */
sp_status sp_peer_exchange_step(sp_peer_exchange* exchange, float position_rate_factor);
void sp_peer_exchange_destroy(sp_peer_exchange* exchange);
/* ------------------------------------------ multi-GPU through the library: communicator */

/* The view-sharded step of several GPUs driven through this ABI alone (no other collective
 * library in the caller): the communicator the survey of the reference's multi-GPU boundary
 * names sp_comm_init(ncclUniqueId, nranks, rank), the gradient exchange with the Adam step, and
 * the collectives of a densification. NCCL is loaded when first needed (libnccl.so.2: the one
 * already in the process, else the system's); without it these calls return SP_ERR_NCCL and
 * the rest of the library works. No counterpart in the reference, which trains on one device.
 *
 * Use: one rank calls sp_comm_unique_id and passes the 128 bytes to the others over any host
 * channel; every rank (one process per GPU) calls sp_comm_init with its own context; then, per
 * step, each rank's backward passes (accumulated over its views with accumulate_gradients, or
 * one view), then sp_exchange_step on every rank. Collective calls must be made by every rank
 * in the same order. Every wait on the host for the other ranks is bounded by the
 * communicator's time limit: past it the communicator is aborted and the call returns
 * SP_ERR_TIMEOUT (the communicator is then unusable; destroy it). */
#define SP_COMM_ID_BYTES 128
typedef struct sp_comm sp_comm;
/* ncclGetUniqueId: the rendezvous of a new communicator (call on one rank only; that process
 * must live until every rank's sp_comm_init has returned). */
sp_status sp_comm_unique_id(uint8_t out[SP_COMM_ID_BYTES]);
/* The NCCL version loaded (e.g. 22703), 0 when NCCL cannot be loaded. */
int sp_comm_nccl_version(void);
/* ncclCommInitRank on ctx's device, non-blocking, waiting up to timeout_ms for every rank. */
sp_status sp_comm_init(sp_context* ctx, const uint8_t id[SP_COMM_ID_BYTES], uint32_t world, uint32_t rank,
                       uint32_t timeout_ms, sp_comm** out);
void sp_comm_destroy(sp_comm* comm);
uint32_t sp_comm_rank(const sp_comm* comm);
uint32_t sp_comm_world(const sp_comm* comm);
/* Enqueues a one-element all-reduce on the context's stream: work any rank enqueues after it
 * starts only once every rank's work enqueued before it has completed. */
sp_status sp_comm_barrier(sp_comm* comm);
/* Waits (host) for the context's stream, up to the time limit; SP_ERR_TIMEOUT past it (a rank
 * that stopped leaves the others' collectives waiting), with the communicator aborted. */
sp_status sp_comm_wait(sp_comm* comm);
/* Sums the parameter gradients of every rank's rasterizer in place (ncclAllReduce). */
sp_status sp_allreduce_grads(sp_comm* comm, sp_rasterizer* r);
/* The sharded Adam step: the gradients reduce-scattered in place (rank r receives the sum of
 * its share [r n / world, (r + 1) n / world) of the Gaussians), Adam and the scale clamp on that
 * share (moments current on the share only), the parameters all-gathered in place. n must be a
 * multiple of world. */
sp_status sp_adam_step_sharded(sp_comm* comm, sp_adam* adam, float position_rate_factor);

/* The exchange of one step, chosen once. */
enum {
    SP_EXCHANGE_AUTO = 0,     /* PEER where the Gaussians split evenly, else ALLREDUCE; PEER falls
                                 back to SHARDED when a rank cannot map its peers' buffers */
    SP_EXCHANGE_PEER = 1,     /* one kernel per rank over NVLink peer memory (sp_peer_exchange_*),
                                 between two barriers; handles exchanged through the communicator */
    SP_EXCHANGE_SHARDED = 2,  /* sp_adam_step_sharded */
    SP_EXCHANGE_ALLREDUCE = 3 /* sp_allreduce_grads, then the whole Adam step on every rank */
};
typedef struct sp_exchange sp_exchange;
/* Collective: every rank with its optimiser over the same Gaussian count. */
sp_status sp_exchange_create(sp_comm* comm, sp_adam* adam, uint32_t mode, sp_exchange** out);
/* The mode in use (SP_EXCHANGE_PEER, _SHARDED or _ALLREDUCE). */
uint32_t sp_exchange_mode(const sp_exchange* exchange);
/* Enqueues the exchange and the Adam step; every rank's gradients must be enqueued before. */
sp_status sp_exchange_step(sp_exchange* exchange, float position_rate_factor);
/* Times one read of `bytes` of rank `peer`'s gradient buffer over NVLink by this rank's GPU
 * (plain float4 loads from the mapped peer buffer, four in flight per thread as the peer
 * exchange issues them; CUDA events on the context's stream, after one untimed read), into
 * *milliseconds: the link bandwidth the exchange is judged against. Peer-memory exchanges only;
 * the peer must not be writing that buffer meanwhile (call between steps). No counterpart in
 * the reference. */
sp_status sp_exchange_probe_link(sp_exchange* exchange, uint32_t peer, uint64_t bytes, float* milliseconds);
/* Makes the Adam moments whole on every rank (the sharded forms keep each rank's share
 * current only): before a densification. */
sp_status sp_exchange_gather_moments(sp_exchange* exchange);
void sp_exchange_destroy(sp_exchange* exchange);
/* Merges every rank's densify statistics in place before a densification: the mean-gradient
 * sums and visible counts summed, the largest screen radius kept (what one device
 * accumulating every view would hold, up to the order of the sums). */
sp_status sp_comm_merge_densify_stats(sp_comm* comm, sp_rasterizer* r);

/* position_rate_factor (optimizer.rs:59-62): 0.01^(step / max(steps - 1, 1)). Returns a
 * negative value where the reference asserts (steps == 0 or step >= steps). */
float sp_position_rate_factor(uint64_t step, uint64_t steps);
/* Adam::resumed (optimizer.rs:164-188) from moments already in device memory (for example
 * those sp_densify_apply wrote): copied into the new optimiser's own buffers. */
sp_status sp_adam_resume_device(const sp_adam* from, float* d_params, const float* d_gradients,
                                uint64_t gaussian_count, const float* d_first_moment, const float* d_second_moment,
                                sp_adam** out);

/* ----------------------------------------------------------------- densification */

/* DensifySettings::densifies_after (densify.rs:77-83): 1 when the Gaussians are densified
 * after `done` (1-based) of `steps` steps, else 0; -1 where the reference asserts
 * (interval 0, done outside 1..=steps). */
int sp_densify_after(const sp_densify_settings* settings, uint64_t done, uint64_t steps);
/* DensifySettings::resets_opacity_after (densify.rs:84-94): 1 or 0; -1 where the reference
 * asserts (a reset interval that is not a multiple of the densify interval). */
int sp_resets_opacity_after(const sp_densify_settings* settings, uint64_t done);

/* densify (densify.rs:147-257) on the device, where the reference reads every buffer back
 * and rebuilds on the CPU (training.rs:238-266). Two calls around the caller's allocation
 * of the new buffers:
 *
 * sp_densify_plan decides the fate of every Gaussian of `r` from its parameters and the
 * densify statistics its backward passes accumulated (pruned when nearly transparent or
 * oversized on screen; cloned or split when its mean screen-space gradient is above the
 * threshold, the highest first while the count stays within `max_count`), and fills
 * `report` (one small read-back: the call's only synchronisation). `adam` must be the
 * optimiser of r's parameters. When every Gaussian would be pruned it returns
 * SP_ERR_INVALID, with the report filled and no plan (the reference panics).
 *
 * sp_densify_apply writes the report->after Gaussians (stride floats each) and their
 * moments into device buffers of at least `capacity` Gaussians: the kept and cloned ones
 * with their moments in index order, then each clone's copy and each split's two children
 * (centres sampled from the Gaussian with SplitMix64 seeded with `seed`, scales / 1.6) with
 * zero moments; with `reset_opacity`, every opacity lowered to 0.01 at most and its
 * moments zeroed. The parameters, moments and statistics must not change between the
 * calls. The outputs must not overlap the inputs. */
typedef struct sp_densify sp_densify;
sp_status sp_densify_plan(sp_rasterizer* r, const sp_adam* adam, float extent, uint64_t max_count,
                          const sp_densify_settings* settings, int reset_opacity, uint64_t seed, sp_densify** out,
                          sp_densify_report* report);
sp_status sp_densify_apply(sp_densify* plan, float* d_params, float* d_first_moment, float* d_second_moment,
                           uint64_t capacity);
void sp_densify_destroy(sp_densify* plan);

/* ------------------------------------------------------------- pose chain (host f64) */

/* PinholeCamera (camera.rs:8-17): camera-to-world rotation (row-major), centre. */
typedef struct sp_pinhole_camera {
    double rotation[9];
    double translation[3];
    double focal[2];
    double principal_point[2];
    uint32_t width;
    uint32_t height;
} sp_pinhole_camera;

/* PoseCorrection (camera_pose.rs:14-21). */
typedef struct sp_pose_correction {
    double rotation[3];
    double translation[3];
} sp_pose_correction;

/* PoseGradient (camera_pose.rs:23-29). */
typedef struct sp_pose_gradient {
    double rotation[3];
    double translation[3];
    double focal_log_scale;
} sp_pose_gradient;

/* camera_pose::corrected_camera (camera_pose.rs:59-68). */
sp_status sp_corrected_camera(const sp_pinhole_camera* initial, const sp_pose_correction* correction,
                              double focal_log_scale, sp_pinhole_camera* out);
/* camera_pose::pose_gradient (camera_pose.rs:81-99). */
sp_status sp_pose_gradient_of(const sp_pinhole_camera* initial, const sp_pose_correction* correction,
                              double focal_log_scale, const sp_camera_gradient* gradient, sp_pose_gradient* out);

typedef struct sp_pose_refinement sp_pose_refinement;
/* PoseRefinement::new (pose_refinement.rs:66-81). */
sp_status sp_pose_refinement_create(const sp_pinhole_camera* initial, uint32_t view_count,
                                    const sp_learning_rates* rates, float extent, sp_pose_refinement** out);
void sp_pose_refinement_destroy(sp_pose_refinement* p);
/* PoseRefinement::camera (pose_refinement.rs:83-85). */
sp_status sp_pose_refinement_camera(const sp_pose_refinement* p, uint32_t view, sp_pinhole_camera* out);
/* PoseRefinement::step (pose_refinement.rs:113-163); SP_ERR_NONFINITE where it asserts. */
sp_status sp_pose_refinement_step(sp_pose_refinement* p, uint32_t view, const sp_camera_gradient* gradient,
                                  float rate_factor);
/* correction(view), focal_scale(), last_gradient() (pose_refinement.rs:91-105). */
sp_status sp_pose_refinement_correction(const sp_pose_refinement* p, uint32_t view, sp_pose_correction* out);
double sp_pose_refinement_focal_scale(const sp_pose_refinement* p);
sp_status sp_pose_refinement_last_gradient(const sp_pose_refinement* p, sp_pose_gradient* out);

/* Trainer::step_async with pose refinement (training.rs:197-209) in one call: the camera of
 * `view` from the host refinement, sp_train_step with its camera-gradient read-back, then the
 * host pose step of `view` (pose_refinement.rs:113-163). Synchronises once. */
sp_status sp_train_step_host_poses(sp_rasterizer* r, sp_adam* adam, sp_pose_refinement* poses, uint32_t view,
                                   float position_rate_factor, sp_loss_terms* loss_out);

/* The pose refinement on the device (no counterpart in the reference, whose
 * pose_refinement.rs:113-163 runs on the host after reading back the camera gradient every
 * step, training.rs:205-208). A copy of a host refinement's state (sp_pose_refinement) bound
 * to a rasterizer: each step the refinement of the view just trained runs in a one-thread
 * kernel on the camera gradient the backward left in device memory, and writes the camera
 * of the next view for the next forward, so a training loop needs no host synchronisation.
 * The arithmetic is the host refinement's (f64, the same source); results agree with it to
 * the rounding of sin, cos, exp and pow. */
typedef struct sp_device_poses sp_device_poses;
sp_status sp_device_poses_create(sp_rasterizer* r, const sp_pose_refinement* from, sp_device_poses** out);
void sp_device_poses_destroy(sp_device_poses* dp);
/* Enqueues: the rasterizer's camera := view's corrected camera (instead of sp_set_camera). */
sp_status sp_device_poses_set_camera(sp_device_poses* dp, uint32_t view);
/* Enqueues: the refinement step of `view` (after its backward; rate_factor in (0, 1]), then
 * the rasterizer's camera := next_view's corrected camera. */
sp_status sp_device_poses_step(sp_device_poses* dp, uint32_t view, uint32_t next_view, float rate_factor);
/* Synchronises and copies the device state into `into` (a refinement over the same views);
 * SP_ERR_NONFINITE if a step met a non-finite pose gradient (that step changed nothing). */
sp_status sp_device_poses_download(sp_device_poses* dp, sp_pose_refinement* into);
/* Trainer::step_async with the poses refined on the device, without synchronising: forward
 * with the camera already in place (sp_device_poses_set_camera, or the previous step), loss
 * against `view`, backward + Adam (fused when `adam` steps the rasterizer's own
 * parameters), the pose step of `view` and the camera of next_view; if pinned_loss_sums
 * (4 doubles) is not NULL, the loss sums (L1, alpha, D-SSIM, total; divide by the pixel count
 * for the means) land in it asynchronously: written by the loss-sum kernel itself when it is
 * page-locked host memory (cudaHostAlloc, cudaHostRegister, torch's pin_memory), else copied
 * there from the device. */
sp_status sp_train_step_device_poses(sp_rasterizer* r, sp_adam* adam, sp_device_poses* dp, uint32_t view,
                                     uint32_t next_view, float position_rate_factor, double* pinned_loss_sums);


#ifdef __cplusplus
}
#endif

#endif
