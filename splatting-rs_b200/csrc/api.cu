// The C ABI of libsplat_b200 (include/splat.h): context, rasterizer and Adam objects that
// own their device buffers and enqueue the kernels of this directory on one CUDA stream.
// The host-side structure follows instantsplat-rs/src/rasterizer.rs (Rasterizer::new,
// encode_forward / encode_loss / encode_backward, the read-backs) and optimizer.rs (Adam).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda.h>

#include "densify.h"
#include "kernels.h"
#include "objects.h"
#include "pose_math.h"
#include "pose_state.h"

using namespace splat;

namespace {

template <typename T>
sp_status alloc(sp_rasterizer* r, T** out, size_t count, bool zero = true) {
    void* p = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t err = cudaMalloc(&p, bytes);
    if (err != cudaSuccess) return cuda_fail(r->ctx, err, "cudaMalloc");
    r->allocations.push_back(p);
    if (zero) {
        err = cudaMemset(p, 0, bytes);
        if (err != cudaSuccess) return cuda_fail(r->ctx, err, "cudaMemset");
    }
    *out = static_cast<T*>(p);
    return SP_OK;
}

uint32_t ceil_log2(uint64_t v) {
    uint32_t bits = 0;
    while ((1ull << bits) < v) ++bits;
    return bits;
}

sp_status read_device(sp_context* ctx, void* host, const void* device, size_t bytes) {
    if (!host) return fail(ctx, SP_ERR_INVALID, "null host buffer");
    if (bytes == 0) return SP_OK;
    SP_CUDA(ctx, cudaMemcpyAsync(host, device, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return sync_stream(ctx);
}

sp_status device_status(sp_rasterizer* r, DeviceMeta* meta_out) {
    DeviceMeta meta;
    sp_status s = read_device(r->ctx, &meta, r->meta, sizeof(meta));
    if (s != SP_OK) return s;
    if (meta_out) *meta_out = meta;
    if (meta.status != 0) {
        const sp_status status = (sp_status)meta.status;
        // Clear it so that later passes report their own.
        cudaMemsetAsync(&r->meta->status, 0, sizeof(uint32_t), r->ctx->stream);
        return fail(r->ctx, status, "a device-side wait gave up (sort look-back timeout)");
    }
    return SP_OK;
}

float position_rate_factor(uint64_t step, uint64_t steps) {
    const uint64_t denominator = std::max<uint64_t>(steps - 1, 1);
    return std::pow(SP_POSITION_RATE_FINAL_OVER_INITIAL, (float)step / (float)denominator);
}

void learning_rates_by_slot(const sp_learning_rates& rates, float position_scale, uint32_t stride, float* out) {
    // LearningRates::by_slot (optimizer.rs:82-100); the SH degree 1-3 slots take sh_rest.
    for (uint32_t slot = 0; slot < stride; ++slot) {
        float rate;
        if (slot < 3) rate = rates.position * position_scale;
        else if (slot < 6) rate = rates.log_scale;
        else if (slot < 10) rate = rates.rotation;
        else if (slot == 10) rate = rates.opacity;
        else if (slot < 14) rate = rates.sh_dc;
        else rate = rates.sh_rest;
        out[slot] = rate;
    }
}

}  // namespace

namespace splat {
// loss.cu: deterministic sum of the per-pixel loss terms into workspace[0..4) (the
// workspace holds 4 + 4 * 256 + 1 doubles); with `meta`, its status word and overflow flag
// are copied into status_dst[0..2); with mirror_dst (mapped page-locked host memory), the
// last block then copies mirror_words words from mirror_src there.
cudaError_t launch_loss_sums(const float4* pixel_loss, uint64_t pixels, double* workspace, double* result,
                             const DeviceMeta* meta, uint32_t* status_dst, cudaStream_t stream,
                             const uint32_t* mirror_src = nullptr, uint32_t* mirror_dst = nullptr,
                             uint32_t mirror_words = 0);
}  // namespace splat

extern "C" {

const char* sp_version(void) { return "splat_b200 0.1 (sm_100a)"; }

const char* sp_status_string(sp_status status) {
    switch (status) {
        case SP_OK: return "SP_OK";
        case SP_ERR_INVALID: return "SP_ERR_INVALID";
        case SP_ERR_TOO_MANY_TILES: return "SP_ERR_TOO_MANY_TILES";
        case SP_ERR_OVERFLOW: return "SP_ERR_OVERFLOW";
        case SP_ERR_TIMEOUT: return "SP_ERR_TIMEOUT";
        case SP_ERR_CUDA: return "SP_ERR_CUDA";
        case SP_ERR_NCCL: return "SP_ERR_NCCL";
        case SP_ERR_NONFINITE: return "SP_ERR_NONFINITE";
        case SP_ERR_NO_DEVICE: return "SP_ERR_NO_DEVICE";
        case SP_ERR_OUT_OF_MEMORY: return "SP_ERR_OUT_OF_MEMORY";
    }
    return "unknown status";
}

static sp_status context_create(int device, void* stream, sp_context** out) {
    if (!out) return SP_ERR_INVALID;
    *out = nullptr;
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) return SP_ERR_NO_DEVICE;
    if (device < 0 || device >= devices) return SP_ERR_INVALID;
    sp_context* ctx = new sp_context();
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess) {
        delete ctx;
        return SP_ERR_CUDA;
    }
    if (stream) {
        ctx->stream = static_cast<cudaStream_t>(stream);
    } else {
        if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
            delete ctx;
            return SP_ERR_CUDA;
        }
        ctx->own_stream = true;
    }
    *out = ctx;
    return SP_OK;
}

sp_status sp_context_create(int device, sp_context** out) { return context_create(device, nullptr, out); }

sp_status sp_context_create_on_stream(int device, void* stream, sp_context** out) {
    return context_create(device, stream, out);
}

void sp_context_destroy(sp_context* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (int k = 0; k < SP_K_COUNT; ++k)
        for (auto& pair : ctx->recorded[k]) {
            cudaEventDestroy(pair.first);
            cudaEventDestroy(pair.second);
        }
    for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
    if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

sp_status sp_context_sync(sp_context* ctx) {
    if (!ctx) return SP_ERR_INVALID;
    SP_CHECK(select_device(ctx));
    return sync_stream(ctx);
}

void* sp_context_stream(sp_context* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

const char* sp_last_error(const sp_context* ctx) { return ctx ? ctx->error.c_str() : "null context"; }

sp_status sp_camera_uniform_from_pinhole(const double rotation_c2w[9], const double translation[3],
                                         const double focal[2], const double principal_point[2], uint32_t width,
                                         uint32_t height, sp_camera_uniform* out) {
    if (!rotation_c2w || !translation || !focal || !principal_point || !out) return SP_ERR_INVALID;
    // camera.rs:46-70 (pose_math.h, shared with the device pose step).
    *out = splat::pose::uniform_of(rotation_c2w, translation, focal, principal_point, width, height);
    return SP_OK;
}

void sp_options_default(sp_options* out) {
    if (!out) return;
    std::memset(out, 0, sizeof(*out));
    out->key_mode = SP_KEYS_REF20;
    out->backward_mode = SP_BWD_ATOMIC;
    out->sh_degree = 0;
    out->intersections_per_gaussian = SP_INTERSECTIONS_PER_GAUSSIAN;
    out->accumulate_gradients = 0;
    out->loss_weights.l1 = SP_LOSS_L1;
    out->loss_weights.dssim = SP_LOSS_DSSIM;
    out->loss_weights.alpha = SP_LOSS_ALPHA;
    out->tile_culling = SP_TILES_RECTANGLE;
}

void sp_rasterizer_destroy(sp_rasterizer* r) {
    if (!r) return;
    cudaSetDevice(r->ctx->device);
    cudaStreamSynchronize(r->ctx->stream);
    for (void* p : r->allocations) cudaFree(p);
    if (r->readback) cudaFreeHost(r->readback);
    delete r;
}

sp_status sp_rasterizer_create(sp_context* ctx, const float* d_params, uint64_t gaussian_count, uint32_t width,
                               uint32_t height, const float* d_ground_truth, uint32_t view_count,
                               const sp_options* options, sp_rasterizer** out) {
    if (!ctx || !out) return SP_ERR_INVALID;
    *out = nullptr;
    sp_options opt;
    if (options) opt = *options;
    else sp_options_default(&opt);
    // rasterizer.rs:185-199.
    SP_REQUIRE(ctx, gaussian_count > 0, SP_ERR_INVALID, "no Gaussians");
    SP_REQUIRE(ctx, gaussian_count < (1ull << kGaussianBits), SP_ERR_INVALID, "2^28 Gaussians or more");
    SP_REQUIRE(ctx, d_params != nullptr, SP_ERR_INVALID, "null params buffer");
    SP_REQUIRE(ctx, width > 0 && height > 0, SP_ERR_INVALID, "empty image");
    SP_REQUIRE(ctx, view_count == 0 || d_ground_truth != nullptr, SP_ERR_INVALID, "null ground truth buffer");
    SP_REQUIRE(ctx, opt.sh_degree <= 3, SP_ERR_INVALID, "SH degree above 3");
    SP_REQUIRE(ctx, opt.key_mode == SP_KEYS_REF20 || opt.key_mode == SP_KEYS_FULL32, SP_ERR_INVALID, "key mode");
    SP_REQUIRE(ctx, opt.backward_mode == SP_BWD_DETERMINISTIC || opt.backward_mode == SP_BWD_ATOMIC, SP_ERR_INVALID,
               "backward mode");
    SP_REQUIRE(ctx, opt.intersections_per_gaussian > 0, SP_ERR_INVALID, "intersections per Gaussian");
    SP_REQUIRE(ctx, opt.tile_culling == SP_TILES_RECTANGLE || opt.tile_culling == SP_TILES_ELLIPSE, SP_ERR_INVALID,
               "tile culling");
    // The deterministic backward addresses its per-(Gaussian, tile) slots by the tile's index
    // in the Gaussian's rectangle.
    SP_REQUIRE(ctx, opt.tile_culling == SP_TILES_RECTANGLE || opt.backward_mode == SP_BWD_ATOMIC, SP_ERR_INVALID,
               "tile culling needs the atomic backward");
    const uint32_t tiles_x = (width + SP_TILE - 1) / SP_TILE, tiles_y = (height + SP_TILE - 1) / SP_TILE;
    SP_REQUIRE(ctx, tiles_x <= 0xffffu && tiles_y <= 0xffffu, SP_ERR_TOO_MANY_TILES,
               "over 65535 tiles on a side");
    const uint64_t capacity = gaussian_count * opt.intersections_per_gaussian;
    SP_REQUIRE(ctx, capacity < (1ull << 30), SP_ERR_INVALID, "intersection capacity must stay below 2^30");
    SP_CHECK(select_device(ctx));

    sp_rasterizer* r = new sp_rasterizer();
    r->ctx = ctx;
    r->params = d_params;
    r->n = gaussian_count;
    r->width = width;
    r->height = height;
    r->tiles_x = tiles_x;
    r->tiles_y = tiles_y;
    r->tiles = tiles_x * tiles_y;
    r->ground_truth = d_ground_truth;
    r->views = view_count;
    r->options = opt;
    r->stride = SP_PARAM_STRIDE(opt.sh_degree);
    r->capacity = capacity;
    r->blocks = (uint32_t)((gaussian_count + kBlock - 1) / kBlock);
    r->max_partitions = (uint32_t)((capacity + kSortPartition - 1) / kSortPartition);
    const uint32_t tile_bits = ceil_log2(r->tiles);
    r->plan.tile_bits = (int)tile_bits;
    // REF20 order: compressed 32-bit keys (tile << r) | (depth key - nearest), r the frame's
    // depth-key range (< 2^19), wherever tile_bits + 19 fits 32 bits (up to 8192 tiles);
    // beyond, and for FULL32, the reference's layout in 64 bits.
    r->plan.compressed = opt.key_mode == SP_KEYS_REF20 && (int)tile_bits + kMaxDepthRangeBits <= 32;
    r->plan.key_bits = (int)tile_bits + (r->plan.compressed            ? kMaxDepthRangeBits
                                         : opt.key_mode == SP_KEYS_FULL32 ? 32
                                                                          : SP_DEPTH_BITS);
    r->plan.key64 = r->plan.key_bits > 32 || opt.key_mode == SP_KEYS_FULL32;
    r->plan.passes = (r->plan.key_bits + 7) / 8;
    r->plan.tile_shift = opt.key_mode == SP_KEYS_FULL32 ? 32 : SP_DEPTH_BITS;

    const uint64_t n = gaussian_count, p = r->pixels();
    const size_t key_bytes = r->plan.key64 ? 8 : 4;
    sp_status s = SP_OK;
#define SP_ALLOC(ptr, count)                                  \
    if ((s = alloc(r, &(ptr), (count))) != SP_OK) {           \
        sp_rasterizer_destroy(r);                             \
        return s;                                             \
    }
    SP_ALLOC(r->records, n * kRecord);
    SP_ALLOC(r->reach, n);
    SP_ALLOC(r->radii, n);
    SP_ALLOC(r->offsets, n);
    SP_ALLOC(r->block_totals, r->blocks);
    SP_ALLOC(r->block_offsets, r->blocks);
    SP_ALLOC(r->meta, 1);
    {
        // An empty depth-key range for the first frame's projection to widen.
        const uint32_t empty = 0xffffffffu;
        const cudaError_t err = cudaMemcpy(&r->meta->depth_lo, &empty, sizeof(empty), cudaMemcpyHostToDevice);
        if (err != cudaSuccess) {
            sp_rasterizer_destroy(r);
            return cuda_fail(ctx, err, "meta");
        }
    }
    {
        unsigned char* k0 = nullptr;
        unsigned char* k1 = nullptr;
        SP_ALLOC(k0, capacity * key_bytes);
        SP_ALLOC(k1, capacity * key_bytes);
        r->keys[0] = k0;
        r->keys[1] = k1;
    }
    SP_ALLOC(r->values[0], capacity);
    SP_ALLOC(r->values[1], capacity);
    SP_ALLOC(r->sort_histograms, (size_t)kSortMaxPasses * kSortRadix);
    SP_ALLOC(r->sort_tickets, kSortMaxPasses);
    SP_ALLOC(r->lookback, (size_t)std::max<uint32_t>(r->max_partitions, 1) * kSortRadix);
    SP_ALLOC(r->ranges, r->tiles);
    SP_ALLOC(r->tile_order, r->tiles);
    SP_ALLOC(r->camera_dev, 1);
    SP_ALLOC(r->image, p);
    SP_ALLOC(r->contributions, p);
    SP_ALLOC(r->ssim_partials, p * 3);
    SP_ALLOC(r->loss_gradient, p);
    SP_ALLOC(r->pixel_loss, p);
    SP_ALLOC(r->loss_sums, 4 + 4 * 256 + 1);
    SP_ALLOC(r->readback_dev, 1);
    r->camera_gradient = r->readback_dev->camera;
    r->loss_result = r->readback_dev->loss;
    if (opt.backward_mode == SP_BWD_DETERMINISTIC) {
        SP_ALLOC(r->slot_gradients, capacity * SP_GRAD_STRIDE);
    } else {
        SP_ALLOC(r->gaussian_gradients, n * 3);
    }
    SP_ALLOC(r->param_gradients, n * r->stride);
    SP_ALLOC(r->camera_partials, (size_t)r->blocks * SP_CAMERA_GRAD_STRIDE);
    SP_ALLOC(r->camera_done, 1);
    SP_ALLOC(r->densify_stats, n);
#undef SP_ALLOC
    {
        const cudaError_t err = cudaMallocHost(&r->readback, sizeof(sp_rasterizer::StepReadback));
        if (err != cudaSuccess) {
            sp_rasterizer_destroy(r);
            return cuda_fail(ctx, err, "cudaMallocHost");
        }
        // Its device view, for the loss-sum kernel to fill it directly (none: a copy does).
        if (cudaHostGetDevicePointer(&r->readback_mapped, r->readback, 0) != cudaSuccess) {
            r->readback_mapped = nullptr;
            cudaGetLastError();
        }
    }
    // The default camera of rasterizer.rs:202-213: identity pose, unit focal.
    const double identity[9] = {1, 0, 0, 0, 1, 0, 0, 0, 1}, zero[3] = {0, 0, 0}, unit[2] = {1, 1}, origin[2] = {0, 0};
    sp_camera_uniform_from_pinhole(identity, zero, unit, origin, width, height, &r->camera);
    {
        const cudaError_t err = cudaMemcpy(r->camera_dev, &r->camera, sizeof(sp_camera_uniform), cudaMemcpyHostToDevice);
        if (err != cudaSuccess) {
            sp_rasterizer_destroy(r);
            return cuda_fail(ctx, err, "camera upload");
        }
    }
    r->has_camera = true;
    *out = r;
    return SP_OK;
}

uint32_t sp_rasterizer_param_stride(const sp_rasterizer* r) { return r ? r->stride : 0; }

sp_status sp_set_camera(sp_rasterizer* r, const sp_camera_uniform* camera) {
    if (!r || !camera) return SP_ERR_INVALID;
    // rasterizer.rs:399.
    SP_REQUIRE(r->ctx, camera->width == r->width && camera->height == r->height, SP_ERR_INVALID, "camera image size");
    SP_REQUIRE(r->ctx, camera->tiles_x == r->tiles_x && camera->tiles_y == r->tiles_y, SP_ERR_INVALID,
               "camera tile grid");
    r->camera = *camera;
    r->camera_on_device = false;
    return SP_OK;
}

sp_status sp_forward(sp_rasterizer* r) {
    NvtxRange range("sp_forward");
    if (!r) return SP_ERR_INVALID;
    sp_context* ctx = r->ctx;
    SP_CHECK(select_device(ctx));
    cudaStream_t st = ctx->stream;
    {
        KernelSpan span(ctx, SP_K_PROJECT);
        SP_CUDA(ctx, launch_project(r->params, r->n, (int)r->options.sh_degree, r->camera,
                                    r->camera_on_device ? r->camera_dev : nullptr, r->records, r->radii, r->offsets,
                                    r->block_totals, r->plan.compressed ? r->meta : nullptr, r->reach,
                                    (int)r->options.tile_culling, st));
    }
    {
        KernelSpan span(ctx, SP_K_SCAN);
        SP_CUDA(ctx, launch_scan_blocks(r->block_totals, r->block_offsets, r->blocks, r->capacity, r->meta,
                                        r->sort_histograms, r->sort_tickets, r->plan, st));
    }
    {
        KernelSpan span(ctx, SP_K_EMIT);
        SP_CUDA(ctx, launch_emit(r->records, r->reach, r->offsets, r->block_offsets, r->n, r->camera,
                                 (int)r->options.key_mode, (int)r->options.tile_culling, r->plan, r->meta, r->keys[0],
                                 r->keys[1], r->values[0], r->values[1], r->sort_histograms, st));
    }
    // Passes past the frame's key width return at once; the result lands in buffer passes & 1.
    for (int pass = 0; pass < r->plan.passes; ++pass) {
        KernelSpan span(ctx, SP_K_SORT);
        SP_CUDA(ctx, launch_sort_pass(r->plan, pass, ++r->sequence, r->keys[0], r->values[0], r->keys[1],
                                      r->values[1], r->sort_histograms, r->sort_tickets, r->lookback,
                                      r->max_partitions, r->meta, st));
    }
    r->sorted_buffer = r->plan.passes & 1;
    {
        KernelSpan span(ctx, SP_K_RANGES);
        SP_CUDA(ctx,
                launch_ranges(r->plan, r->keys[r->sorted_buffer], r->meta, r->capacity, r->ranges, r->tiles, st));
    }
    {
        KernelSpan span(ctx, SP_K_TILE_ORDER);
        SP_CUDA(ctx, launch_tile_order(r->ranges, r->tiles, r->tile_order, st));
    }
    {
        KernelSpan span(ctx, SP_K_BLEND_FORWARD);
        SP_CUDA(ctx, launch_blend_forward(r->records, r->values[r->sorted_buffer], r->ranges, r->tile_order,
                                          r->camera, r->image, r->contributions, st));
    }
    r->forward_done = true;
    return SP_OK;
}

sp_status sp_loss(sp_rasterizer* r, uint32_t view) {
    NvtxRange range("sp_loss");
    if (!r) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, view < r->views, SP_ERR_INVALID, "view index out of range");
    SP_CHECK(select_device(r->ctx));
    const float4* gt = reinterpret_cast<const float4*>(r->ground_truth) + (size_t)view * r->pixels();
    {
        KernelSpan span(r->ctx, SP_K_SSIM);
        SP_CUDA(r->ctx, launch_ssim(r->image, gt, r->width, r->height, r->ssim_partials, r->ctx->stream));
    }
    {
        KernelSpan span(r->ctx, SP_K_LOSS);
        const bool clear = r->options.backward_mode == SP_BWD_ATOMIC;
        SP_CUDA(r->ctx, launch_loss(r->image, gt, r->ssim_partials, r->width, r->height, r->options.loss_weights,
                                    r->loss_gradient, r->pixel_loss, clear ? r->gaussian_gradients : nullptr,
                                    clear ? r->n * 3 : 0, r->ctx->stream));
        r->blend_sums_zero = clear;
    }
    return SP_OK;
}

namespace {

// The blend backward (K8) of sp_backward and sp_backward_adam.
sp_status blend_backward(sp_rasterizer* r) {
    cudaStream_t st = r->ctx->stream;
    KernelSpan span(r->ctx, SP_K_BLEND_BACKWARD);
    // The sums start at zero: zeroed by this view's sp_loss (k_loss), else here.
    if (r->options.backward_mode == SP_BWD_ATOMIC && !r->blend_sums_zero)
        SP_CUDA(r->ctx, cudaMemsetAsync(r->gaussian_gradients, 0, r->n * 3 * sizeof(float4), st));
    r->blend_sums_zero = false;
    SP_CUDA(r->ctx, launch_blend_backward((int)r->options.backward_mode, r->records, r->values[r->sorted_buffer],
                                          r->ranges, r->tile_order, r->offsets, r->camera, r->image,
                                          r->contributions, r->loss_gradient, r->slot_gradients,
                                          r->gaussian_gradients, st));
    return SP_OK;
}

}  // namespace

sp_status sp_backward_adam(sp_rasterizer* r, sp_adam* adam, float position_rate_factor) {
    NvtxRange range("sp_backward_adam");
    if (!r || !adam) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, r->forward_done, SP_ERR_INVALID, "backward before any forward pass");
    SP_REQUIRE(r->ctx,
               adam->params == r->params && adam->gradients == r->param_gradients && adam->n == r->n &&
                   adam->stride == r->stride,
               SP_ERR_INVALID, "the Adam state does not belong to this rasterizer's parameters");
    SP_REQUIRE(r->ctx, !r->options.accumulate_gradients, SP_ERR_INVALID,
               "a fused step cannot accumulate gradients over views");
    SP_CHECK(select_device(r->ctx));
    SP_CHECK(sp_adam_advance(adam, position_rate_factor));
    SP_CHECK(blend_backward(r));
    AdamLaunch step{adam->params, adam->first_moment, adam->second_moment, adam->lr_by_slot.data(),
                    adam->bias1, adam->bias2, adam->max_log_scale, adam->max_log_anisotropy};
    KernelSpan span(r->ctx, SP_K_BACKWARD_ADAM);
    SP_CUDA(r->ctx, launch_project_backward(r->params, r->n, (int)r->options.sh_degree, (int)r->options.backward_mode,
                                            r->camera, r->camera_on_device ? r->camera_dev : nullptr, r->records,
                                            r->radii, r->offsets, r->slot_gradients,
                                            r->capacity, r->gaussian_gradients, r->param_gradients, 0,
                                            r->camera_partials, r->camera_done, r->camera_gradient,
                                            r->densify_stats, &step, 0, r->n, r->ctx->stream));
    return SP_OK;
}

sp_status sp_backward_blend(sp_rasterizer* r) {
    if (!r) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, r->forward_done, SP_ERR_INVALID, "backward before any forward pass");
    SP_CHECK(select_device(r->ctx));
    return blend_backward(r);
}

sp_status sp_backward_project(sp_rasterizer* r, uint64_t first, uint64_t count) {
    if (!r) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, r->forward_done, SP_ERR_INVALID, "backward before any forward pass");
    SP_REQUIRE(r->ctx, first % kBlock == 0 && first <= r->n && count <= r->n - first, SP_ERR_INVALID,
               "range: first a multiple of 256, inside the Gaussians");
    SP_CHECK(select_device(r->ctx));
    KernelSpan span(r->ctx, SP_K_PROJECT_BACKWARD);
    SP_CUDA(r->ctx, launch_project_backward(r->params, r->n, (int)r->options.sh_degree, (int)r->options.backward_mode,
                                            r->camera, r->camera_on_device ? r->camera_dev : nullptr, r->records,
                                            r->radii, r->offsets, r->slot_gradients, r->capacity,
                                            r->gaussian_gradients, r->param_gradients,
                                            (int)r->options.accumulate_gradients, r->camera_partials, r->camera_done,
                                            r->camera_gradient, r->densify_stats, nullptr, first, count,
                                            r->ctx->stream));
    return SP_OK;
}

sp_status sp_backward(sp_rasterizer* r) {
    NvtxRange range("sp_backward");
    if (!r) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, r->forward_done, SP_ERR_INVALID, "backward before any forward pass");
    SP_CHECK(select_device(r->ctx));
    cudaStream_t st = r->ctx->stream;
    SP_CHECK(blend_backward(r));
    {
        KernelSpan span(r->ctx, SP_K_PROJECT_BACKWARD);
        SP_CUDA(r->ctx, launch_project_backward(
                            r->params, r->n, (int)r->options.sh_degree, (int)r->options.backward_mode, r->camera,
                            r->camera_on_device ? r->camera_dev : nullptr,
                            r->records, r->radii, r->offsets, r->slot_gradients, r->capacity, r->gaussian_gradients,
                            r->param_gradients, (int)r->options.accumulate_gradients, r->camera_partials,
                            r->camera_done, r->camera_gradient, r->densify_stats, nullptr, 0, r->n, st));
    }
    return SP_OK;
}

static sp_status write_pixels(sp_rasterizer* r, float4* dst, const float* src, int src_is_device) {
    if (!r || !src) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, cudaMemcpyAsync(dst, src, r->pixels() * sizeof(float4),
                                    src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                    r->ctx->stream));
    if (!src_is_device) return sync_stream(r->ctx);
    return SP_OK;
}

sp_status sp_write_loss_gradient(sp_rasterizer* r, const float* src, int src_is_device) {
    return write_pixels(r, r ? r->loss_gradient : nullptr, src, src_is_device);
}

sp_status sp_write_image(sp_rasterizer* r, const float* src, int src_is_device) {
    return write_pixels(r, r ? r->image : nullptr, src, src_is_device);
}

sp_status sp_write_densify_stats(sp_rasterizer* r, const sp_densify_stats* host) {
    if (!r || !host) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, cudaMemcpyAsync(r->densify_stats, host, r->n * sizeof(float4), cudaMemcpyHostToDevice,
                                    r->ctx->stream));
    return sync_stream(r->ctx);
}

float* sp_param_gradients(sp_rasterizer* r) { return r ? r->param_gradients : nullptr; }

float* sp_camera_gradient_device(sp_rasterizer* r) { return r ? r->camera_gradient : nullptr; }

sp_densify_stats* sp_densify_stats_device(sp_rasterizer* r) {
    return r ? reinterpret_cast<sp_densify_stats*>(r->densify_stats) : nullptr;
}

sp_status sp_zero_param_gradients(sp_rasterizer* r) {
    if (!r) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, cudaMemsetAsync(r->param_gradients, 0, r->n * r->stride * sizeof(float), r->ctx->stream));
    return SP_OK;
}

sp_status sp_clear_densify_stats(sp_rasterizer* r) {
    if (!r) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, cudaMemsetAsync(r->densify_stats, 0, r->n * sizeof(float4), r->ctx->stream));
    return SP_OK;
}

sp_status sp_read_loss_gradient(sp_rasterizer* r, float* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->loss_gradient, r->pixels() * sizeof(float4));
}

sp_status sp_read_param_gradients(sp_rasterizer* r, float* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->param_gradients, r->n * r->stride * sizeof(float));
}

sp_status sp_read_densify_stats(sp_rasterizer* r, sp_densify_stats* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->densify_stats, r->n * sizeof(float4));
}

sp_status sp_read_camera_gradient(sp_rasterizer* r, sp_camera_gradient* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->camera_gradient, SP_CAMERA_GRAD_STRIDE * sizeof(float));
}

sp_status sp_read_image(sp_rasterizer* r, float* host_rgbt) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host_rgbt, r->image, r->pixels() * sizeof(float4));
}

sp_status sp_read_pixel_loss(sp_rasterizer* r, float* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->pixel_loss, r->pixels() * sizeof(float4));
}

static sp_status overflow_error(sp_rasterizer* r);

sp_status sp_read_loss(sp_rasterizer* r, sp_loss_terms* out) {
    if (!r || !out) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    // LossTerms::from_pixel_loss (loss.rs:49-63): means in f64, summed on the device.
    SP_CUDA(r->ctx, launch_loss_sums(r->pixel_loss, r->pixels(), r->loss_sums, r->loss_result, nullptr, nullptr,
                                     r->ctx->stream));
    double sums[4];
    SP_CHECK(read_device(r->ctx, sums, r->loss_result, sizeof(sums)));
    const double pixels = (double)r->pixels();
    out->l1 = (float)(sums[0] / pixels);
    out->alpha = (float)(sums[1] / pixels);
    out->dssim = (float)(sums[2] / pixels);
    out->total = (float)(sums[3] / pixels);
    // The loss of a frame rendered from truncated lists, or after a device-side wait gave up,
    // comes with the error (the terms are filled in all the same).
    DeviceMeta meta;
    SP_CHECK(device_status(r, &meta));
    if (meta.overflow) return overflow_error(r);
    return SP_OK;
}

static sp_status overflow_error(sp_rasterizer* r) {
    DeviceMeta meta{};
    const bool known = read_device(r->ctx, &meta, r->meta, sizeof(meta)) == SP_OK;
    const uint64_t needed = ((uint64_t)meta.total_hi << 32) | meta.total_lo;
    return fail(r->ctx, SP_ERR_OVERFLOW,
                "intersection list overflow: " + (known ? std::to_string(needed) : std::string("more than ")) +
                    (known ? " (Gaussian, tile) pairs, " : "") + "the capacity is " + std::to_string(r->capacity) +
                    "; Gaussians are too large for the image, or reserve more with sp_reserve_intersections");
}

sp_status sp_intersections_needed(sp_rasterizer* r, uint64_t* total) {
    if (!r || !total) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    DeviceMeta meta;
    SP_CHECK(read_device(r->ctx, &meta, r->meta, sizeof(meta)));
    *total = ((uint64_t)meta.total_hi << 32) | meta.total_lo;
    return SP_OK;
}

sp_status sp_reserve_intersections(sp_rasterizer* r, uint64_t capacity) {
    if (!r) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, capacity < (1ull << 32), SP_ERR_INVALID, "2^32 intersections or more");
    if (capacity <= r->capacity) return SP_OK;
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, cudaStreamSynchronize(r->ctx->stream));
    const uint32_t partitions = (uint32_t)((capacity + kSortPartition - 1) / kSortPartition);
    const size_t key_bytes = r->plan.key64 ? 8 : 4;
    // Every capacity-sized buffer: the key and value ping-pong pairs, the sort's look-back
    // words and (deterministic backward) the per-slot gradients. The new ones are allocated
    // first, so that a failure leaves the rasterizer as it was.
    void** slots[6] = {&r->keys[0], &r->keys[1], reinterpret_cast<void**>(&r->values[0]),
                       reinterpret_cast<void**>(&r->values[1]), reinterpret_cast<void**>(&r->lookback),
                       reinterpret_cast<void**>(&r->slot_gradients)};
    const size_t bytes[6] = {capacity * key_bytes, capacity * key_bytes, capacity * sizeof(uint32_t),
                             capacity * sizeof(uint32_t),
                             (size_t)std::max<uint32_t>(partitions, 1) * kSortRadix * sizeof(unsigned long long),
                             r->slot_gradients ? capacity * SP_GRAD_STRIDE * sizeof(float) : 0};
    void* fresh[6] = {};
    for (int k = 0; k < 6; ++k) {
        if (bytes[k] == 0) continue;
        cudaError_t err = cudaMalloc(&fresh[k], bytes[k]);
        if (err == cudaSuccess && k == 4) err = cudaMemset(fresh[k], 0, bytes[k]);
        if (err != cudaSuccess) {
            for (int j = 0; j <= k; ++j)
                if (fresh[j]) cudaFree(fresh[j]);
            return cuda_fail(r->ctx, err, "cudaMalloc (sp_reserve_intersections)");
        }
    }
    for (int k = 0; k < 6; ++k) {
        if (!fresh[k]) continue;
        void* old = *slots[k];
        auto at = std::find(r->allocations.begin(), r->allocations.end(), old);
        if (at != r->allocations.end()) r->allocations.erase(at);
        cudaFree(old);
        *slots[k] = fresh[k];
        r->allocations.push_back(fresh[k]);
    }
    r->capacity = capacity;
    r->max_partitions = partitions;
    r->forward_done = false;  // the lists of the last forward pass are gone
    return SP_OK;
}

sp_status sp_read_intersections(sp_rasterizer* r, sp_intersection_meta* out) {
    if (!r || !out) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    DeviceMeta meta;
    SP_CHECK(device_status(r, &meta));
    out->count = meta.count;
    out->sort_blocks = meta.sort_blocks;
    out->histogram_length = meta.histogram_length;
    out->overflow = meta.overflow;
    out->capacity = meta.capacity;
    // rasterizer.rs:536-544.
    if (meta.overflow) return overflow_error(r);
    return SP_OK;
}

sp_status sp_train_step(sp_rasterizer* r, sp_adam* adam, const sp_camera_uniform* camera, uint32_t view,
                        float position_rate_factor, sp_camera_gradient* camera_gradient_out, sp_loss_terms* loss_out) {
    NvtxRange range("sp_train_step");
    if (!r || !adam || !camera) return SP_ERR_INVALID;
    SP_CHECK(sp_set_camera(r, camera));
    SP_CHECK(sp_forward(r));
    SP_CHECK(sp_loss(r, view));
    if (!r->options.accumulate_gradients && adam->params == r->params && adam->gradients == r->param_gradients) {
        SP_CHECK(sp_backward_adam(r, adam, position_rate_factor));
    } else {
        SP_CHECK(sp_backward(r));
        SP_CHECK(sp_adam_step(adam, position_rate_factor));
    }
    if (!camera_gradient_out && !loss_out) return SP_OK;
    cudaStream_t st = r->ctx->stream;
    if (loss_out) {
        // The loss-sum kernel also copies the step's status next to the camera gradient and the
        // sums, then the whole read-back into the page-locked host struct itself (its device
        // view): no copy follows the step's last kernel (else one copy brings it).
        const uint32_t words = (uint32_t)(sizeof(sp_rasterizer::StepReadback) / sizeof(uint32_t));
        SP_CUDA(r->ctx, launch_loss_sums(r->pixel_loss, r->pixels(), r->loss_sums, r->loss_result, r->meta,
                                         &r->readback_dev->status, st,
                                         reinterpret_cast<const uint32_t*>(r->readback_dev),
                                         reinterpret_cast<uint32_t*>(r->readback_mapped), words));
        if (!r->readback_mapped)
            SP_CUDA(r->ctx,
                    cudaMemcpyAsync(r->readback, r->readback_dev, sizeof(*r->readback), cudaMemcpyDeviceToHost, st));
    } else {
        SP_CUDA(r->ctx, cudaMemcpyAsync(&r->readback->status, &r->meta->status, sizeof(uint32_t),
                                        cudaMemcpyDeviceToHost, st));
        SP_CUDA(r->ctx, cudaMemcpyAsync(&r->readback->overflow, &r->meta->overflow, sizeof(uint32_t),
                                        cudaMemcpyDeviceToHost, st));
        SP_CUDA(r->ctx, cudaMemcpyAsync(r->readback->camera, r->camera_gradient, sizeof(r->readback->camera),
                                        cudaMemcpyDeviceToHost, st));
    }
    SP_CHECK(sync_stream(r->ctx));
    if (r->readback->status != 0) return device_status(r, nullptr);
    // The step trained on a truncated intersection list: the error of the reference's
    // read_step_async -> read_intersections_async (training.rs:271, rasterizer.rs:536-544).
    if (r->readback->overflow) return overflow_error(r);
    if (camera_gradient_out) std::memcpy(camera_gradient_out, r->readback->camera, sizeof(sp_camera_gradient));
    if (loss_out) {
        const double pixels = (double)r->pixels();
        loss_out->l1 = (float)(r->readback->loss[0] / pixels);
        loss_out->alpha = (float)(r->readback->loss[1] / pixels);
        loss_out->dssim = (float)(r->readback->loss[2] / pixels);
        loss_out->total = (float)(r->readback->loss[3] / pixels);
    }
    return SP_OK;
}

sp_status sp_train_step_host_poses(sp_rasterizer* r, sp_adam* adam, sp_pose_refinement* poses, uint32_t view,
                                   float position_rate_factor, sp_loss_terms* loss_out) {
    if (!r || !adam || !poses || view >= poses->initial.size()) return SP_ERR_INVALID;
    // training.rs:197-209 with pose refinement: the view's corrected camera, the step, the
    // camera gradient read back, the host pose step (pose_refinement.rs:113-163).
    const sp_camera_uniform camera = splat::pose::uniform_of(
        splat::pose::corrected(poses->initial[view], poses->views[view].correction, poses->shared.focal_log_scale));
    sp_camera_gradient gradient;
    SP_CHECK(sp_train_step(r, adam, &camera, view, position_rate_factor, &gradient, loss_out));
    const sp_status status = sp_pose_refinement_step(poses, view, &gradient, position_rate_factor);
    if (status != SP_OK) return fail(r->ctx, status, "pose step: non-finite pose gradient");
    return SP_OK;
}

// ------------------------------------------------------------------ device pose refinement

struct sp_device_poses {
    sp_rasterizer* r = nullptr;
    uint32_t views = 0;
    sp_pinhole_camera* initial = nullptr;
    splat::pose::ViewState* states = nullptr;
    splat::pose::SharedState* shared = nullptr;
};

void sp_device_poses_destroy(sp_device_poses* dp) {
    if (!dp) return;
    cudaSetDevice(dp->r->ctx->device);
    cudaStreamSynchronize(dp->r->ctx->stream);
    cudaFree(dp->initial);
    cudaFree(dp->states);
    cudaFree(dp->shared);
    delete dp;
}

sp_status sp_device_poses_create(sp_rasterizer* r, const sp_pose_refinement* from, sp_device_poses** out) {
    if (!r || !from || !out) return SP_ERR_INVALID;
    *out = nullptr;
    const uint32_t views = (uint32_t)from->initial.size();
    SP_REQUIRE(r->ctx, views > 0, SP_ERR_INVALID, "no views");
    for (const sp_pinhole_camera& c : from->initial)
        SP_REQUIRE(r->ctx, c.width == r->width && c.height == r->height, SP_ERR_INVALID, "camera image size");
    SP_CHECK(select_device(r->ctx));
    sp_device_poses* dp = new sp_device_poses();
    dp->r = r;
    dp->views = views;
    cudaError_t err = cudaMalloc(&dp->initial, views * sizeof(sp_pinhole_camera));
    if (err == cudaSuccess) err = cudaMalloc(&dp->states, views * sizeof(splat::pose::ViewState));
    if (err == cudaSuccess) err = cudaMalloc(&dp->shared, sizeof(splat::pose::SharedState));
    if (err == cudaSuccess)
        err = cudaMemcpy(dp->initial, from->initial.data(), views * sizeof(sp_pinhole_camera), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(dp->states, from->views.data(), views * sizeof(splat::pose::ViewState), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(dp->shared, &from->shared, sizeof(splat::pose::SharedState), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        sp_device_poses_destroy(dp);
        return cuda_fail(r->ctx, err, "device pose state");
    }
    *out = dp;
    return SP_OK;
}

sp_status sp_device_poses_set_camera(sp_device_poses* dp, uint32_t view) {
    if (!dp) return SP_ERR_INVALID;
    sp_rasterizer* r = dp->r;
    SP_REQUIRE(r->ctx, view < dp->views, SP_ERR_INVALID, "view index out of range");
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, launch_pose_step(dp->initial, dp->states, dp->shared, r->camera_gradient, dp->views, dp->views,
                                     view, 0.0, r->camera_dev, r->ctx->stream));
    r->camera_on_device = true;
    return SP_OK;
}

sp_status sp_device_poses_step(sp_device_poses* dp, uint32_t view, uint32_t next_view, float rate_factor) {
    if (!dp) return SP_ERR_INVALID;
    sp_rasterizer* r = dp->r;
    SP_REQUIRE(r->ctx, view < dp->views && next_view < dp->views, SP_ERR_INVALID, "view index out of range");
    // pose_refinement.rs:113-163.
    SP_REQUIRE(r->ctx, rate_factor > 0.0f && rate_factor <= 1.0f, SP_ERR_INVALID,
               "position rate factor must be in (0, 1]");
    SP_CHECK(select_device(r->ctx));
    SP_CUDA(r->ctx, launch_pose_step(dp->initial, dp->states, dp->shared, r->camera_gradient, dp->views, view,
                                     next_view, (double)rate_factor, r->camera_dev, r->ctx->stream));
    r->camera_on_device = true;
    return SP_OK;
}

sp_status sp_device_poses_download(sp_device_poses* dp, sp_pose_refinement* into) {
    if (!dp || !into || into->initial.size() != dp->views) return SP_ERR_INVALID;
    sp_rasterizer* r = dp->r;
    SP_CHECK(select_device(r->ctx));
    SP_CHECK(read_device(r->ctx, into->views.data(), dp->states, dp->views * sizeof(splat::pose::ViewState)));
    splat::pose::SharedState shared;
    SP_CHECK(read_device(r->ctx, &shared, dp->shared, sizeof(shared)));
    into->shared = shared;
    if (shared.status != 0) return fail(r->ctx, (sp_status)shared.status, "a device pose step met a non-finite gradient");
    return SP_OK;
}

sp_status sp_train_step_device_poses(sp_rasterizer* r, sp_adam* adam, sp_device_poses* dp, uint32_t view,
                                     uint32_t next_view, float position_rate_factor, double* pinned_loss_sums) {
    if (!r || !adam || !dp || dp->r != r) return SP_ERR_INVALID;
    SP_CHECK(sp_forward(r));
    SP_CHECK(sp_loss(r, view));
    if (adam->params == r->params && adam->gradients == r->param_gradients && adam->n == r->n) {
        SP_CHECK(sp_backward_adam(r, adam, position_rate_factor));
    } else {
        SP_CHECK(sp_backward(r));
        SP_CHECK(sp_adam_step(adam, position_rate_factor));
    }
    SP_CHECK(sp_device_poses_step(dp, view, next_view, position_rate_factor));
    if (pinned_loss_sums) {
        cudaStream_t st = r->ctx->stream;
        // Page-locked host memory the device can address: the loss-sum kernel writes the sums
        // there itself, so no copy breaks the launch chain into the next step. Other memory
        // takes the device buffer and an asynchronous copy.
        cudaPointerAttributes attributes{};
        double* direct = nullptr;
        if (cudaPointerGetAttributes(&attributes, pinned_loss_sums) == cudaSuccess &&
            attributes.type == cudaMemoryTypeHost && attributes.devicePointer)
            direct = static_cast<double*>(attributes.devicePointer);
        else
            cudaGetLastError();  // an address CUDA does not know: not an error, the copy serves
        SP_CUDA(r->ctx, launch_loss_sums(r->pixel_loss, r->pixels(), r->loss_sums, direct ? direct : r->loss_result,
                                         nullptr, nullptr, st));
        if (!direct)
            SP_CUDA(r->ctx,
                    cudaMemcpyAsync(pinned_loss_sums, r->loss_result, 4 * sizeof(double), cudaMemcpyDeviceToHost, st));
    }
    return SP_OK;
}

sp_status sp_render(sp_rasterizer* r, const sp_camera_uniform* camera, float* host_rgbt) {
    NvtxRange range("sp_render");
    if (!r) return SP_ERR_INVALID;
    SP_CHECK(sp_set_camera(r, camera));
    SP_CHECK(sp_forward(r));
    sp_intersection_meta meta;
    SP_CHECK(sp_read_intersections(r, &meta));
    return sp_read_image(r, host_rgbt);
}

sp_status sp_read_projected(sp_rasterizer* r, sp_projected* host) {
    if (!r || !host) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    sp_projected* tmp = nullptr;
    SP_CUDA(r->ctx, cudaMallocAsync((void**)&tmp, r->n * sizeof(sp_projected), r->ctx->stream));
    cudaError_t err = launch_to_projected(r->records, r->radii, r->n, tmp, r->ctx->stream);
    sp_status s = err == cudaSuccess ? read_device(r->ctx, host, tmp, r->n * sizeof(sp_projected))
                                     : cuda_fail(r->ctx, err, "launch_to_projected");
    cudaFreeAsync(tmp, r->ctx->stream);
    cudaStreamSynchronize(r->ctx->stream);
    return s;
}

sp_status sp_read_sorted_intersections(sp_rasterizer* r, uint64_t* keys_host, uint32_t* gaussians_host) {
    if (!r || !keys_host || !gaussians_host) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    DeviceMeta meta;
    SP_CHECK(device_status(r, &meta));
    const uint64_t count = meta.count;
    if (r->plan.key64) {
        SP_CHECK(read_device(r->ctx, keys_host, r->keys[r->sorted_buffer], count * 8));
    } else {
        std::vector<uint32_t> keys(count);
        SP_CHECK(read_device(r->ctx, keys.data(), r->keys[r->sorted_buffer], count * 4));
        if (r->plan.compressed) {
            // Back to the reference's layout: (tile << 20) | depth key.
            const uint32_t mask = meta.key_shift ? (uint32_t)((1ull << meta.key_shift) - 1) : 0u;
            for (uint64_t i = 0; i < count; ++i)
                keys_host[i] = ((uint64_t)(keys[i] >> meta.key_shift) << SP_DEPTH_BITS) |
                               (uint64_t)((keys[i] & mask) + meta.key_base);
        } else {
            for (uint64_t i = 0; i < count; ++i) keys_host[i] = keys[i];
        }
    }
    SP_CHECK(read_device(r->ctx, gaussians_host, r->values[r->sorted_buffer], count * 4));
    // The Gaussian indices without the blend kernels' block bits.
    for (uint64_t i = 0; i < count; ++i) gaussians_host[i] &= kGaussianMask;
    return SP_OK;
}

sp_status sp_read_tile_ranges(sp_rasterizer* r, uint32_t* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->ranges, (size_t)r->tiles * sizeof(uint2));
}

sp_status sp_read_contributions(sp_rasterizer* r, uint32_t* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->contributions, r->pixels() * sizeof(uint32_t));
}

sp_status sp_read_tile_offsets(sp_rasterizer* r, uint32_t* host) {
    if (!r) return SP_ERR_INVALID;
    return read_device(r->ctx, host, r->offsets, r->n * sizeof(uint32_t));
}

sp_status sp_read_gaussian_blend_gradients(sp_rasterizer* r, float* host) {
    if (!r || !host) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    const uint64_t n = r->n;
    if (r->options.backward_mode == SP_BWD_ATOMIC) {
        std::vector<float4> sums(n * 3);
        SP_CHECK(read_device(r->ctx, sums.data(), r->gaussian_gradients, n * 3 * sizeof(float4)));
        for (uint64_t g = 0; g < n; ++g) {
            const float4 a = sums[g * 3], b = sums[g * 3 + 1], c = sums[g * 3 + 2];
            const float v[SP_GRAD_STRIDE] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, 0.0f};
            std::memcpy(host + g * SP_GRAD_STRIDE, v, sizeof(v));
        }
        return SP_OK;
    }
    // Deterministic mode: each Gaussian's slots, in slot order (project_backward.wgsl:38-55).
    std::vector<float4> records(n * kRecord);
    std::vector<uint32_t> offsets(n), radii(n);
    std::vector<float> slots(r->capacity * SP_GRAD_STRIDE);
    SP_CHECK(read_device(r->ctx, records.data(), r->records, n * kRecord * sizeof(float4)));
    SP_CHECK(read_device(r->ctx, offsets.data(), r->offsets, n * 4));
    SP_CHECK(read_device(r->ctx, radii.data(), r->radii, n * 4));
    SP_CHECK(read_device(r->ctx, slots.data(), r->slot_gradients, slots.size() * sizeof(float)));
    for (uint64_t g = 0; g < n; ++g) {
        float v[SP_GRAD_STRIDE] = {0};
        if (radii[g] != 0) {
            uint32_t lo, hi;
            std::memcpy(&lo, &records[g * kRecord + 2].z, 4);
            std::memcpy(&hi, &records[g * kRecord + 2].w, 4);
            const uint32_t count = ((hi & 0xffffu) - (lo & 0xffffu)) * ((hi >> 16) - (lo >> 16));
            for (uint32_t k = 0; k < count; ++k) {
                const uint64_t slot = (uint64_t)offsets[g] + k;
                if (slot >= r->capacity) break;
                for (int c = 0; c < 9; ++c) v[c] += slots[slot * SP_GRAD_STRIDE + c];
            }
        }
        std::memcpy(host + g * SP_GRAD_STRIDE, v, sizeof(v));
    }
    return SP_OK;
}

sp_status sp_count_blend_work(sp_rasterizer* r, uint64_t* forward_pairs, uint64_t* backward_pairs,
                              uint64_t* taken_pairs) {
    if (!r || !forward_pairs || !backward_pairs) return SP_ERR_INVALID;
    SP_REQUIRE(r->ctx, r->forward_done, SP_ERR_INVALID, "count before any forward pass");
    SP_CHECK(select_device(r->ctx));
    unsigned long long* counts = nullptr;
    SP_CUDA(r->ctx, cudaMallocAsync((void**)&counts, 3 * sizeof(unsigned long long), r->ctx->stream));
    cudaError_t err = cudaMemsetAsync(counts, 0, 3 * sizeof(unsigned long long), r->ctx->stream);
    if (err == cudaSuccess)
        err = launch_count_blend(r->records, r->values[r->sorted_buffer], r->ranges, r->camera, r->contributions,
                                 counts, r->ctx->stream);
    unsigned long long host[3] = {0, 0, 0};
    sp_status s = err == cudaSuccess ? read_device(r->ctx, host, counts, sizeof(host))
                                     : cuda_fail(r->ctx, err, "launch_count_blend");
    cudaFreeAsync(counts, r->ctx->stream);
    cudaStreamSynchronize(r->ctx->stream);
    *forward_pairs = host[0];
    *backward_pairs = host[1];
    if (taken_pairs) *taken_pairs = host[2];
    return s;
}

sp_status sp_debug_stall_sort_partition(sp_rasterizer* r, uint32_t partition) {
    if (!r) return SP_ERR_INVALID;
    SP_CHECK(select_device(r->ctx));
    const uint32_t value = partition == 0xffffffffu ? 0u : partition + 1u;
    SP_CUDA(r->ctx, cudaMemcpyAsync(&r->meta->stall_partition, &value, sizeof(value), cudaMemcpyHostToDevice,
                                    r->ctx->stream));
    return sync_stream(r->ctx);
}

sp_status sp_profile_enable(sp_context* ctx, int enable) {
    if (!ctx) return SP_ERR_INVALID;
    SP_CHECK(select_device(ctx));
    ctx->profiling = enable != 0;
    return SP_OK;
}

sp_status sp_profile_read(sp_context* ctx, double* ms, uint64_t* launches) {
    if (!ctx || !ms || !launches) return SP_ERR_INVALID;
    SP_CHECK(select_device(ctx));
    SP_CHECK(sync_stream(ctx));
    for (int k = 0; k < SP_K_COUNT; ++k) {
        for (auto& pair : ctx->recorded[k]) {
            float elapsed = 0.0f;
            SP_CUDA(ctx, cudaEventElapsedTime(&elapsed, pair.first, pair.second));
            ms[k] += elapsed;
            launches[k] += 1;
            ctx->event_pool.push_back(pair.first);
            ctx->event_pool.push_back(pair.second);
        }
        ctx->recorded[k].clear();
    }
    return SP_OK;
}

// ------------------------------------------------------------------------------- Adam

// Moments `m` and `v` (host or device memory by `kind`; null: zeroed) are copied on the
// context's stream, which then finishes them before the call returns.
static sp_status adam_make(sp_context* ctx, float* d_params, const float* d_gradients, uint64_t n, uint32_t sh_degree,
                           const sp_learning_rates& rates, float position_scale, uint32_t step,
                           const float* m, const float* v, cudaMemcpyKind kind, sp_adam** out) {
    // optimizer.rs:137-159, 200-243.
    SP_REQUIRE(ctx, n > 0, SP_ERR_INVALID, "no Gaussians");
    SP_REQUIRE(ctx, d_params && d_gradients, SP_ERR_INVALID, "null params or gradients buffer");
    SP_REQUIRE(ctx, sh_degree <= 3, SP_ERR_INVALID, "SH degree above 3");
    SP_REQUIRE(ctx, position_scale > 0.0f, SP_ERR_INVALID, "camera extent must be positive");  // prune.rs:34
    SP_CHECK(select_device(ctx));
    sp_adam* a = new sp_adam();
    a->ctx = ctx;
    a->params = d_params;
    a->gradients = d_gradients;
    a->n = n;
    a->sh_degree = sh_degree;
    a->stride = SP_PARAM_STRIDE(sh_degree);
    a->rates = rates;
    a->position_scale = position_scale;
    a->step = step;
    a->max_log_scale = std::log(SP_SCALE_MAX_EXTENT_FRACTION * position_scale);
    a->max_log_anisotropy = std::log(SP_SCALE_MAX_ANISOTROPY);
    const size_t bytes = n * a->stride * sizeof(float);
    cudaError_t err = cudaMalloc(&a->first_moment, bytes);
    if (err == cudaSuccess) err = cudaMalloc(&a->second_moment, bytes);
    if (err == cudaSuccess) {
        if (m) err = cudaMemcpyAsync(a->first_moment, m, bytes, kind, ctx->stream);
        else err = cudaMemsetAsync(a->first_moment, 0, bytes, ctx->stream);
    }
    if (err == cudaSuccess) {
        if (v) err = cudaMemcpyAsync(a->second_moment, v, bytes, kind, ctx->stream);
        else err = cudaMemsetAsync(a->second_moment, 0, bytes, ctx->stream);
    }
    if (err == cudaSuccess) err = cudaStreamSynchronize(ctx->stream);
    if (err != cudaSuccess) {
        cudaFree(a->first_moment);
        cudaFree(a->second_moment);
        delete a;
        return cuda_fail(ctx, err, "Adam moments");
    }
    *out = a;
    return SP_OK;
}

sp_status sp_adam_create(sp_context* ctx, float* d_params, const float* d_gradients, uint64_t gaussian_count,
                         uint32_t sh_degree, const sp_learning_rates* rates, float position_scale, sp_adam** out) {
    if (!ctx || !rates || !out) return SP_ERR_INVALID;
    *out = nullptr;
    return adam_make(ctx, d_params, d_gradients, gaussian_count, sh_degree, *rates, position_scale, 0, nullptr,
                     nullptr, cudaMemcpyHostToDevice, out);
}

sp_status sp_adam_resume(const sp_adam* from, float* d_params, const float* d_gradients, uint64_t gaussian_count,
                         const float* host_first_moment, const float* host_second_moment, sp_adam** out) {
    if (!from || !out) return SP_ERR_INVALID;
    *out = nullptr;
    SP_REQUIRE(from->ctx, host_first_moment && host_second_moment, SP_ERR_INVALID, "moments");
    return adam_make(from->ctx, d_params, d_gradients, gaussian_count, from->sh_degree, from->rates,
                     from->position_scale, from->step, host_first_moment, host_second_moment,
                     cudaMemcpyHostToDevice, out);
}

sp_status sp_adam_resume_device(const sp_adam* from, float* d_params, const float* d_gradients,
                                uint64_t gaussian_count, const float* d_first_moment, const float* d_second_moment,
                                sp_adam** out) {
    if (!from || !out) return SP_ERR_INVALID;
    *out = nullptr;
    SP_REQUIRE(from->ctx, d_first_moment && d_second_moment, SP_ERR_INVALID, "moments");
    return adam_make(from->ctx, d_params, d_gradients, gaussian_count, from->sh_degree, from->rates,
                     from->position_scale, from->step, d_first_moment, d_second_moment,
                     cudaMemcpyDeviceToDevice, out);
}

void sp_adam_destroy(sp_adam* a) {
    if (!a) return;
    cudaSetDevice(a->ctx->device);
    cudaStreamSynchronize(a->ctx->stream);
    cudaFree(a->first_moment);
    cudaFree(a->second_moment);
    delete a;
}

sp_status sp_adam_advance(sp_adam* a, float position_rate_factor) {
    if (!a) return SP_ERR_INVALID;
    // optimizer.rs:248-256.
    SP_REQUIRE(a->ctx, position_rate_factor > 0.0f && position_rate_factor <= 1.0f, SP_ERR_INVALID,
               "position rate factor must be in (0, 1]");
    a->step += 1;
    a->lr_by_slot.assign(a->stride, 0.0f);
    learning_rates_by_slot(a->rates, a->position_scale * position_rate_factor, a->stride, a->lr_by_slot.data());
    a->bias1 = 1.0f - std::pow(SP_ADAM_BETA1, (float)a->step);
    a->bias2 = 1.0f - std::pow(SP_ADAM_BETA2, (float)a->step);
    return SP_OK;
}

sp_status sp_adam_step_range(sp_adam* a, uint64_t first, uint64_t count) {
    if (!a) return SP_ERR_INVALID;
    SP_REQUIRE(a->ctx, a->step > 0 && !a->lr_by_slot.empty(), SP_ERR_INVALID, "sp_adam_advance first");
    SP_REQUIRE(a->ctx, first <= a->n && count <= a->n - first, SP_ERR_INVALID, "range outside the Gaussians");
    SP_CHECK(select_device(a->ctx));
    KernelSpan span(a->ctx, SP_K_ADAM);
    SP_CUDA(a->ctx, launch_adam(a->params, a->gradients, a->first_moment, a->second_moment, first, count, (int)a->stride,
                                a->lr_by_slot.data(), a->bias1, a->bias2, a->max_log_scale, a->max_log_anisotropy,
                                a->ctx->stream));
    return SP_OK;
}

sp_status sp_adam_step(sp_adam* a, float position_rate_factor) {
    NvtxRange range("sp_adam_step");
    SP_CHECK(sp_adam_advance(a, position_rate_factor));
    return sp_adam_step_range(a, 0, a->n);
}

uint32_t sp_adam_steps_taken(const sp_adam* a) { return a ? a->step : 0; }

sp_status sp_adam_read_moments(sp_adam* a, float* host_first, float* host_second) {
    if (!a) return SP_ERR_INVALID;
    SP_CHECK(select_device(a->ctx));
    const size_t bytes = a->n * a->stride * sizeof(float);
    SP_CHECK(read_device(a->ctx, host_first, a->first_moment, bytes));
    return read_device(a->ctx, host_second, a->second_moment, bytes);
}

// ------------------------------------------------- multi-GPU exchange over peer memory

}  // extern "C"

namespace {

// The allocation holding device pointer `p` (its base and p's offset in it): CUDA IPC shares
// whole allocations. cuMemGetAddressRange through the runtime's driver entry point, so the
// library needs no link to the driver library.
sp_status allocation_of(sp_context* ctx, const void* p, void** base, uint64_t* offset) {
    using AddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static AddressRange address_range = nullptr;
    if (!address_range) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult found;
        const cudaError_t err = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &found);
        if (err != cudaSuccess || found != cudaDriverEntryPointSuccess || !fn)
            return fail(ctx, SP_ERR_CUDA, "cuMemGetAddressRange is not available");
        address_range = reinterpret_cast<AddressRange>(fn);
    }
    CUdeviceptr b = 0;
    size_t size = 0;
    if (address_range(&b, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
        return fail(ctx, SP_ERR_CUDA, "the buffer is not a device allocation");
    *base = reinterpret_cast<void*>(b);
    *offset = (uint64_t)(reinterpret_cast<uintptr_t>(p) - (uintptr_t)b);
    return SP_OK;
}

}  // namespace

extern "C" {

sp_status sp_peer_export(const sp_adam* a, sp_peer_handle* out) {
    if (!a || !out) return SP_ERR_INVALID;
    std::memset(out, 0, sizeof(*out));
    SP_CHECK(select_device(a->ctx));
    void* base = nullptr;
    cudaIpcMemHandle_t h;
    SP_CHECK(allocation_of(a->ctx, a->params, &base, &out->params_offset));
    SP_CUDA(a->ctx, cudaIpcGetMemHandle(&h, base));
    std::memcpy(out->params, &h, sizeof(h));
    SP_CHECK(allocation_of(a->ctx, a->gradients, &base, &out->gradients_offset));
    SP_CUDA(a->ctx, cudaIpcGetMemHandle(&h, base));
    std::memcpy(out->gradients, &h, sizeof(h));
    out->gaussian_count = a->n;
    out->stride = a->stride;
    out->device = a->ctx->device;
    return SP_OK;
}

void sp_peer_exchange_destroy(sp_peer_exchange* ex) {
    if (!ex) return;
    cudaSetDevice(ex->adam->ctx->device);
    cudaStreamSynchronize(ex->adam->ctx->stream);
    for (void* p : ex->opened) cudaIpcCloseMemHandle(p);
    delete ex;
}

sp_status sp_peer_exchange_create(sp_adam* a, uint32_t rank, uint32_t world, const sp_peer_handle* handles,
                                  sp_peer_exchange** out) {
    if (!a || !handles || !out) return SP_ERR_INVALID;
    *out = nullptr;
    sp_context* ctx = a->ctx;
    SP_REQUIRE(ctx, world >= 1 && world <= (uint32_t)kMaxPeers && rank < world, SP_ERR_INVALID,
               "rank and world (at most 8 ranks)");
    SP_REQUIRE(ctx, a->n % world == 0, SP_ERR_INVALID, "the Gaussians do not split evenly over the ranks");
    for (uint32_t r = 0; r < world; ++r)
        SP_REQUIRE(ctx, handles[r].gaussian_count == a->n && handles[r].stride == a->stride, SP_ERR_INVALID,
                   "every rank's optimiser must hold the same Gaussians");
    SP_CHECK(select_device(ctx));
    sp_peer_exchange* ex = new sp_peer_exchange();
    ex->adam = a;
    ex->peers.world = world;
    ex->peers.rank = rank;
    ex->count = a->n / world;
    ex->first = (uint64_t)rank * ex->count;
    for (uint32_t r = 0; r < world; ++r) {
        if (r == rank) {
            ex->peers.params[r] = a->params;
            ex->peers.gradients[r] = a->gradients;
            continue;
        }
        for (int which = 0; which < 2; ++which) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, which == 0 ? handles[r].params : handles[r].gradients, sizeof(h));
            void* base = nullptr;
            const cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
            if (err != cudaSuccess) {
                sp_peer_exchange_destroy(ex);
                return cuda_fail(ctx, err, "cudaIpcOpenMemHandle (a peer's buffer)");
            }
            ex->opened.push_back(base);
            char* p = static_cast<char*>(base) + (which == 0 ? handles[r].params_offset : handles[r].gradients_offset);
            if (which == 0) ex->peers.params[r] = reinterpret_cast<float*>(p);
            else ex->peers.gradients[r] = reinterpret_cast<const float*>(p);
        }
    }
    *out = ex;
    return SP_OK;
}

sp_status sp_peer_exchange_step(sp_peer_exchange* ex, float position_rate_factor) {
    NvtxRange range("sp_peer_exchange_step");
    if (!ex) return SP_ERR_INVALID;
    sp_adam* a = ex->adam;
    SP_CHECK(sp_adam_advance(a, position_rate_factor));
    SP_CHECK(select_device(a->ctx));
    KernelSpan span(a->ctx, SP_K_PEER_ADAM);
    SP_CUDA(a->ctx, launch_adam_peer(ex->peers, a->first_moment, a->second_moment, ex->first, ex->count,
                                     (int)a->stride, a->lr_by_slot.data(), a->bias1, a->bias2, a->max_log_scale,
                                     a->max_log_anisotropy, a->ctx->stream));
    return SP_OK;
}

float* sp_adam_first_moment_device(sp_adam* a) { return a ? a->first_moment : nullptr; }

float* sp_adam_second_moment_device(sp_adam* a) { return a ? a->second_moment : nullptr; }

float sp_position_rate_factor(uint64_t step, uint64_t steps) {
    // optimizer.rs:59-62 asserts steps > 0 && step < steps.
    if (steps == 0 || step >= steps) return -1.0f;
    return position_rate_factor(step, steps);
}

// ----------------------------------------------------------------------- densification

int sp_densify_after(const sp_densify_settings* s, uint64_t done, uint64_t steps) {
    // densify.rs:77-83.
    if (!s || s->interval == 0 || done < 1 || done > steps) return -1;
    return done >= s->start && done % s->interval == 0 && (float)done <= s->stop_fraction * (float)steps;
}

int sp_resets_opacity_after(const sp_densify_settings* s, uint64_t done) {
    // densify.rs:84-94; interval 0 is None.
    if (!s) return -1;
    if (s->opacity_reset_interval == 0) return 0;
    if (s->interval == 0 || s->opacity_reset_interval % s->interval != 0) return -1;
    return done % s->opacity_reset_interval == 0;
}

}  // extern "C"

struct sp_densify {
    sp_rasterizer* r = nullptr;
    const sp_adam* adam = nullptr;
    DensifyConstants constants{};
    uint64_t seed = 0;
    uint32_t reset_opacity = 0;
    void* block = nullptr;  // fate, keys, tallies and state in one allocation
    uint8_t* fate = nullptr;
    uint32_t* keys = nullptr;
    DensifyTally* tallies = nullptr;
    DensifyState* state = nullptr;
    sp_densify_report report{};
};

extern "C" {

void sp_densify_destroy(sp_densify* plan) {
    if (!plan) return;
    cudaSetDevice(plan->r->ctx->device);
    cudaStreamSynchronize(plan->r->ctx->stream);
    cudaFree(plan->block);
    delete plan;
}

sp_status sp_densify_plan(sp_rasterizer* r, const sp_adam* adam, float extent, uint64_t max_count,
                          const sp_densify_settings* settings, int reset_opacity, uint64_t seed, sp_densify** out,
                          sp_densify_report* report) {
    if (!r || !adam || !settings || !out || !report) return SP_ERR_INVALID;
    *out = nullptr;
    sp_context* ctx = r->ctx;
    // densify.rs:163-166.
    SP_REQUIRE(ctx, extent > 0.0f, SP_ERR_INVALID, "camera extent must be positive");
    SP_REQUIRE(ctx, adam->ctx == ctx && adam->params == r->params && adam->n == r->n && adam->stride == r->stride,
               SP_ERR_INVALID, "the optimiser is not the one of the rasterizer's parameters");
    SP_CHECK(select_device(ctx));
    sp_densify* plan = new sp_densify();
    plan->r = r;
    plan->adam = adam;
    plan->seed = seed;
    plan->reset_opacity = reset_opacity ? 1u : 0u;
    DensifyConstants& c = plan->constants;
    c.prune_opacity = settings->prune_opacity;
    c.max_screen_radius = settings->max_screen_radius;
    c.gradient_threshold = settings->gradient_threshold;
    c.split_log_scale = std::log(settings->split_scale_fraction * extent);
    c.log_split_divisor = std::log(1.6f);                  // SPLIT_SCALE_DIVISOR
    c.reset_logit = std::log(0.01f / (1.0f - 0.01f));     // logit(RESET_OPACITY)
    const uint64_t n = r->n;
    const uint32_t tiles = densify_tiles(n);
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t fate_bytes = align(n), keys_bytes = align(n * 4), tally_bytes = align(tiles * sizeof(DensifyTally));
    cudaError_t err = cudaMalloc(&plan->block, fate_bytes + keys_bytes + tally_bytes + sizeof(DensifyState));
    if (err != cudaSuccess) {
        delete plan;
        return cuda_fail(ctx, err, "densify scratch");
    }
    char* base = static_cast<char*>(plan->block);
    plan->fate = reinterpret_cast<uint8_t*>(base);
    plan->keys = reinterpret_cast<uint32_t*>(base + fate_bytes);
    plan->tallies = reinterpret_cast<DensifyTally*>(base + fate_bytes + keys_bytes);
    plan->state = reinterpret_cast<DensifyState*>(base + fate_bytes + keys_bytes + tally_bytes);
    sp_status status = SP_OK;
    {
        KernelSpan span(ctx, SP_K_DENSIFY);
        err = launch_densify_plan(r->params, r->densify_stats, n, r->stride, c, max_count, plan->fate, plan->keys,
                                  plan->tallies, plan->state, plan->reset_opacity, ctx->stream);
    }
    if (err != cudaSuccess) status = cuda_fail(ctx, err, "densify plan");
    if (status == SP_OK)
        status = read_device(ctx, &plan->report, &plan->state->report, sizeof(sp_densify_report));
    if (status != SP_OK) {
        sp_densify_destroy(plan);
        return status;
    }
    *report = plan->report;
    if (plan->report.after == 0) {
        sp_densify_destroy(plan);
        return fail(ctx, SP_ERR_INVALID, "densification pruned every Gaussian");  // densify.rs:255
    }
    *out = plan;
    return SP_OK;
}

sp_status sp_densify_apply(sp_densify* plan, float* d_params, float* d_first_moment, float* d_second_moment,
                           uint64_t capacity) {
    if (!plan) return SP_ERR_INVALID;
    sp_context* ctx = plan->r->ctx;
    SP_REQUIRE(ctx, d_params && d_first_moment && d_second_moment, SP_ERR_INVALID, "null output buffer");
    SP_REQUIRE(ctx, capacity >= plan->report.after, SP_ERR_INVALID, "the outputs hold fewer Gaussians than report.after");
    SP_CHECK(select_device(ctx));
    KernelSpan span(ctx, SP_K_DENSIFY);
    const sp_adam* a = plan->adam;
    SP_CUDA(ctx, launch_densify_write(plan->r->params, a->first_moment, a->second_moment, plan->r->n, a->sh_degree,
                                      plan->constants, plan->fate, plan->tallies, plan->state, plan->seed,
                                      plan->reset_opacity, d_params, d_first_moment, d_second_moment, ctx->stream));
    return SP_OK;
}

}  // extern "C"
