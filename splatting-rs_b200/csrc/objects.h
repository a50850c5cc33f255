// The objects behind the C ABI's opaque handles (sp_context, sp_rasterizer, sp_adam,
// sp_peer_exchange) and the error helpers the translation units of the ABI share (api.cu,
// comm.cu). Private to the library: callers see only include/splat.h.
#pragma once

#include <string>
#include <utility>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "kernels.h"

// A named range around an ABI call, for profilers on the host timeline (NVTX v3, header only:
// without a profiler attached a push and a pop cost a few nanoseconds).
class NvtxRange {
   public:
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

using splat::DeviceMeta;
using splat::PeerBuffers;
using splat::SortPlan;

struct sp_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::string error;
    // Per-kernel device timing (sp_profile_enable / sp_profile_read).
    bool profiling = false;
    std::vector<cudaEvent_t> event_pool;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> recorded[SP_K_COUNT];

    cudaEvent_t take_event() {
        if (!event_pool.empty()) {
            cudaEvent_t e = event_pool.back();
            event_pool.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }
};

// Records a pair of events around the launches in its scope when profiling is on.
class KernelSpan {
   public:
    KernelSpan(sp_context* ctx, int kernel) : ctx_(ctx), kernel_(kernel) {
        if (ctx_->profiling) {
            start_ = ctx_->take_event();
            cudaEventRecord(start_, ctx_->stream);
        }
    }
    ~KernelSpan() {
        if (start_) {
            cudaEvent_t stop = ctx_->take_event();
            cudaEventRecord(stop, ctx_->stream);
            ctx_->recorded[kernel_].emplace_back(start_, stop);
        }
    }

   private:
    sp_context* ctx_;
    int kernel_;
    cudaEvent_t start_ = nullptr;
};

struct sp_rasterizer {
    sp_context* ctx = nullptr;
    const float* params = nullptr;
    uint64_t n = 0;
    uint32_t width = 0, height = 0, tiles_x = 0, tiles_y = 0, tiles = 0;
    const float* ground_truth = nullptr;
    uint32_t views = 0;
    sp_options options{};
    uint32_t stride = 0;
    uint64_t capacity = 0;
    uint32_t blocks = 0;          // projection blocks of 256 Gaussians
    uint32_t max_partitions = 0;  // sort partitions at full capacity
    SortPlan plan{};
    sp_camera_uniform camera{};
    bool has_camera = false;
    bool forward_done = false;
    // The atomic backward's blend sums were zeroed by the last sp_loss (k_loss) and no backward
    // has added to them since: blend_backward can skip its memset.
    bool blend_sums_zero = false;
    uint32_t sequence = 0;
    int sorted_buffer = 0;
    std::vector<void*> allocations;

    float4* records = nullptr;
    float4* reach = nullptr;  // the blend kernels' culling constants per Gaussian
    uint32_t* radii = nullptr;
    uint32_t* offsets = nullptr;
    uint32_t* block_totals = nullptr;
    unsigned long long* block_offsets = nullptr;
    DeviceMeta* meta = nullptr;
    void* keys[2] = {nullptr, nullptr};
    uint32_t* values[2] = {nullptr, nullptr};
    uint32_t* sort_histograms = nullptr;
    uint32_t* sort_tickets = nullptr;
    unsigned long long* lookback = nullptr;
    uint2* ranges = nullptr;
    uint32_t* tile_order = nullptr;
    // The camera the projection kernels read: written by sp_set_camera (an asynchronous copy)
    // or by the device pose step (sp_device_poses_step).
    sp_camera_uniform* camera_dev = nullptr;
    bool camera_on_device = false;  // the last camera came from the device pose step
    float4* image = nullptr;
    uint32_t* contributions = nullptr;
    float4* ssim_partials = nullptr;
    float4* loss_gradient = nullptr;
    float4* pixel_loss = nullptr;
    double* loss_sums = nullptr;    // the loss-sum kernel's workspace
    double* loss_result = nullptr;  // its 4 sums (inside readback_dev)
    float* slot_gradients = nullptr;
    float4* gaussian_gradients = nullptr;
    float* param_gradients = nullptr;
    float* camera_partials = nullptr;
    uint32_t* camera_done = nullptr;
    float* camera_gradient = nullptr;
    float4* densify_stats = nullptr;
    // Pinned host staging of the per-step read-back (sp_train_step).
    struct StepReadback {
        float camera[SP_CAMERA_GRAD_STRIDE];
        uint32_t status;    // DeviceMeta::status of the step
        uint32_t overflow;  // DeviceMeta::overflow of the step's forward pass
        double loss[4];
    };
    StepReadback* readback = nullptr;
    void* readback_mapped = nullptr;  // `readback` as the device addresses it
    // Its device side: the camera gradient and the loss sums live here (camera_gradient and
    // loss_result point into it), so that a step's read-back is one copy.
    StepReadback* readback_dev = nullptr;

    uint64_t pixels() const { return (uint64_t)width * height; }
};

struct sp_adam {
    sp_context* ctx = nullptr;
    float* params = nullptr;
    const float* gradients = nullptr;
    uint64_t n = 0;
    uint32_t sh_degree = 0, stride = 0;
    sp_learning_rates rates{};
    float position_scale = 1.0f;
    uint32_t step = 0;
    float* first_moment = nullptr;
    float* second_moment = nullptr;
    float max_log_scale = 0.0f, max_log_anisotropy = 0.0f;
    // The rates of the step in progress (sp_adam_advance).
    std::vector<float> lr_by_slot;
    float bias1 = 0.0f, bias2 = 0.0f;
};

struct sp_peer_exchange {
    sp_adam* adam = nullptr;
    PeerBuffers peers{};
    std::vector<void*> opened;  // mapped peer allocations, closed on destroy
    uint64_t first = 0, count = 0;
};

inline sp_status fail(sp_context* ctx, sp_status status, const std::string& message) {
    if (ctx) ctx->error = message;
    return status;
}

inline sp_status cuda_fail(sp_context* ctx, cudaError_t err, const char* what) {
    return fail(ctx, err == cudaErrorMemoryAllocation ? SP_ERR_OUT_OF_MEMORY : SP_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorString(err));
}

#define SP_CUDA(ctx, expr)                                      \
    do {                                                        \
        cudaError_t err_ = (expr);                              \
        if (err_ != cudaSuccess) return cuda_fail(ctx, err_, #expr); \
    } while (0)

inline sp_status select_device(sp_context* ctx) {
    SP_CUDA(ctx, cudaSetDevice(ctx->device));
    return SP_OK;
}

inline sp_status sync_stream(sp_context* ctx) {
    SP_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return SP_OK;
}

#define SP_CHECK(expr)                   \
    do {                                 \
        const sp_status s_ = (expr);     \
        if (s_ != SP_OK) return s_;      \
    } while (0)

#define SP_REQUIRE(ctx, cond, status, message) \
    do {                                       \
        if (!(cond)) return fail(ctx, status, message); \
    } while (0)
