// The pose refinement on the GPU (the reference's pose_refinement.rs:113-163 runs on the
// host after a 56-byte read-back per step): one thread applies the refinement step of the
// view just trained from the camera gradient the projection backward left in device memory,
// then writes the camera uniform of the next view for the next projection. The arithmetic is
// pose_math.h, the same source as the host refinement; compiled with -fmad=false so that it
// differs from the host's only through the math library (sin, cos, exp, pow).
#include "kernels.h"
#include "pose_math.h"

namespace splat {
namespace {

__global__ void k_pose_step(const sp_pinhole_camera* __restrict__ initial, pose::ViewState* states,
                            pose::SharedState* shared, const float* __restrict__ camera_gradient, uint32_t views,
                            uint32_t view, uint32_t next_view, double factor, sp_camera_uniform* camera_out) {
    chain_enter();  // the camera gradient is the previous grid's (the projection backward's)
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    if (view < views) {
        sp_camera_gradient g;
        const float* src = camera_gradient;
        for (int r = 0; r < 3; ++r)
            for (int c = 0; c < 3; ++c) g.world_to_camera_rotation_rows[r][c] = src[r * 3 + c];
        for (int i = 0; i < 3; ++i) g.world_to_camera_translation[i] = src[9 + i];
        g.focal[0] = src[12];
        g.focal[1] = src[13];
        const sp_status status = pose::refine(initial[view], states[view], *shared, view, g, factor);
        if (status != SP_OK && shared->status == 0) shared->status = (uint32_t)status;
    }
    if (next_view < views)
        *camera_out =
            pose::uniform_of(pose::corrected(initial[next_view], states[next_view].correction, shared->focal_log_scale));
}

}  // namespace

cudaError_t launch_pose_step(const sp_pinhole_camera* initial, pose::ViewState* states, pose::SharedState* shared,
                             const float* camera_gradient, uint32_t views, uint32_t view, uint32_t next_view,
                             double factor, sp_camera_uniform* camera_out, cudaStream_t stream) {
    launch_chained(k_pose_step, 1, 32, 0, stream, initial, states, shared, camera_gradient, views, view, next_view,
                   factor, camera_out);
    return cudaGetLastError();
}

}  // namespace splat
