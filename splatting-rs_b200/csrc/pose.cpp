// Host-side camera pose refinement in f64 (pose_refinement.rs:30-163: per-view Adam over 6
// pose parameters plus a shared log focal scale, view 0 fixed) over the pose chain of
// pose_math.h (camera_pose.rs:39-99). As in the reference the pose parameters live on the CPU
// and the GPU supplies the 56-byte camera gradient; sp_device_poses (pose_device.cu) runs the
// same arithmetic on the GPU instead.
#include <cmath>
#include <cstring>
#include <vector>

#include "pose_state.h"

using namespace splat::pose;

extern "C" {

sp_status sp_corrected_camera(const sp_pinhole_camera* initial, const sp_pose_correction* correction,
                              double focal_log_scale, sp_pinhole_camera* out) {
    if (!initial || !correction || !out) return SP_ERR_INVALID;
    *out = corrected(*initial, *correction, focal_log_scale);
    return SP_OK;
}

sp_status sp_pose_gradient_of(const sp_pinhole_camera* initial, const sp_pose_correction* correction,
                              double focal_log_scale, const sp_camera_gradient* gradient, sp_pose_gradient* out) {
    if (!initial || !correction || !gradient || !out) return SP_ERR_INVALID;
    *out = pose_gradient(*initial, *correction, focal_log_scale, *gradient);
    return SP_OK;
}

sp_status sp_pose_refinement_create(const sp_pinhole_camera* initial, uint32_t view_count,
                                    const sp_learning_rates* rates, float extent, sp_pose_refinement** out) {
    if (!initial || !rates || !out) return SP_ERR_INVALID;
    *out = nullptr;
    // pose_refinement.rs:67-81.
    if (view_count <= kFixedView) return SP_ERR_INVALID;
    if (!(extent > 0.0f)) return SP_ERR_INVALID;
    sp_pose_refinement* p = new sp_pose_refinement();
    p->initial.assign(initial, initial + view_count);
    p->views.assign(view_count, ViewState{});
    p->shared.rotation_rate = (double)rates->camera_rotation;
    p->shared.translation_rate = (double)rates->camera_translation * (double)extent;
    p->shared.focal_rate = (double)rates->camera_focal;
    *out = p;
    return SP_OK;
}

void sp_pose_refinement_destroy(sp_pose_refinement* p) { delete p; }

sp_status sp_pose_refinement_camera(const sp_pose_refinement* p, uint32_t view, sp_pinhole_camera* out) {
    if (!p || !out || view >= p->initial.size()) return SP_ERR_INVALID;
    *out = corrected(p->initial[view], p->views[view].correction, p->shared.focal_log_scale);
    return SP_OK;
}

sp_status sp_pose_refinement_step(sp_pose_refinement* p, uint32_t view, const sp_camera_gradient* gradient,
                                  float rate_factor) {
    if (!p || !gradient || view >= p->initial.size()) return SP_ERR_INVALID;
    // pose_refinement.rs:113-163.
    if (!(rate_factor > 0.0f && rate_factor <= 1.0f)) return SP_ERR_INVALID;
    return refine(p->initial[view], p->views[view], p->shared, view, *gradient, (double)rate_factor);
}

sp_status sp_pose_refinement_correction(const sp_pose_refinement* p, uint32_t view, sp_pose_correction* out) {
    if (!p || !out || view >= p->views.size()) return SP_ERR_INVALID;
    *out = p->views[view].correction;
    return SP_OK;
}

double sp_pose_refinement_focal_scale(const sp_pose_refinement* p) {
    return p ? std::exp(p->shared.focal_log_scale) : 0.0;
}

sp_status sp_pose_refinement_last_gradient(const sp_pose_refinement* p, sp_pose_gradient* out) {
    if (!p || !out) return SP_ERR_INVALID;
    *out = p->shared.last_gradient;
    return SP_OK;
}

}  // extern "C"
