// The camera pose chain in f64 as host + device inline functions, shared by the host pose
// refinement (pose.cpp) and its device kernel (pose_device.cu): camera_pose.rs:34-99 (so(3)
// exponential and left Jacobian, the corrected camera, the chain rule from a CameraGradient
// to the 7 pose parameters), camera.rs:46-70 (the camera uniform) and the f64 Adam of
// pose_refinement.rs:30-62. The same source runs on both sides; sin, cos, exp, sqrt and pow
// are the host C library's on the CPU and CUDA's on the GPU, so the two agree to rounding.
#pragma once

#include <stdint.h>

#include <cmath>

#include "../../include/splat.h"
#include "../../include/splat_constants.h"
#include "../../include/splat_math.h"

namespace splat {
namespace pose {

struct Mat3 {
    double m[3][3];
};
struct Vec3 {
    double v[3];
};

SP_HD Mat3 identity() {
    Mat3 r{};
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = i == j ? 1.0 : 0.0;
    return r;
}

SP_HD Mat3 mul(const Mat3& a, const Mat3& b) {
    Mat3 r{};
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) {
            double s = 0.0;
            for (int k = 0; k < 3; ++k) s += a.m[i][k] * b.m[k][j];
            r.m[i][j] = s;
        }
    return r;
}

SP_HD Mat3 add(const Mat3& a, const Mat3& b) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[i][j] + b.m[i][j];
    return r;
}

SP_HD Mat3 scale(const Mat3& a, double s) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[i][j] * s;
    return r;
}

SP_HD Mat3 transpose(const Mat3& a) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[j][i];
    return r;
}

SP_HD Vec3 mul(const Mat3& a, const Vec3& x) {
    Vec3 r{};
    for (int i = 0; i < 3; ++i) {
        double s = 0.0;
        for (int k = 0; k < 3; ++k) s += a.m[i][k] * x.v[k];
        r.v[i] = s;
    }
    return r;
}

SP_HD double norm(const Vec3& x) { return std::sqrt(x.v[0] * x.v[0] + x.v[1] * x.v[1] + x.v[2] * x.v[2]); }

SP_HD Vec3 cross(const Vec3& a, const Vec3& b) {
    return {{a.v[1] * b.v[2] - a.v[2] * b.v[1], a.v[2] * b.v[0] - a.v[0] * b.v[2], a.v[0] * b.v[1] - a.v[1] * b.v[0]}};
}

// camera_pose.rs:34-36.
SP_HD Mat3 skew(const Vec3& v) {
    Mat3 r{};
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = 0.0;
    r.m[0][1] = -v.v[2];
    r.m[0][2] = v.v[1];
    r.m[1][0] = v.v[2];
    r.m[1][2] = -v.v[0];
    r.m[2][0] = -v.v[1];
    r.m[2][1] = v.v[0];
    return r;
}

constexpr double kSmallAngle = 1e-6;  // camera_pose.rs:31-32
constexpr uint32_t kFixedView = 0;    // pose_refinement.rs:14

// so3_exp (camera_pose.rs:38-46), Rodrigues.
SP_HD Mat3 so3_exp(const Vec3& omega) {
    const double angle = norm(omega);
    const Mat3 k = skew(omega);
    const Mat3 kk = mul(k, k);
    if (angle < kSmallAngle) return add(add(identity(), k), scale(kk, 0.5));
    return add(add(identity(), scale(k, std::sin(angle) / angle)), scale(kk, (1.0 - std::cos(angle)) / (angle * angle)));
}

// so3_left_jacobian (camera_pose.rs:48-57).
SP_HD Mat3 so3_left_jacobian(const Vec3& omega) {
    const double angle = norm(omega);
    const Mat3 k = skew(omega);
    const Mat3 kk = mul(k, k);
    if (angle < kSmallAngle) return add(add(identity(), scale(k, 0.5)), scale(kk, 1.0 / 6.0));
    const double angle2 = angle * angle;
    return add(add(identity(), scale(k, (1.0 - std::cos(angle)) / angle2)),
               scale(kk, (angle - std::sin(angle)) / (angle2 * angle)));
}

SP_HD Vec3 vee(const Mat3& s) { return {{s.m[2][1], s.m[0][2], s.m[1][0]}}; }

SP_HD Mat3 rotation_of(const sp_pinhole_camera& c) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = c.rotation[i * 3 + j];
    return r;
}

// camera_pose.rs:59-68: the rotation correction applied on the left, the translation
// added, both focal lengths scaled by exp(focal_log_scale).
SP_HD sp_pinhole_camera corrected(const sp_pinhole_camera& initial, const sp_pose_correction& correction,
                                  double focal_log_scale) {
    const double focal_scale = std::exp(focal_log_scale);
    sp_pinhole_camera out = initial;
    const Mat3 r = mul(so3_exp({{correction.rotation[0], correction.rotation[1], correction.rotation[2]}}),
                       rotation_of(initial));
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) out.rotation[i * 3 + j] = r.m[i][j];
    for (int i = 0; i < 3; ++i) out.translation[i] = initial.translation[i] + correction.translation[i];
    out.focal[0] = initial.focal[0] * focal_scale;
    out.focal[1] = initial.focal[1] * focal_scale;
    return out;
}

// camera_pose.rs:81-99.
SP_HD sp_pose_gradient pose_gradient(const sp_pinhole_camera& initial, const sp_pose_correction& correction,
                                     double focal_log_scale, const sp_camera_gradient& gradient) {
    const sp_pinhole_camera camera = corrected(initial, correction, focal_log_scale);
    const Mat3 w = transpose(rotation_of(camera));
    Mat3 d_w;
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) d_w.m[r][c] = (double)gradient.world_to_camera_rotation_rows[r][c];
    const Vec3 d_t_wc = {{gradient.world_to_camera_translation[0], gradient.world_to_camera_translation[1],
                          gradient.world_to_camera_translation[2]}};
    const Mat3 a = mul(transpose(w), d_w);
    const Vec3 wt_dt = mul(transpose(w), d_t_wc);
    const Vec3 d_center = {{-wt_dt.v[0], -wt_dt.v[1], -wt_dt.v[2]}};
    const Mat3 at = transpose(a);
    Mat3 diff;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) diff.m[i][j] = at.m[i][j] - a.m[i][j];
    const Vec3 v = vee(diff);
    const Vec3 c = cross({{camera.translation[0], camera.translation[1], camera.translation[2]}}, d_center);
    const Vec3 d_phi = {{v.v[0] - c.v[0], v.v[1] - c.v[1], v.v[2] - c.v[2]}};
    const Vec3 d_rot =
        mul(transpose(so3_left_jacobian({{correction.rotation[0], correction.rotation[1], correction.rotation[2]}})),
            d_phi);
    sp_pose_gradient out;
    for (int i = 0; i < 3; ++i) {
        out.rotation[i] = d_rot.v[i];
        out.translation[i] = d_center.v[i];
    }
    out.focal_log_scale = camera.focal[0] * (double)gradient.focal[0] + camera.focal[1] * (double)gradient.focal[1];
    return out;
}

// pose_refinement.rs:30-62: one Adam step over n f64 parameters; `steps` counts the steps
// taken before this one and is advanced.
SP_HD void adam_update(double* params, const double* gradient, const double* rates, double* first, double* second,
                       uint32_t& steps, int n) {
    steps += 1;
    const double beta1 = (double)SP_ADAM_BETA1, beta2 = (double)SP_ADAM_BETA2;
    const double bias1 = 1.0 - std::pow(beta1, (double)steps);
    const double bias2 = 1.0 - std::pow(beta2, (double)steps);
    for (int i = 0; i < n; ++i) {
        first[i] = beta1 * first[i] + (1.0 - beta1) * gradient[i];
        second[i] = beta2 * second[i] + (1.0 - beta2) * gradient[i] * gradient[i];
        const double first_hat = first[i] / bias1;
        const double second_hat = second[i] / bias2;
        params[i] -= rates[i] * first_hat / (std::sqrt(second_hat) + (double)SP_ADAM_EPSILON);
    }
}

// camera.rs:46-70: W = R^T, t = -W C, the rows (W | t) and the intrinsics to f32.
SP_HD sp_camera_uniform uniform_of(const double rotation_c2w[9], const double translation[3], const double focal[2],
                                   const double principal_point[2], uint32_t width, uint32_t height) {
    sp_camera_uniform out;
    double w[3][3], t[3];
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) w[r][c] = rotation_c2w[c * 3 + r];
    for (int r = 0; r < 3; ++r) t[r] = -(w[r][0] * translation[0] + w[r][1] * translation[1] + w[r][2] * translation[2]);
    for (int r = 0; r < 3; ++r) {
        for (int c = 0; c < 3; ++c) out.world_to_camera_rows[r][c] = (float)w[r][c];
        out.world_to_camera_rows[r][3] = (float)t[r];
    }
    out.focal[0] = (float)focal[0];
    out.focal[1] = (float)focal[1];
    out.principal_point[0] = (float)principal_point[0];
    out.principal_point[1] = (float)principal_point[1];
    out.width = width;
    out.height = height;
    out.tiles_x = (width + SP_TILE - 1) / SP_TILE;
    out.tiles_y = (height + SP_TILE - 1) / SP_TILE;
    return out;
}

SP_HD sp_camera_uniform uniform_of(const sp_pinhole_camera& c) {
    return uniform_of(c.rotation, c.translation, c.focal, c.principal_point, c.width, c.height);
}

// The per-view state of the refinement: the correction and its moments.
struct ViewState {
    sp_pose_correction correction;
    double first[6], second[6];
    uint32_t steps;
    uint32_t pad;
};

// The shared state: the log focal scale and its moments, the base rates, the last pose
// gradient and a status word (SP_ERR_NONFINITE when a step met a non-finite gradient).
struct SharedState {
    double focal_log_scale, focal_first, focal_second;
    double rotation_rate, translation_rate, focal_rate;
    sp_pose_gradient last_gradient;
    uint32_t focal_steps;
    uint32_t status;
};

SP_HD bool finite(double x) { return x - x == 0.0; }

// pose_refinement.rs:113-163: the step of view `view` from its camera gradient. Returns
// SP_ERR_NONFINITE (and changes nothing) when the pose gradient is not finite.
SP_HD sp_status refine(const sp_pinhole_camera& initial, ViewState& vs, SharedState& sh, uint32_t view,
                       const sp_camera_gradient& gradient, double factor) {
    const sp_pose_gradient g = pose_gradient(initial, vs.correction, sh.focal_log_scale, gradient);
    bool ok = finite(g.focal_log_scale);
    for (int i = 0; i < 3; ++i) ok = ok && finite(g.rotation[i]) && finite(g.translation[i]);
    if (!ok) return SP_ERR_NONFINITE;
    sh.last_gradient = g;
    if (view != kFixedView) {
        double params[6] = {vs.correction.rotation[0],    vs.correction.rotation[1],    vs.correction.rotation[2],
                            vs.correction.translation[0], vs.correction.translation[1], vs.correction.translation[2]};
        const double grads[6] = {g.rotation[0], g.rotation[1], g.rotation[2],
                                 g.translation[0], g.translation[1], g.translation[2]};
        const double rr = sh.rotation_rate * factor, tr = sh.translation_rate * factor;
        const double rates[6] = {rr, rr, rr, tr, tr, tr};
        adam_update(params, grads, rates, vs.first, vs.second, vs.steps, 6);
        for (int i = 0; i < 3; ++i) {
            vs.correction.rotation[i] = params[i];
            vs.correction.translation[i] = params[3 + i];
        }
    }
    double focal = sh.focal_log_scale;
    const double fg = g.focal_log_scale, fr = sh.focal_rate * factor;
    adam_update(&focal, &fg, &fr, &sh.focal_first, &sh.focal_second, sh.focal_steps, 1);
    sh.focal_log_scale = focal;
    return SP_OK;
}

}  // namespace pose
}  // namespace splat
