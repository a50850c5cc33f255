// Host-side camera pose chain in f64: camera_pose.rs:39-99 (so(3) exponential, its left
// Jacobian, the corrected camera and the chain rule from a CameraGradient to the pose
// parameters) and pose_refinement.rs:30-163 (per-view Adam over 6 pose parameters plus a
// shared log focal scale, view 0 fixed). The pose parameters are 7 per view, so they stay
// on the CPU as in the reference; the GPU only supplies the 56-byte camera gradient.
#include <cmath>
#include <cstring>
#include <vector>

#include "../../include/splat.h"
#include "../../include/splat_constants.h"

namespace {

struct Mat3 {
    double m[3][3];
};
struct Vec3 {
    double v[3];
};

Mat3 identity() {
    Mat3 r{};
    for (int i = 0; i < 3; ++i) r.m[i][i] = 1.0;
    return r;
}

Mat3 mul(const Mat3& a, const Mat3& b) {
    Mat3 r{};
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            for (int k = 0; k < 3; ++k) r.m[i][j] += a.m[i][k] * b.m[k][j];
    return r;
}

Mat3 add(const Mat3& a, const Mat3& b) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[i][j] + b.m[i][j];
    return r;
}

Mat3 scale(const Mat3& a, double s) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[i][j] * s;
    return r;
}

Mat3 transpose(const Mat3& a) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[j][i];
    return r;
}

Vec3 mul(const Mat3& a, const Vec3& x) {
    Vec3 r{};
    for (int i = 0; i < 3; ++i)
        for (int k = 0; k < 3; ++k) r.v[i] += a.m[i][k] * x.v[k];
    return r;
}

double norm(const Vec3& x) { return std::sqrt(x.v[0] * x.v[0] + x.v[1] * x.v[1] + x.v[2] * x.v[2]); }

Vec3 cross(const Vec3& a, const Vec3& b) {
    return {{a.v[1] * b.v[2] - a.v[2] * b.v[1], a.v[2] * b.v[0] - a.v[0] * b.v[2], a.v[0] * b.v[1] - a.v[1] * b.v[0]}};
}

// camera_pose.rs:34-36.
Mat3 skew(const Vec3& v) {
    Mat3 r{};
    r.m[0][1] = -v.v[2];
    r.m[0][2] = v.v[1];
    r.m[1][0] = v.v[2];
    r.m[1][2] = -v.v[0];
    r.m[2][0] = -v.v[1];
    r.m[2][1] = v.v[0];
    return r;
}

constexpr double kSmallAngle = 1e-6;  // camera_pose.rs:31-32

// so3_exp (camera_pose.rs:38-46), Rodrigues.
Mat3 so3_exp(const Vec3& omega) {
    const double angle = norm(omega);
    const Mat3 k = skew(omega);
    const Mat3 kk = mul(k, k);
    if (angle < kSmallAngle) return add(add(identity(), k), scale(kk, 0.5));
    return add(add(identity(), scale(k, std::sin(angle) / angle)), scale(kk, (1.0 - std::cos(angle)) / (angle * angle)));
}

// so3_left_jacobian (camera_pose.rs:48-57).
Mat3 so3_left_jacobian(const Vec3& omega) {
    const double angle = norm(omega);
    const Mat3 k = skew(omega);
    const Mat3 kk = mul(k, k);
    if (angle < kSmallAngle) return add(add(identity(), scale(k, 0.5)), scale(kk, 1.0 / 6.0));
    const double angle2 = angle * angle;
    return add(add(identity(), scale(k, (1.0 - std::cos(angle)) / angle2)),
               scale(kk, (angle - std::sin(angle)) / (angle2 * angle)));
}

Vec3 vee(const Mat3& s) { return {{s.m[2][1], s.m[0][2], s.m[1][0]}}; }

Mat3 rotation_of(const sp_pinhole_camera& c) {
    Mat3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = c.rotation[i * 3 + j];
    return r;
}

sp_pinhole_camera corrected(const sp_pinhole_camera& initial, const sp_pose_correction& correction,
                            double focal_log_scale) {
    // camera_pose.rs:59-68.
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

sp_pose_gradient pose_gradient(const sp_pinhole_camera& initial, const sp_pose_correction& correction,
                               double focal_log_scale, const sp_camera_gradient& gradient) {
    // camera_pose.rs:81-99.
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

// pose_refinement.rs:30-62: Adam over a few f64 parameters.
struct Moments {
    std::vector<double> first, second;
    uint32_t steps = 0;
    explicit Moments(size_t n) : first(n, 0.0), second(n, 0.0) {}
    void update(double* params, const double* gradient, const double* rates) {
        steps += 1;
        const double beta1 = (double)SP_ADAM_BETA1, beta2 = (double)SP_ADAM_BETA2;
        const double bias1 = 1.0 - std::pow(beta1, (int)steps);
        const double bias2 = 1.0 - std::pow(beta2, (int)steps);
        for (size_t i = 0; i < first.size(); ++i) {
            first[i] = beta1 * first[i] + (1.0 - beta1) * gradient[i];
            second[i] = beta2 * second[i] + (1.0 - beta2) * gradient[i] * gradient[i];
            const double first_hat = first[i] / bias1;
            const double second_hat = second[i] / bias2;
            params[i] -= rates[i] * first_hat / (std::sqrt(second_hat) + (double)SP_ADAM_EPSILON);
        }
    }
};

constexpr uint32_t kFixedView = 0;  // pose_refinement.rs:14

}  // namespace

struct sp_pose_refinement {
    std::vector<sp_pinhole_camera> initial;
    std::vector<sp_pose_correction> corrections;
    double focal_log_scale = 0.0;
    sp_pose_gradient last_gradient{};
    std::vector<Moments> moments;
    Moments focal_moments{1};
    double rotation_rate = 0.0, translation_rate = 0.0, focal_rate = 0.0;
};

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
    p->corrections.assign(view_count, sp_pose_correction{});
    for (uint32_t v = 0; v < view_count; ++v) p->moments.emplace_back(6);
    p->rotation_rate = (double)rates->camera_rotation;
    p->translation_rate = (double)rates->camera_translation * (double)extent;
    p->focal_rate = (double)rates->camera_focal;
    *out = p;
    return SP_OK;
}

void sp_pose_refinement_destroy(sp_pose_refinement* p) { delete p; }

sp_status sp_pose_refinement_camera(const sp_pose_refinement* p, uint32_t view, sp_pinhole_camera* out) {
    if (!p || !out || view >= p->initial.size()) return SP_ERR_INVALID;
    *out = corrected(p->initial[view], p->corrections[view], p->focal_log_scale);
    return SP_OK;
}

sp_status sp_pose_refinement_step(sp_pose_refinement* p, uint32_t view, const sp_camera_gradient* gradient,
                                  float rate_factor) {
    if (!p || !gradient || view >= p->initial.size()) return SP_ERR_INVALID;
    // pose_refinement.rs:113-163.
    if (!(rate_factor > 0.0f && rate_factor <= 1.0f)) return SP_ERR_INVALID;
    const sp_pose_gradient g = pose_gradient(p->initial[view], p->corrections[view], p->focal_log_scale, *gradient);
    bool finite = std::isfinite(g.focal_log_scale);
    for (int i = 0; i < 3; ++i) finite = finite && std::isfinite(g.rotation[i]) && std::isfinite(g.translation[i]);
    if (!finite) return SP_ERR_NONFINITE;
    p->last_gradient = g;
    const double factor = (double)rate_factor;
    if (view != kFixedView) {
        sp_pose_correction& c = p->corrections[view];
        double params[6] = {c.rotation[0], c.rotation[1], c.rotation[2], c.translation[0], c.translation[1],
                            c.translation[2]};
        const double grads[6] = {g.rotation[0], g.rotation[1], g.rotation[2],
                                 g.translation[0], g.translation[1], g.translation[2]};
        const double rr = p->rotation_rate * factor, tr = p->translation_rate * factor;
        const double rates[6] = {rr, rr, rr, tr, tr, tr};
        p->moments[view].update(params, grads, rates);
        for (int i = 0; i < 3; ++i) {
            c.rotation[i] = params[i];
            c.translation[i] = params[3 + i];
        }
    }
    double focal = p->focal_log_scale;
    const double fg = g.focal_log_scale, fr = p->focal_rate * factor;
    p->focal_moments.update(&focal, &fg, &fr);
    p->focal_log_scale = focal;
    return SP_OK;
}

sp_status sp_pose_refinement_correction(const sp_pose_refinement* p, uint32_t view, sp_pose_correction* out) {
    if (!p || !out || view >= p->corrections.size()) return SP_ERR_INVALID;
    *out = p->corrections[view];
    return SP_OK;
}

double sp_pose_refinement_focal_scale(const sp_pose_refinement* p) { return p ? std::exp(p->focal_log_scale) : 0.0; }

sp_status sp_pose_refinement_last_gradient(const sp_pose_refinement* p, sp_pose_gradient* out) {
    if (!p || !out) return SP_ERR_INVALID;
    *out = p->last_gradient;
    return SP_OK;
}

}  // extern "C"
