// CPU oracle of the differentiable Gaussian-splatting path — TEST INFRASTRUCTURE ONLY.
//
// A plain C++ restatement of the reference's WGSL kernels (instantsplat-rs/src/shaders/)
// and the Rust host arithmetic around them. See splat_oracle.h for who may call it and
// how it is pinned. Compiled with -ffp-contract=off and without fast-math, so every
// expression is evaluated in the order written, in IEEE single precision.
//
// Matrices are row-major arrays here: X[i][j] is row i, column j. WGSL's matrices are
// column-major (m[c][r]); each translation below says which entry it reads.

#include "splat_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/splat_constants.h"
#include "../include/splat_math.h"

namespace {

int g_threads = 0;

int threads() {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

uint32_t stride_of(uint32_t sh_degree) { return SP_PARAM_STRIDE(sh_degree); }

// world_to_camera (common.wgsl:72-75): dot(rows[i], (p, 1)), summed left to right.
inline float row_dot(const float r[4], float x, float y, float z) {
    return r[0] * x + r[1] * y + r[2] * z + r[3] * 1.0f;
}

// SH basis of degree <= 3 at unit direction (x, y, z): (d + 1)^2 values.
void sh_basis(uint32_t degree, float x, float y, float z, float* b) {
    b[0] = SP_SH_C0;
    if (degree < 1) return;
    b[1] = -SP_SH_C1 * y;
    b[2] = SP_SH_C1 * z;
    b[3] = -SP_SH_C1 * x;
    if (degree < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
    b[4] = SP_SH_C2_0 * xy;
    b[5] = SP_SH_C2_1 * yz;
    b[6] = SP_SH_C2_2 * (2.0f * zz - xx - yy);
    b[7] = SP_SH_C2_3 * xz;
    b[8] = SP_SH_C2_4 * (xx - yy);
    if (degree < 3) return;
    b[9] = SP_SH_C3_0 * y * (3.0f * xx - yy);
    b[10] = SP_SH_C3_1 * xy * z;
    b[11] = SP_SH_C3_2 * y * (4.0f * zz - xx - yy);
    b[12] = SP_SH_C3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    b[13] = SP_SH_C3_4 * x * (4.0f * zz - xx - yy);
    b[14] = SP_SH_C3_5 * z * (xx - yy);
    b[15] = SP_SH_C3_6 * x * (xx - 3.0f * yy);
}

// d basis_k / d(x, y, z) for the basis above (k >= 1).
void sh_basis_gradient(uint32_t degree, float x, float y, float z, float (*g)[3]) {
    for (int k = 0; k < 16; ++k) g[k][0] = g[k][1] = g[k][2] = 0.0f;
    if (degree < 1) return;
    g[1][1] = -SP_SH_C1;
    g[2][2] = SP_SH_C1;
    g[3][0] = -SP_SH_C1;
    if (degree < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    g[4][0] = SP_SH_C2_0 * y;
    g[4][1] = SP_SH_C2_0 * x;
    g[5][1] = SP_SH_C2_1 * z;
    g[5][2] = SP_SH_C2_1 * y;
    g[6][0] = -2.0f * SP_SH_C2_2 * x;
    g[6][1] = -2.0f * SP_SH_C2_2 * y;
    g[6][2] = 4.0f * SP_SH_C2_2 * z;
    g[7][0] = SP_SH_C2_3 * z;
    g[7][2] = SP_SH_C2_3 * x;
    g[8][0] = 2.0f * SP_SH_C2_4 * x;
    g[8][1] = -2.0f * SP_SH_C2_4 * y;
    if (degree < 3) return;
    g[9][0] = SP_SH_C3_0 * 6.0f * x * y;
    g[9][1] = SP_SH_C3_0 * (3.0f * xx - 3.0f * yy);
    g[10][0] = SP_SH_C3_1 * y * z;
    g[10][1] = SP_SH_C3_1 * x * z;
    g[10][2] = SP_SH_C3_1 * x * y;
    g[11][0] = SP_SH_C3_2 * -2.0f * x * y;
    g[11][1] = SP_SH_C3_2 * (4.0f * zz - xx - 3.0f * yy);
    g[11][2] = SP_SH_C3_2 * 8.0f * y * z;
    g[12][0] = SP_SH_C3_3 * -6.0f * x * z;
    g[12][1] = SP_SH_C3_3 * -6.0f * y * z;
    g[12][2] = SP_SH_C3_3 * (6.0f * zz - 3.0f * xx - 3.0f * yy);
    g[13][0] = SP_SH_C3_4 * (4.0f * zz - 3.0f * xx - yy);
    g[13][1] = SP_SH_C3_4 * -2.0f * x * y;
    g[13][2] = SP_SH_C3_4 * 8.0f * x * z;
    g[14][0] = SP_SH_C3_5 * 2.0f * x * z;
    g[14][1] = SP_SH_C3_5 * -2.0f * y * z;
    g[14][2] = SP_SH_C3_5 * (xx - yy);
    g[15][0] = SP_SH_C3_6 * (3.0f * xx - 3.0f * yy);
    g[15][1] = SP_SH_C3_6 * -6.0f * x * y;
}

// Camera centre in world space, -W^T t, and the unit direction from it to `pos`.
void view_direction(const sp_camera_uniform& cam, const float* pos, float dir[3], float* length) {
    const float (*r)[4] = cam.world_to_camera_rows;
    float c[3];
    for (int j = 0; j < 3; ++j) c[j] = -(r[0][j] * r[0][3] + r[1][j] * r[1][3] + r[2][j] * r[2][3]);
    const float v[3] = {pos[0] - c[0], pos[1] - c[1], pos[2] - c[2]};
    const float len = std::sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    dir[0] = v[0] / len;
    dir[1] = v[1] / len;
    dir[2] = v[2] / len;
    *length = len;
}

// Colour before the clamp at 0: SH_C0 * dc + 0.5 at degree 0 (project_forward.wgsl:83-86),
// the full SH sum + 0.5 above.
void raw_color(const float* params, uint32_t sh_degree, const sp_camera_uniform& cam, float out[3]) {
    const float* sh = params + SP_SLOT_SH;
    if (sh_degree == 0) {
        for (int c = 0; c < 3; ++c) out[c] = SP_SH_C0 * sh[c] + 0.5f;
        return;
    }
    float dir[3], len;
    view_direction(cam, params, dir, &len);
    float b[16];
    sh_basis(sh_degree, dir[0], dir[1], dir[2], b);
    const int count = (int)((sh_degree + 1) * (sh_degree + 1));
    for (int c = 0; c < 3; ++c) {
        float s = b[0] * sh[c];
        for (int k = 1; k < count; ++k) s = s + b[k] * sh[3 * k + c];
        out[c] = s + 0.5f;
    }
}

// quaternion_to_matrix (common.wgsl:92-103): R[i][k] = column k, row i.
void rotation_of(float r, float x, float y, float z, float R[3][3]) {
    // Column 0.
    R[0][0] = 1.0f - 2.0f * (y * y + z * z);
    R[1][0] = 2.0f * (x * y + r * z);
    R[2][0] = 2.0f * (x * z - r * y);
    // Column 1.
    R[0][1] = 2.0f * (x * y - r * z);
    R[1][1] = 1.0f - 2.0f * (x * x + z * z);
    R[2][1] = 2.0f * (y * z + r * x);
    // Column 2.
    R[0][2] = 2.0f * (x * z + r * y);
    R[1][2] = 2.0f * (y * z - r * x);
    R[2][2] = 1.0f - 2.0f * (x * x + y * y);
}

struct Geometry {
    float pc[3];
    float scale[3];
    float q[4];       // normalised (w, x, y, z)
    float q_length;   // length of the raw quaternion
    float R[3][3];
    float M[3][3];
    float Sigma[3][3];
    float limit[2];
    bool clamped[2];
    float tx, ty, z2;
    float J[2][3];
    float W[3][3];
    float T[2][3];
    float a, b, c, det;
};

// The forward quantities shared by project_forward.wgsl:43-86 and project_backward.wgsl:65-97.
void geometry(const float* p, const sp_camera_uniform& cam, Geometry& g) {
    const float (*rows)[4] = cam.world_to_camera_rows;
    g.pc[0] = row_dot(rows[0], p[0], p[1], p[2]);
    g.pc[1] = row_dot(rows[1], p[0], p[1], p[2]);
    g.pc[2] = row_dot(rows[2], p[0], p[1], p[2]);
    for (int k = 0; k < 3; ++k) g.scale[k] = sp_expf(p[SP_SLOT_LOG_SCALE + k]);
    const float* qr = p + SP_SLOT_ROTATION;
    g.q_length = std::sqrt(qr[0] * qr[0] + qr[1] * qr[1] + qr[2] * qr[2] + qr[3] * qr[3]);
    for (int k = 0; k < 4; ++k) g.q[k] = qr[k] / g.q_length;
    rotation_of(g.q[0], g.q[1], g.q[2], g.q[3], g.R);
    // m = mat3x3(r[0] * scale.x, r[1] * scale.y, r[2] * scale.z): column k scaled.
    for (int i = 0; i < 3; ++i)
        for (int k = 0; k < 3; ++k) g.M[i][k] = g.R[i][k] * g.scale[k];
    // sigma = m * transpose(m).
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) g.Sigma[i][j] = g.M[i][0] * g.M[j][0] + g.M[i][1] * g.M[j][1] + g.M[i][2] * g.M[j][2];
    const float fx = cam.focal[0], fy = cam.focal[1];
    g.limit[0] = SP_VIEW_LIMIT_FACTOR * (float)cam.width / (2.0f * fx);
    g.limit[1] = SP_VIEW_LIMIT_FACTOR * (float)cam.height / (2.0f * fy);
    const float xz = g.pc[0] / g.pc[2];
    const float yz = g.pc[1] / g.pc[2];
    g.clamped[0] = std::fabs(xz) > g.limit[0];
    g.clamped[1] = std::fabs(yz) > g.limit[1];
    // clamp(e, lo, hi) = min(max(e, lo), hi).
    g.tx = std::min(std::max(xz, -g.limit[0]), g.limit[0]) * g.pc[2];
    g.ty = std::min(std::max(yz, -g.limit[1]), g.limit[1]) * g.pc[2];
    g.z2 = g.pc[2] * g.pc[2];
    g.J[0][0] = fx / g.pc[2];
    g.J[0][1] = 0.0f;
    g.J[0][2] = -fx * g.tx / g.z2;
    g.J[1][0] = 0.0f;
    g.J[1][1] = fy / g.pc[2];
    g.J[1][2] = -fy * g.ty / g.z2;
    // world_to_camera_rotation (common.wgsl:78-85): W[k][j] = rows[k][j].
    for (int k = 0; k < 3; ++k)
        for (int j = 0; j < 3; ++j) g.W[k][j] = rows[k][j];
    // t = j * w.
    for (int r = 0; r < 2; ++r)
        for (int j = 0; j < 3; ++j) g.T[r][j] = g.J[r][0] * g.W[0][j] + g.J[r][1] * g.W[1][j] + g.J[r][2] * g.W[2][j];
    // cov2d = (t * sigma) * transpose(t).
    float TS[2][3];
    for (int r = 0; r < 2; ++r)
        for (int j = 0; j < 3; ++j)
            TS[r][j] = g.T[r][0] * g.Sigma[0][j] + g.T[r][1] * g.Sigma[1][j] + g.T[r][2] * g.Sigma[2][j];
    float cov[2][2];
    for (int r = 0; r < 2; ++r)
        for (int s = 0; s < 2; ++s) cov[r][s] = TS[r][0] * g.T[s][0] + TS[r][1] * g.T[s][1] + TS[r][2] * g.T[s][2];
    g.a = cov[0][0] + SP_COVARIANCE_BLUR;
    g.b = cov[0][1];  // cov2d[1][0]: column 1, row 0
    g.c = cov[1][1] + SP_COVARIANCE_BLUR;
    g.det = g.a * g.c - g.b * g.b;
}

void culled(sp_projected& out, uint32_t& count) {
    std::memset(&out, 0, sizeof(out));
    count = 0;
}

// project_forward.wgsl:19-93 for one Gaussian.
void project_one(const float* p, uint32_t sh_degree, const sp_camera_uniform& cam, sp_projected& out,
                 uint32_t& count) {
    const float (*rows)[4] = cam.world_to_camera_rows;
    const float pz = row_dot(rows[2], p[0], p[1], p[2]);
    if (pz < SP_NEAR_Z) {
        culled(out, count);
        return;
    }
    Geometry g;
    geometry(p, cam, g);
    if (g.det <= 0.0f) {
        culled(out, count);
        return;
    }
    const float conic[3] = {g.c / g.det, -g.b / g.det, g.a / g.det};
    const float mid = 0.5f * (g.a + g.c);
    const float largest = mid + std::sqrt(std::max(0.1f, mid * mid - g.det));
    const float radius = std::ceil(3.0f * std::sqrt(largest));
    const float mean[2] = {cam.focal[0] * g.pc[0] / g.pc[2] + cam.principal_point[0],
                           cam.focal[1] * g.pc[1] / g.pc[2] + cam.principal_point[1]};
    const float tiles[2] = {(float)cam.tiles_x, (float)cam.tiles_y};
    float tmin[2], tmax[2];
    for (int k = 0; k < 2; ++k) {
        tmin[k] = std::min(std::max(std::floor((mean[k] - radius) / (float)SP_TILE), 0.0f), tiles[k]);
        tmax[k] = std::min(std::max(std::floor((mean[k] + radius) / (float)SP_TILE) + 1.0f, 0.0f), tiles[k]);
    }
    const float cnt = (tmax[0] - tmin[0]) * (tmax[1] - tmin[1]);
    if (cnt <= 0.0f) {
        culled(out, count);
        return;
    }
    std::memset(&out, 0, sizeof(out));
    out.mean[0] = mean[0];
    out.mean[1] = mean[1];
    out.conic[0] = conic[0];
    out.conic[1] = conic[1];
    out.conic[2] = conic[2];
    out.depth = g.pc[2];
    float col[3];
    raw_color(p, sh_degree, cam, col);
    for (int c = 0; c < 3; ++c) out.color[c] = std::max(0.0f, col[c]);
    out.opacity = sp_sigmoid(p[SP_SLOT_OPACITY]);
    out.radius = (uint32_t)radius;
    out.tile_min[0] = (uint32_t)tmin[0];
    out.tile_min[1] = (uint32_t)tmin[1];
    out.tile_max[0] = (uint32_t)tmax[0];
    out.tile_max[1] = (uint32_t)tmax[1];
    count = (uint32_t)cnt;
}

inline uint64_t key_of(int key_mode, uint32_t tile, float depth) {
    const uint32_t bits = sp_float_to_bits(depth);
    if (key_mode == SP_KEYS_FULL32) return ((uint64_t)tile << 32) | bits;
    return ((uint64_t)tile << SP_DEPTH_BITS) | (bits >> (32 - SP_DEPTH_BITS));
}

inline uint32_t tile_of(int key_mode, uint64_t key) {
    return (uint32_t)(key >> (key_mode == SP_KEYS_FULL32 ? 32 : SP_DEPTH_BITS));
}

// The SSIM window along one axis (common.wgsl:110-122).
void ssim_taps(float taps[2 * SP_SSIM_RADIUS + 1]) {
    float sum = 0.0f;
    for (int k = 0; k <= 2 * SP_SSIM_RADIUS; ++k) {
        const float d = (float)(k - SP_SSIM_RADIUS);
        taps[k] = sp_expf(-d * d / (2.0f * SP_SSIM_SIGMA * SP_SSIM_SIGMA));
        sum += taps[k];
    }
    for (int k = 0; k <= 2 * SP_SSIM_RADIUS; ++k) taps[k] /= sum;
}

inline float sign_of(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

}  // namespace

extern "C" {

void or_set_threads(int t) { g_threads = t; }
int or_get_threads(void) { return threads(); }

float or_libm_expf(float x) { return std::exp(x); }
float or_sp_expf(float x) { return sp_expf(x); }
float or_sp_expf_exact(float x) { return sp_expf_exact(x); }

void or_project(const float* params, uint64_t n, uint32_t sh_degree, const sp_camera_uniform* cam,
                sp_projected* out, uint32_t* tile_counts) {
    const uint32_t stride = stride_of(sh_degree);
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t g = 0; g < (int64_t)n; ++g) project_one(params + g * stride, sh_degree, *cam, out[g], tile_counts[g]);
}

uint64_t or_scan(const uint32_t* counts, uint64_t n, uint64_t capacity, uint32_t* offsets,
                 sp_intersection_meta* meta) {
    uint64_t total = 0;
    for (uint64_t g = 0; g < n; ++g) {
        offsets[g] = (uint32_t)total;
        total += counts[g];
    }
    const uint64_t count = std::min<uint64_t>(total, capacity);
    meta->count = (uint32_t)count;
    meta->overflow = total > capacity ? 1u : 0u;
    meta->sort_blocks = (uint32_t)((count + 1023) / 1024);
    meta->histogram_length = 16u * meta->sort_blocks;
    meta->capacity = (uint32_t)capacity;
    return total;
}

uint64_t or_bin(const sp_projected* proj, const uint32_t* offsets, uint64_t n, const sp_camera_uniform* cam,
                uint64_t capacity, int key_mode, uint64_t* sorted_keys, uint32_t* sorted_gaussians,
                uint32_t* sorted_slots, uint32_t* ranges) {
    uint64_t total = 0;
    for (uint64_t g = 0; g < n; ++g) {
        const sp_projected& p = proj[g];
        if (p.radius != 0) total += (uint64_t)(p.tile_max[0] - p.tile_min[0]) * (p.tile_max[1] - p.tile_min[1]);
    }
    const uint64_t count = std::min<uint64_t>(total, capacity);
    std::vector<uint64_t> keys(count);
    std::vector<uint32_t> gauss(count);
    // emit_tile_keys.wgsl:13-36: row-major over the rectangle, dropped at the capacity.
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t g = 0; g < (int64_t)n; ++g) {
        const sp_projected& p = proj[g];
        if (p.radius == 0) continue;
        uint64_t index = offsets[g];
        for (uint32_t ty = p.tile_min[1]; ty < p.tile_max[1]; ++ty)
            for (uint32_t tx = p.tile_min[0]; tx < p.tile_max[0]; ++tx) {
                if (index < capacity) {
                    keys[index] = key_of(key_mode, ty * cam->tiles_x + tx, p.depth);
                    gauss[index] = (uint32_t)g;
                }
                ++index;
            }
    }
    // Stable LSD radix sort by key, 8 bits a pass, over the key's significant bits:
    // ties keep emission order (sort.rs:1-3, sort_scatter.wgsl:1-4).
    std::vector<uint32_t> order(count), next(count);
    for (uint64_t i = 0; i < count; ++i) order[i] = (uint32_t)i;
    uint64_t max_key = 0;
    for (uint64_t i = 0; i < count; ++i) max_key = std::max(max_key, keys[i]);
    for (int shift = 0; shift < 64 && (max_key >> shift) != 0; shift += 8) {
        uint64_t histogram[257] = {0};
        for (uint64_t i = 0; i < count; ++i) ++histogram[((keys[order[i]] >> shift) & 255) + 1];
        for (int d = 0; d < 256; ++d) histogram[d + 1] += histogram[d];
        for (uint64_t i = 0; i < count; ++i) next[histogram[(keys[order[i]] >> shift) & 255]++] = order[i];
        order.swap(next);
    }
    for (uint64_t i = 0; i < count; ++i) {
        sorted_keys[i] = keys[order[i]];
        sorted_gaussians[i] = gauss[order[i]];
        sorted_slots[i] = order[i];
    }
    // tile_ranges.wgsl:9-22 over a zeroed buffer (rasterizer.rs:410).
    const uint64_t tiles = (uint64_t)cam->tiles_x * cam->tiles_y;
    std::memset(ranges, 0, tiles * 2 * sizeof(uint32_t));
    for (uint64_t i = 0; i < count; ++i) {
        const uint32_t tile = tile_of(key_mode, sorted_keys[i]);
        if (i == 0 || tile_of(key_mode, sorted_keys[i - 1]) != tile) ranges[2 * tile] = (uint32_t)i;
        if (i + 1 == count || tile_of(key_mode, sorted_keys[i + 1]) != tile) ranges[2 * tile + 1] = (uint32_t)(i + 1);
    }
    return count;
}

void or_blend_forward(const sp_projected* proj, const uint32_t* sorted_gaussians, const uint32_t* ranges,
                      const sp_camera_uniform* cam, float* image, uint32_t* contributions) {
    const int64_t tiles = (int64_t)cam->tiles_x * cam->tiles_y;
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads())
    for (int64_t tile = 0; tile < tiles; ++tile) {
        const uint32_t gx = (uint32_t)(tile % cam->tiles_x), gy = (uint32_t)(tile / cam->tiles_x);
        const uint32_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
        for (uint32_t ly = 0; ly < SP_TILE; ++ly)
            for (uint32_t lx = 0; lx < SP_TILE; ++lx) {
                const uint32_t px = gx * SP_TILE + lx, py = gy * SP_TILE + ly;
                if (px >= cam->width || py >= cam->height) continue;
                const float pixel[2] = {(float)px, (float)py};
                float transmittance = 1.0f;
                float color[3] = {0.0f, 0.0f, 0.0f};
                uint32_t contributed = 0;
                // rasterize_forward.wgsl:43-78, the batches flattened: a finished pixel
                // idles through the rest of the list, which is a break here.
                for (uint32_t j = 0; j < end - start; ++j) {
                    const sp_projected& p = proj[sorted_gaussians[start + j]];
                    const float d[2] = {p.mean[0] - pixel[0], p.mean[1] - pixel[1]};
                    const float power = -0.5f * (p.conic[0] * d[0] * d[0] + p.conic[2] * d[1] * d[1]) -
                                        p.conic[1] * d[0] * d[1];
                    if (power <= 0.0f) {
                        const float alpha = std::min(SP_MAX_ALPHA, p.opacity * sp_expf_exact(power));
                        if (alpha >= SP_MIN_ALPHA) {
                            const float next = transmittance * (1.0f - alpha);
                            if (next < SP_MIN_TRANSMITTANCE) break;
                            for (int c = 0; c < 3; ++c) color[c] += p.color[c] * alpha * transmittance;
                            transmittance = next;
                            contributed = j + 1;
                        }
                    }
                }
                const uint64_t index = (uint64_t)py * cam->width + px;
                image[index * 4 + 0] = color[0];
                image[index * 4 + 1] = color[1];
                image[index * 4 + 2] = color[2];
                image[index * 4 + 3] = transmittance;
                contributions[index] = contributed;
            }
    }
}

void or_ssim(const float* image, const float* gt, uint32_t width, uint32_t height, float* partials) {
    float taps[2 * SP_SSIM_RADIUS + 1];
    ssim_taps(taps);
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t py = 0; py < (int64_t)height; ++py)
        for (int64_t px = 0; px < (int64_t)width; ++px) {
            const uint64_t i = (uint64_t)py * width + px;
            float mu_x[3] = {0}, mu_y[3] = {0}, e_xx[3] = {0}, e_yy[3] = {0}, e_xy[3] = {0};
            // ssim_forward.wgsl:48-69.
            for (int dy = -SP_SSIM_RADIUS; dy <= SP_SSIM_RADIUS; ++dy) {
                const int64_t qy = py + dy;
                if (qy < 0 || qy >= (int64_t)height) continue;
                for (int dx = -SP_SSIM_RADIUS; dx <= SP_SSIM_RADIUS; ++dx) {
                    const int64_t qx = px + dx;
                    if (qx < 0 || qx >= (int64_t)width) continue;
                    const float w = taps[dx + SP_SSIM_RADIUS] * taps[dy + SP_SSIM_RADIUS];
                    const uint64_t q = (uint64_t)qy * width + qx;
                    for (int c = 0; c < 3; ++c) {
                        const float x = image[q * 4 + c], y = gt[q * 4 + c];
                        mu_x[c] += w * x;
                        mu_y[c] += w * y;
                        e_xx[c] += w * x * x;
                        e_yy[c] += w * y * y;
                        e_xy[c] += w * x * y;
                    }
                }
            }
            const float mask = gt[i * 4 + 3];
            for (int c = 0; c < 3; ++c) {
                // ssim_forward.wgsl:70-90.
                const float sigma_xx = e_xx[c] - mu_x[c] * mu_x[c];
                const float sigma_yy = e_yy[c] - mu_y[c] * mu_y[c];
                const float sigma_xy = e_xy[c] - mu_x[c] * mu_y[c];
                const float a = mu_x[c] * mu_x[c] + mu_y[c] * mu_y[c] + SP_SSIM_C1;
                const float b = sigma_xx + sigma_yy + SP_SSIM_C2;
                const float cc = 2.0f * mu_x[c] * mu_y[c] + SP_SSIM_C1;
                const float d = 2.0f * sigma_xy + SP_SSIM_C2;
                const float ab = a * b;
                const float ssim = cc * d / ab;
                const float d_mu = mask * (2.0f * mu_y[c] * (d - cc) / ab - 2.0f * mu_x[c] * cc * d * (b - a) / (ab * ab));
                const float d_exx = mask * (-cc * d / (ab * b));
                const float d_exy = mask * (2.0f * cc / ab);
                const uint64_t base = (i * 3 + c) * 4;
                partials[base + 0] = ssim;
                partials[base + 1] = d_mu;
                partials[base + 2] = d_exx;
                partials[base + 3] = d_exy;
            }
        }
}

void or_loss(const float* image, const float* gt, const float* partials, uint32_t width, uint32_t height,
             const sp_loss_weights* weights, float* loss_gradient, float* pixel_loss) {
    float taps[2 * SP_SSIM_RADIUS + 1];
    ssim_taps(taps);
    const float pixels = (float)((uint64_t)width * height);
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t py = 0; py < (int64_t)height; ++py)
        for (int64_t px = 0; px < (int64_t)width; ++px) {
            const uint64_t i = (uint64_t)py * width + px;
            float d_mu[3] = {0}, d_exx[3] = {0}, d_exy[3] = {0};
            // loss.wgsl:44-63.
            for (int dy = -SP_SSIM_RADIUS; dy <= SP_SSIM_RADIUS; ++dy) {
                const int64_t qy = py + dy;
                if (qy < 0 || qy >= (int64_t)height) continue;
                for (int dx = -SP_SSIM_RADIUS; dx <= SP_SSIM_RADIUS; ++dx) {
                    const int64_t qx = px + dx;
                    if (qx < 0 || qx >= (int64_t)width) continue;
                    const float w = taps[dx + SP_SSIM_RADIUS] * taps[dy + SP_SSIM_RADIUS];
                    const uint64_t q = (uint64_t)qy * width + qx;
                    for (int c = 0; c < 3; ++c) {
                        const uint64_t base = (q * 3 + c) * 4;
                        d_mu[c] += w * partials[base + 1];
                        d_exx[c] += w * partials[base + 2];
                        d_exy[c] += w * partials[base + 3];
                    }
                }
            }
            // loss.wgsl:64-96.
            const float mask = gt[i * 4 + 3];
            float dssim = 0.0f;
            for (int c = 0; c < 3; ++c) dssim += mask * (1.0f - partials[(i * 3 + c) * 4]);
            float l1 = 0.0f;
            for (int c = 0; c < 3; ++c) {
                const float x = image[i * 4 + c], y = gt[i * 4 + c];
                const float d_ssim = d_mu[c] + 2.0f * x * d_exx[c] + y * d_exy[c];
                const float difference = x - y;
                loss_gradient[i * 4 + c] =
                    (weights->l1 * mask * sign_of(difference) - weights->dssim * d_ssim) / (3.0f * pixels);
            }
            const float dx0 = image[i * 4 + 0] - gt[i * 4 + 0];
            const float dx1 = image[i * 4 + 1] - gt[i * 4 + 1];
            const float dx2 = image[i * 4 + 2] - gt[i * 4 + 2];
            const float coverage = 1.0f - image[i * 4 + 3];
            const float alpha_difference = coverage - gt[i * 4 + 3];
            loss_gradient[i * 4 + 3] = -weights->alpha * sign_of(alpha_difference) / pixels;
            l1 = mask * (std::fabs(dx0) + std::fabs(dx1) + std::fabs(dx2)) / 3.0f;
            const float alpha_error = std::fabs(alpha_difference);
            pixel_loss[i * 4 + 0] = l1;
            pixel_loss[i * 4 + 1] = alpha_error;
            pixel_loss[i * 4 + 2] = dssim / 3.0f;
            pixel_loss[i * 4 + 3] =
                weights->l1 * l1 + weights->alpha * alpha_error + weights->dssim * dssim / 3.0f;
        }
}

// The blend backward; with `magnitudes` non-null, each slot also receives, per component, the
// sum over its pixels of the term's rounding scale (in double): the magnitude of everything
// the term is computed from, so that reordered sums, cancellation inside dL/dalpha (the
// difference of T (g . c) and (g . behind + g_T T_final) / (1 - alpha)) and the rounding the
// transmittance accumulates over the pixel's contributors are all bounded by a small multiple
// of 2^-24 times it. Per (pixel, Gaussian):
//   colour c:   |g_c alpha T| (1 + n)
//   dL/dalpha:  (T sum_c |g_c colour_c| + (sum_c |g_c behind_c| + |g_T T_final|) / (1 - alpha)) (1 + n)
//   opacity:    that times e^power;   d_power: that times opacity e^power
//   mean:       |d_power| scale times (|conic_0 d_0| + |conic_1 d_1|) and (|conic_1 d_0| + |conic_2 d_1|)
//   conic:      |d_power| scale times d_0^2 / 2, |d_0 d_1|, d_1^2 / 2
// with n the pixel's contributor count (the length of its transmittance product).
static void blend_backward(const sp_projected* proj, const uint32_t* sorted_gaussians, const uint32_t* sorted_slots,
                           const uint32_t* ranges, const sp_camera_uniform* cam, const float* image,
                           const uint32_t* contributions, const float* loss_gradient, float* intersection_gradients,
                           double* magnitudes) {
    const int64_t tiles = (int64_t)cam->tiles_x * cam->tiles_y;
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads())
    for (int64_t tile = 0; tile < tiles; ++tile) {
        const uint32_t gx = (uint32_t)(tile % cam->tiles_x), gy = (uint32_t)(tile / cam->tiles_x);
        const uint32_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
        const uint32_t count = end - start;
        if (count == 0) continue;
        std::vector<float> sums((size_t)count * SP_GRAD_STRIDE, 0.0f);
        std::vector<double> mags(magnitudes ? (size_t)count * SP_GRAD_STRIDE : 0, 0.0);
        for (uint32_t ly = 0; ly < SP_TILE; ++ly)
            for (uint32_t lx = 0; lx < SP_TILE; ++lx) {
                const uint32_t px = gx * SP_TILE + lx, py = gy * SP_TILE + ly;
                if (px >= cam->width || py >= cam->height) continue;
                const uint64_t index = (uint64_t)py * cam->width + px;
                const float pixel[2] = {(float)px, (float)py};
                // rasterize_backward.wgsl:35-49.
                float transmittance = image[index * 4 + 3];
                const uint32_t contributed = contributions[index];
                const float* gradient = loss_gradient + index * 4;
                float behind[4] = {0.0f, 0.0f, 0.0f, transmittance};
                // rasterize_backward.wgsl:58-101, back to front over the contributors.
                for (int64_t j = (int64_t)std::min(contributed, count) - 1; j >= 0; --j) {
                    const sp_projected& p = proj[sorted_gaussians[start + j]];
                    const float d[2] = {p.mean[0] - pixel[0], p.mean[1] - pixel[1]};
                    const float* conic = p.conic;
                    const float power = -0.5f * (conic[0] * d[0] * d[0] + conic[2] * d[1] * d[1]) - conic[1] * d[0] * d[1];
                    if (power > 0.0f) continue;
                    const float gaussian = sp_expf_exact(power);
                    const float opacity = p.opacity;
                    const float alpha_unclamped = opacity * gaussian;
                    const float alpha = std::min(SP_MAX_ALPHA, alpha_unclamped);
                    if (alpha < SP_MIN_ALPHA) continue;
                    transmittance = transmittance / (1.0f - alpha);
                    const float color[4] = {p.color[0], p.color[1], p.color[2], 0.0f};
                    float d_alpha = 0.0f;
                    for (int c = 0; c < 4; ++c)
                        d_alpha += gradient[c] * (color[c] * transmittance - behind[c] / (1.0f - alpha));
                    float* s = &sums[(size_t)j * SP_GRAD_STRIDE];
                    float term[SP_GRAD_STRIDE] = {};
                    for (int c = 0; c < 3; ++c) term[5 + c] = gradient[c] * alpha * transmittance;
                    for (int c = 0; c < 4; ++c) behind[c] += color[c] * alpha * transmittance;
                    const bool unclamped = alpha_unclamped < SP_MAX_ALPHA;
                    if (unclamped) {
                        term[8] = d_alpha * gaussian;
                        const float d_power = d_alpha * opacity * gaussian;
                        term[0] = -d_power * (conic[0] * d[0] + conic[1] * d[1]);
                        term[1] = -d_power * (conic[1] * d[0] + conic[2] * d[1]);
                        term[2] = -0.5f * d_power * d[0] * d[0];
                        term[3] = -d_power * d[0] * d[1];
                        term[4] = -0.5f * d_power * d[1] * d[1];
                    }
                    for (int c = 5; c < 8; ++c) s[c] += term[c];
                    if (unclamped)
                        for (int c : {8, 0, 1, 2, 3, 4}) s[c] += term[c];
                    if (magnitudes) {
                        double* m = &mags[(size_t)j * SP_GRAD_STRIDE];
                        const double depth = 1.0 + (double)contributed, t = transmittance;
                        for (int c = 0; c < 3; ++c) m[5 + c] += std::fabs((double)term[5 + c]) * depth;
                        if (unclamped) {
                            double parts = 0.0, behind_parts = std::fabs((double)gradient[3]) * (double)image[index * 4 + 3];
                            for (int c = 0; c < 3; ++c) {
                                parts += std::fabs((double)gradient[c] * (double)color[c]);
                                behind_parts += std::fabs((double)gradient[c] * ((double)behind[c] - (double)color[c] * alpha * t));
                            }
                            const double da = (t * parts + behind_parts / (1.0 - (double)alpha)) * depth;
                            const double dp = da * (double)opacity * (double)gaussian;
                            const double d0 = d[0], d1 = d[1];
                            m[8] += da * (double)gaussian;
                            m[0] += dp * (std::fabs(conic[0] * d0) + std::fabs(conic[1] * d1));
                            m[1] += dp * (std::fabs(conic[1] * d0) + std::fabs(conic[2] * d1));
                            m[2] += dp * 0.5 * d0 * d0;
                            m[3] += dp * std::fabs(d0 * d1);
                            m[4] += dp * 0.5 * d1 * d1;
                        }
                    }
                }
            }
        for (uint32_t j = 0; j < count; ++j) {
            float* out = intersection_gradients + (uint64_t)sorted_slots[start + j] * SP_GRAD_STRIDE;
            for (int c = 0; c < SP_GRAD_STRIDE; ++c) out[c] = sums[(size_t)j * SP_GRAD_STRIDE + c];
            if (magnitudes) {
                double* m = magnitudes + (uint64_t)sorted_slots[start + j] * SP_GRAD_STRIDE;
                for (int c = 0; c < SP_GRAD_STRIDE; ++c) m[c] = mags[(size_t)j * SP_GRAD_STRIDE + c];
            }
        }
    }
}

void or_blend_backward(const sp_projected* proj, const uint32_t* sorted_gaussians, const uint32_t* sorted_slots,
                       const uint32_t* ranges, const sp_camera_uniform* cam, const float* image,
                       const uint32_t* contributions, const float* loss_gradient, float* intersection_gradients) {
    blend_backward(proj, sorted_gaussians, sorted_slots, ranges, cam, image, contributions, loss_gradient,
                   intersection_gradients, nullptr);
}

void or_blend_backward_magnitudes(const sp_projected* proj, const uint32_t* sorted_gaussians,
                                  const uint32_t* sorted_slots, const uint32_t* ranges, const sp_camera_uniform* cam,
                                  const float* image, const uint32_t* contributions, const float* loss_gradient,
                                  float* intersection_gradients, double* magnitudes) {
    blend_backward(proj, sorted_gaussians, sorted_slots, ranges, cam, image, contributions, loss_gradient,
                   intersection_gradients, magnitudes);
}

void or_project_backward(const float* params, uint64_t n, uint32_t sh_degree, const sp_camera_uniform* cam,
                         const sp_projected* proj, const uint32_t* offsets, const float* intersection_gradients,
                         uint64_t capacity, float* param_gradients, float* camera_gradient,
                         sp_densify_stats* stats) {
    const uint32_t stride = stride_of(sh_degree);
    const int64_t groups = (int64_t)((n + 255) / 256);
    std::vector<float> partials((size_t)groups * SP_CAMERA_GRAD_STRIDE, 0.0f);
    const float fx = cam->focal[0], fy = cam->focal[1];
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t group = 0; group < groups; ++group) {
        std::vector<float> local(256 * SP_CAMERA_GRAD_STRIDE, 0.0f);
        for (int t = 0; t < 256; ++t) {
            const uint64_t gi = (uint64_t)group * 256 + t;
            if (gi >= n) continue;
            float* grads = param_gradients + gi * stride;
            for (uint32_t k = 0; k < stride; ++k) grads[k] = 0.0f;
            float* cgrad = &local[(size_t)t * SP_CAMERA_GRAD_STRIDE];
            const sp_projected& p = proj[gi];
            if (p.radius == 0) continue;
            // project_backward.wgsl:38-55.
            const uint32_t count = (p.tile_max[0] - p.tile_min[0]) * (p.tile_max[1] - p.tile_min[1]);
            float d_mean[2] = {0, 0}, d_conic[3] = {0, 0, 0}, d_color[3] = {0, 0, 0}, d_opacity = 0.0f;
            for (uint32_t k = 0; k < count; ++k) {
                const uint64_t slot = (uint64_t)offsets[gi] + k;
                if (slot >= capacity) break;
                const float* s = intersection_gradients + slot * SP_GRAD_STRIDE;
                d_mean[0] += s[0];
                d_mean[1] += s[1];
                d_conic[0] += s[2];
                d_conic[1] += s[3];
                d_conic[2] += s[4];
                d_color[0] += s[5];
                d_color[1] += s[6];
                d_color[2] += s[7];
                d_opacity += s[8];
            }
            // project_backward.wgsl:56-63.
            const float half_image[2] = {0.5f * (float)cam->width, 0.5f * (float)cam->height};
            const float m0 = d_mean[0] * half_image[0], m1 = d_mean[1] * half_image[1];
            sp_densify_stats& st = stats[gi];
            st.mean_gradient_sum = st.mean_gradient_sum + std::sqrt(m0 * m0 + m1 * m1);
            st.visible_count = st.visible_count + 1.0f;
            st.max_radius = std::max(st.max_radius, (float)p.radius);
            st._pad = 0.0f;

            const float* prm = params + gi * stride;
            Geometry g;
            geometry(prm, *cam, g);
            if (g.det <= 0.0f) continue;
            const float* pc = g.pc;
            const float z3 = g.z2 * pc[2];
            // project_backward.wgsl:103-110: opacity and colour.
            const float opacity = p.opacity;
            grads[SP_SLOT_OPACITY] = d_opacity * opacity * (1.0f - opacity);
            float color_raw[3];
            raw_color(prm, sh_degree, *cam, color_raw);
            float d_col[3];
            for (int c = 0; c < 3; ++c) d_col[c] = color_raw[c] > 0.0f ? d_color[c] : 0.0f;
            float d_position_sh[3] = {0.0f, 0.0f, 0.0f};
            if (sh_degree == 0) {
                for (int c = 0; c < 3; ++c)
                    grads[SP_SLOT_SH + c] = SP_SH_C0 * d_color[c] * (color_raw[c] > 0.0f ? 1.0f : 0.0f);
            } else {
                float dir[3], len;
                view_direction(*cam, prm, dir, &len);
                float b[16], bg[16][3];
                sh_basis(sh_degree, dir[0], dir[1], dir[2], b);
                sh_basis_gradient(sh_degree, dir[0], dir[1], dir[2], bg);
                const int kcount = (int)((sh_degree + 1) * (sh_degree + 1));
                float d_dir[3] = {0.0f, 0.0f, 0.0f};
                for (int k = 0; k < kcount; ++k)
                    for (int c = 0; c < 3; ++c) {
                        grads[SP_SLOT_SH + 3 * k + c] = b[k] * d_col[c];
                        const float w = d_col[c] * prm[SP_SLOT_SH + 3 * k + c];
                        for (int a = 0; a < 3; ++a) d_dir[a] += w * bg[k][a];
                    }
                const float dd = dir[0] * d_dir[0] + dir[1] * d_dir[1] + dir[2] * d_dir[2];
                for (int a = 0; a < 3; ++a) d_position_sh[a] = (d_dir[a] - dir[a] * dd) / len;
            }
            // project_backward.wgsl:112-121: dL/dcov2d from dL/dconic.
            const float C[2][2] = {{p.conic[0], p.conic[1]}, {p.conic[1], p.conic[2]}};
            const float dC[2][2] = {{d_conic[0], 0.5f * d_conic[1]}, {0.5f * d_conic[1], d_conic[2]}};
            float CdC[2][2], F[2][2];
            for (int i = 0; i < 2; ++i)
                for (int j = 0; j < 2; ++j) CdC[i][j] = C[i][0] * dC[0][j] + C[i][1] * dC[1][j];
            for (int i = 0; i < 2; ++i)
                for (int j = 0; j < 2; ++j) F[i][j] = -1.0f * (CdC[i][0] * C[0][j] + CdC[i][1] * C[1][j]);
            const float off = 0.5f * (F[1][0] + F[0][1]);
            const float G[2][2] = {{F[0][0], off}, {off, F[1][1]}};
            // project_backward.wgsl:123-125.
            float A[3][2], dS[3][3], B[2][3], dT[2][3];
            for (int i = 0; i < 3; ++i)
                for (int s = 0; s < 2; ++s) A[i][s] = g.T[0][i] * G[0][s] + g.T[1][i] * G[1][s];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j) dS[i][j] = A[i][0] * g.T[0][j] + A[i][1] * g.T[1][j];
            for (int r = 0; r < 2; ++r)
                for (int j = 0; j < 3; ++j) B[r][j] = G[r][0] * g.T[0][j] + G[r][1] * g.T[1][j];
            for (int r = 0; r < 2; ++r)
                for (int j = 0; j < 3; ++j)
                    dT[r][j] = 2.0f * (B[r][0] * g.Sigma[0][j] + B[r][1] * g.Sigma[1][j] + B[r][2] * g.Sigma[2][j]);
            // project_backward.wgsl:126-127: d_j = d_t * transpose(w).
            float dJ[2][3];
            for (int r = 0; r < 2; ++r)
                for (int k = 0; k < 3; ++k) dJ[r][k] = dT[r][0] * g.W[k][0] + dT[r][1] * g.W[k][1] + dT[r][2] * g.W[k][2];
            // project_backward.wgsl:129-137.
            float d_pc[3] = {0.0f, 0.0f, 0.0f};
            d_pc[0] += g.clamped[0] ? 0.0f : -fx / g.z2 * dJ[0][2];
            d_pc[1] += g.clamped[1] ? 0.0f : -fy / g.z2 * dJ[1][2];
            d_pc[2] += -fx / g.z2 * dJ[0][0] - fy / g.z2 * dJ[1][1] + 2.0f * fx * g.tx / z3 * dJ[0][2] +
                       2.0f * fy * g.ty / z3 * dJ[1][2];
            d_pc[0] += d_mean[0] * fx / pc[2];
            d_pc[1] += d_mean[1] * fy / pc[2];
            d_pc[2] += -d_mean[0] * fx * pc[0] / g.z2 - d_mean[1] * fy * pc[1] / g.z2;
            // project_backward.wgsl:138-141: transpose(w) * d_pc.
            for (int j = 0; j < 3; ++j)
                grads[SP_SLOT_POSITION + j] = g.W[0][j] * d_pc[0] + g.W[1][j] * d_pc[1] + g.W[2][j] * d_pc[2];
            // project_backward.wgsl:145-157: the camera.
            for (int r = 0; r < 3; ++r)
                for (int c = 0; c < 3; ++c) {
                    const float jt_dt = g.J[0][r] * dT[0][c] + g.J[1][r] * dT[1][c];
                    cgrad[r * 3 + c] = d_pc[r] * prm[c] + jt_dt;
                }
            cgrad[9] = d_pc[0];
            cgrad[10] = d_pc[1];
            cgrad[11] = d_pc[2];
            cgrad[12] = d_mean[0] * pc[0] / pc[2] + dJ[0][0] / pc[2] + (g.clamped[0] ? 0.0f : -g.tx / g.z2 * dJ[0][2]);
            cgrad[13] = d_mean[1] * pc[1] / pc[2] + dJ[1][1] / pc[2] + (g.clamped[1] ? 0.0f : -g.ty / g.z2 * dJ[1][2]);
            // The view direction of SH degree >= 1 (no reference counterpart): the
            // position, and the camera centre c = -W^T t, which moves with W and t.
            if (sh_degree > 0) {
                for (int a = 0; a < 3; ++a) grads[SP_SLOT_POSITION + a] += d_position_sh[a];
                const float (*rows)[4] = cam->world_to_camera_rows;
                // dL/dc = -d_position_sh; dL/dt_i = -(W dL/dc)_i; dL/dW_ij = -t_i (dL/dc)_j.
                for (int i = 0; i < 3; ++i) {
                    cgrad[9 + i] += g.W[i][0] * d_position_sh[0] + g.W[i][1] * d_position_sh[1] + g.W[i][2] * d_position_sh[2];
                    for (int j = 0; j < 3; ++j) cgrad[i * 3 + j] += rows[i][3] * d_position_sh[j];
                }
            }
            // project_backward.wgsl:159-165: scales.
            float dM[3][3];
            for (int i = 0; i < 3; ++i)
                for (int k = 0; k < 3; ++k)
                    dM[i][k] = 2.0f * (dS[i][0] * g.M[0][k] + dS[i][1] * g.M[1][k] + dS[i][2] * g.M[2][k]);
            for (int k = 0; k < 3; ++k)
                grads[SP_SLOT_LOG_SCALE + k] =
                    (g.R[0][k] * dM[0][k] + g.R[1][k] * dM[1][k] + g.R[2][k] * dM[2][k]) * g.scale[k];
            // project_backward.wgsl:166-192: the quaternion.
            float dR[3][3];
            for (int i = 0; i < 3; ++i)
                for (int k = 0; k < 3; ++k) dR[i][k] = dM[i][k] * g.scale[k];
            const float r00 = dR[0][0], r01 = dR[0][1], r02 = dR[0][2];
            const float r10 = dR[1][0], r11 = dR[1][1], r12 = dR[1][2];
            const float r20 = dR[2][0], r21 = dR[2][1], r22 = dR[2][2];
            const float qw = g.q[0], qx = g.q[1], qy = g.q[2], qz = g.q[3];
            const float du[4] = {
                2.0f * (qz * (r10 - r01) + qy * (r02 - r20) + qx * (r21 - r12)),
                2.0f * (qy * (r01 + r10) + qz * (r02 + r20) + qw * (r21 - r12)) - 4.0f * qx * (r11 + r22),
                2.0f * (qx * (r01 + r10) + qw * (r02 - r20) + qz * (r12 + r21)) - 4.0f * qy * (r00 + r22),
                2.0f * (qw * (r10 - r01) + qx * (r02 + r20) + qy * (r12 + r21)) - 4.0f * qz * (r00 + r11),
            };
            const float qdu = g.q[0] * du[0] + g.q[1] * du[1] + g.q[2] * du[2] + g.q[3] * du[3];
            for (int k = 0; k < 4; ++k) grads[SP_SLOT_ROTATION + k] = (du[k] - g.q[k] * qdu) / g.q_length;
        }
        // project_backward.wgsl:211-226: tree reduction over the workgroup.
        for (int half = 128; half > 0; half >>= 1)
            for (int t = 0; t < half; ++t)
                for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c)
                    local[(size_t)t * SP_CAMERA_GRAD_STRIDE + c] += local[(size_t)(t + half) * SP_CAMERA_GRAD_STRIDE + c];
        for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) partials[(size_t)group * SP_CAMERA_GRAD_STRIDE + c] = local[c];
    }
    // reduce_camera_gradient.wgsl:10-34.
    std::vector<float> sums(256 * SP_CAMERA_GRAD_STRIDE, 0.0f);
    for (int t = 0; t < 256; ++t)
        for (int64_t i = t; i < groups; i += 256)
            for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c)
                sums[(size_t)t * SP_CAMERA_GRAD_STRIDE + c] += partials[(size_t)i * SP_CAMERA_GRAD_STRIDE + c];
    for (int half = 128; half > 0; half >>= 1)
        for (int t = 0; t < half; ++t)
            for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c)
                sums[(size_t)t * SP_CAMERA_GRAD_STRIDE + c] += sums[(size_t)(t + half) * SP_CAMERA_GRAD_STRIDE + c];
    for (int c = 0; c < SP_CAMERA_GRAD_STRIDE; ++c) camera_gradient[c] = sums[c];
}

void or_learning_rates_by_slot(const sp_learning_rates* rates, float position_scale, uint32_t stride, float* out) {
    for (uint32_t slot = 0; slot < stride; ++slot) {
        float rate;
        if (slot < 3) rate = rates->position * position_scale;
        else if (slot < 6) rate = rates->log_scale;
        else if (slot < 10) rate = rates->rotation;
        else if (slot == 10) rate = rates->opacity;
        else if (slot < 14) rate = rates->sh_dc;
        else rate = rates->sh_rest;
        out[slot] = rate;
    }
}

float or_bias_correction(float beta, uint32_t step) { return 1.0f - std::pow(beta, (float)step); }

void or_adam_step(float* params, const float* gradients, float* m1, float* m2, uint64_t n, uint32_t stride,
                  const float* lr_by_slot, float bias1, float bias2, float max_log_scale,
                  float max_log_anisotropy) {
    const int64_t count = (int64_t)(n * stride);
    // adam.wgsl:20-37.
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t i = 0; i < count; ++i) {
        const float rate = lr_by_slot[i % stride];
        const float g = gradients[i];
        const float m = SP_ADAM_BETA1 * m1[i] + (1.0f - SP_ADAM_BETA1) * g;
        const float v = SP_ADAM_BETA2 * m2[i] + (1.0f - SP_ADAM_BETA2) * g * g;
        m1[i] = m;
        m2[i] = v;
        const float m_hat = m / bias1;
        const float v_hat = v / bias2;
        params[i] -= rate * m_hat / (std::sqrt(v_hat) + SP_ADAM_EPSILON);
    }
    // clamp_scales.wgsl:15-29.
#pragma omp parallel for schedule(static) num_threads(threads())
    for (int64_t g = 0; g < (int64_t)n; ++g) {
        float* ls = params + g * stride + SP_SLOT_LOG_SCALE;
        for (int k = 0; k < 3; ++k) ls[k] = std::min(ls[k], max_log_scale);
        const float smallest = std::min(ls[0], std::min(ls[1], ls[2]));
        for (int k = 0; k < 3; ++k) ls[k] = std::min(ls[k], smallest + max_log_anisotropy);
    }
}

double or_train_step(float* params, uint64_t n, uint32_t sh_degree, const sp_camera_uniform* cam,
                     const float* gt, float* m1, float* m2, const float* lr_by_slot, uint32_t step,
                     float max_log_scale, float max_log_anisotropy, uint64_t* count_out) {
    const uint32_t stride = stride_of(sh_degree);
    const uint64_t capacity = n * SP_INTERSECTIONS_PER_GAUSSIAN;
    const uint64_t pixels = (uint64_t)cam->width * cam->height;
    const uint64_t tiles = (uint64_t)cam->tiles_x * cam->tiles_y;
    std::vector<sp_projected> proj(n);
    std::vector<uint32_t> counts(n), offsets(n);
    or_project(params, n, sh_degree, cam, proj.data(), counts.data());
    sp_intersection_meta meta;
    const uint64_t total = or_scan(counts.data(), n, capacity, offsets.data(), &meta);
    const uint64_t count = std::min(total, capacity);
    std::vector<uint64_t> keys(count);
    std::vector<uint32_t> gauss(count), slots(count), ranges(tiles * 2);
    const int key_mode = SP_KEYS_REF20;
    or_bin(proj.data(), offsets.data(), n, cam, capacity, key_mode, keys.data(), gauss.data(), slots.data(),
           ranges.data());
    std::vector<float> image(pixels * 4), partials(pixels * 12), loss_gradient(pixels * 4), pixel_loss(pixels * 4);
    std::vector<uint32_t> contributions(pixels);
    or_blend_forward(proj.data(), gauss.data(), ranges.data(), cam, image.data(), contributions.data());
    or_ssim(image.data(), gt, cam->width, cam->height, partials.data());
    const sp_loss_weights weights = {SP_LOSS_L1, SP_LOSS_DSSIM, SP_LOSS_ALPHA};
    or_loss(image.data(), gt, partials.data(), cam->width, cam->height, &weights, loss_gradient.data(),
            pixel_loss.data());
    std::vector<float> slot_gradients(std::max<uint64_t>(count, 1) * SP_GRAD_STRIDE, 0.0f);
    or_blend_backward(proj.data(), gauss.data(), slots.data(), ranges.data(), cam, image.data(),
                      contributions.data(), loss_gradient.data(), slot_gradients.data());
    std::vector<float> param_gradients(n * stride);
    float camera_gradient[SP_CAMERA_GRAD_STRIDE];
    std::vector<sp_densify_stats> stats(n);
    std::memset(stats.data(), 0, n * sizeof(sp_densify_stats));
    or_project_backward(params, n, sh_degree, cam, proj.data(), offsets.data(), slot_gradients.data(), count,
                        param_gradients.data(), camera_gradient, stats.data());
    or_adam_step(params, param_gradients.data(), m1, m2, n, stride, lr_by_slot,
                 or_bias_correction(SP_ADAM_BETA1, step), or_bias_correction(SP_ADAM_BETA2, step), max_log_scale,
                 max_log_anisotropy);
    double loss = 0.0;
    for (uint64_t i = 0; i < pixels; ++i) loss += pixel_loss[i * 4 + 3];
    if (count_out) *count_out = count;
    return loss / (double)pixels;
}

// ---------------------------------------------------------------------------- densify

uint64_t or_splitmix64(uint64_t seed, uint64_t index) {
    // densify.rs:279-285: state += 0x9e3779b97f4a7c15, then the finaliser; the (index + 1)-th
    // call's state is seed + (index + 1) * increment.
    uint64_t z = seed + (index + 1) * 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

uint32_t or_total_order_key(float value) {
    // f32::total_cmp as an unsigned key: negative values bit-inverted, the others with the
    // sign bit set.
    uint32_t bits;
    std::memcpy(&bits, &value, 4);
    return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

namespace {

// SplitMix64::uniform (densify.rs:287-290): (0, 1].
float densify_uniform(uint64_t draw) { return ((float)(draw >> 40) + 1.0f) / (float)(1ull << 24); }

// split_child (densify.rs:259-273) with the draws starting at `index` of the stream.
void split_child(const float* gaussian, uint32_t stride, uint64_t seed, uint64_t index, float* child) {
    float local[3];
    for (int k = 0; k < 3; ++k) {
        const float scale = std::exp(gaussian[3 + k]);
        // SplitMix64::standard_normal (densify.rs:292-296), Box-Muller.
        const float u = densify_uniform(or_splitmix64(seed, index + 2 * k));
        const float v = densify_uniform(or_splitmix64(seed, index + 2 * k + 1));
        const float normal = std::sqrt(-2.0f * std::log(u)) * std::cos(6.28318530717958647692f * v);
        local[k] = scale * normal;
    }
    // nalgebra 0.34 (Cargo.lock): UnitQuaternion::from_quaternion(Quaternion::new(w, x, y, z))
    // divides by the norm of the coordinates stored as (x, y, z, w), whose 4-vector dot product
    // sums (x^2 + z^2) + (y^2 + w^2); the rotation of a vector v is t w + q x t + v with
    // t = 2 (q x v).
    const float w0 = gaussian[6], x0 = gaussian[7], y0 = gaussian[8], z0 = gaussian[9];
    const float norm = std::sqrt((x0 * x0 + z0 * z0) + (y0 * y0 + w0 * w0));
    const float w = w0 / norm, qx = x0 / norm, qy = y0 / norm, qz = z0 / norm;
    const float t[3] = {2.0f * (qy * local[2] - qz * local[1]), 2.0f * (qz * local[0] - qx * local[2]),
                        2.0f * (qx * local[1] - qy * local[0])};
    const float c[3] = {qy * t[2] - qz * t[1], qz * t[0] - qx * t[2], qx * t[1] - qy * t[0]};
    std::memcpy(child, gaussian, stride * sizeof(float));
    const float log_divisor = std::log(1.6f);
    for (int k = 0; k < 3; ++k) {
        child[k] += t[k] * w + c[k] + local[k];
        child[3 + k] -= log_divisor;
    }
}

}  // namespace

int or_densify(const float* params, const float* first_moment, const float* second_moment,
               const sp_densify_stats* stats, uint64_t n, uint32_t stride, float extent, uint64_t max_count,
               const sp_densify_settings* settings, int reset_opacity, uint64_t seed, float* out_params,
               float* out_first, float* out_second, uint64_t out_capacity, sp_densify_report* report) {
    // densify.rs:147-257.
    enum Fate : uint8_t { Kept, Cloned, Split, PrunedTransparent, PrunedOversized };
    const float split_log_scale = std::log(settings->split_scale_fraction * extent);
    std::vector<uint8_t> fate(n);
    for (uint64_t g = 0; g < n; ++g) {
        // gaussians.rs:87-89 with the host libm's exp.
        const float logit = params[g * stride + SP_SLOT_OPACITY];
        if (1.0f / (1.0f + std::exp(-logit)) < settings->prune_opacity)
            fate[g] = PrunedTransparent;
        else if (stats[g].max_radius >= settings->max_screen_radius)
            fate[g] = PrunedOversized;
        else
            fate[g] = Kept;
    }
    auto mean_gradient = [&](uint64_t g) {
        return stats[g].visible_count > 0.0f ? stats[g].mean_gradient_sum / stats[g].visible_count : 0.0f;
    };
    std::vector<uint64_t> candidates;
    for (uint64_t g = 0; g < n; ++g)
        if (fate[g] == Kept && mean_gradient(g) > settings->gradient_threshold) candidates.push_back(g);
    // sort_by(|a, b| mean_gradient(b).total_cmp(&mean_gradient(a))), a stable sort.
    std::stable_sort(candidates.begin(), candidates.end(), [&](uint64_t a, uint64_t b) {
        return or_total_order_key(mean_gradient(b)) < or_total_order_key(mean_gradient(a));
    });
    uint64_t kept = 0;
    for (uint64_t g = 0; g < n; ++g) kept += fate[g] == Kept;
    const uint64_t budget = std::min<uint64_t>(max_count > kept ? max_count - kept : 0, candidates.size());
    for (uint64_t c = 0; c < budget; ++c) {
        const uint64_t g = candidates[c];
        float largest = -INFINITY;
        for (int k = 0; k < 3; ++k) largest = std::fmax(largest, params[g * stride + 3 + k]);  // f32::max
        fate[g] = largest > split_log_scale ? Split : Cloned;
    }
    sp_densify_report r{};
    r.before = n;
    r.over_budget = candidates.size() - budget;
    for (uint64_t g = 0; g < n; ++g) {
        r.cloned += fate[g] == Cloned;
        r.split += fate[g] == Split;
        r.pruned_transparent += fate[g] == PrunedTransparent;
        r.pruned_oversized += fate[g] == PrunedOversized;
    }
    const uint64_t copies = kept - r.split;  // kept and cloned Gaussians keep their place
    r.after = copies + r.cloned + 2 * r.split;
    r.opacity_reset = reset_opacity ? 1u : 0u;
    *report = r;
    if (r.after == 0) return 1;
    if (out_capacity < r.after) return 2;
    uint64_t o = 0, made = copies, splits = 0;
    std::vector<float> child(stride);
    for (uint64_t g = 0; g < n; ++g) {
        const float* gaussian = params + g * stride;
        if (fate[g] == Kept || fate[g] == Cloned) {
            std::memcpy(out_params + o * stride, gaussian, stride * sizeof(float));
            std::memcpy(out_first + o * stride, first_moment + g * stride, stride * sizeof(float));
            std::memcpy(out_second + o * stride, second_moment + g * stride, stride * sizeof(float));
            ++o;
        }
    }
    // The new Gaussians after the kept ones, in index order: a clone's copy or a split's two
    // children, with zero moments.
    for (uint64_t g = 0; g < n; ++g) {
        const float* gaussian = params + g * stride;
        if (fate[g] == Cloned) {
            std::memcpy(out_params + made * stride, gaussian, stride * sizeof(float));
            ++made;
        } else if (fate[g] == Split) {
            for (int c = 0; c < 2; ++c) {
                split_child(gaussian, stride, seed, splits * 12 + c * 6, out_params + made * stride);
                ++made;
            }
            ++splits;
        }
    }
    std::memset(out_first + copies * stride, 0, (r.after - copies) * stride * sizeof(float));
    std::memset(out_second + copies * stride, 0, (r.after - copies) * stride * sizeof(float));
    if (reset_opacity) {
        const float reset_logit = std::log(0.01f / (1.0f - 0.01f));  // logit(RESET_OPACITY)
        for (uint64_t g = 0; g < r.after; ++g) {
            float& slot = out_params[g * stride + SP_SLOT_OPACITY];
            slot = std::fmin(slot, reset_logit);  // f32::min
            out_first[g * stride + SP_SLOT_OPACITY] = 0.0f;
            out_second[g * stride + SP_SLOT_OPACITY] = 0.0f;
        }
    }
    return 0;
}

}  // extern "C"
