// Per-Gaussian projection math of project_forward.wgsl:43-86 and project_backward.wgsl:65-97,
// written for one CUDA thread. The operation order is the one the CPU oracle
// (oracle/splat_oracle.cpp, `geometry` and `project_one`) uses, and the file that includes
// this header is compiled with -fmad=false, so the depth, radius and tile rectangle come
// out bit-identical to the oracle's: the tile lists are compared bit for bit.
//
// Matrices are row-major: X[i][j] is row i, column j (WGSL's are column-major).
#pragma once

#include "common.cuh"
#include "exact_div.cuh"

namespace splat {

// std::max / std::min semantics, so that signed zeros resolve as in the oracle.
__device__ __forceinline__ float max_of(float a, float b) { return (a < b) ? b : a; }
__device__ __forceinline__ float min_of(float a, float b) { return (b < a) ? b : a; }

__device__ __forceinline__ float row_dot(const float r[4], float x, float y, float z) {
    return r[0] * x + r[1] * y + r[2] * z + r[3] * 1.0f;
}

// u / d, the IEEE quotient either way: NEWTON takes div_rn (a double-precision reciprocal,
// fewer instructions where the divisor is in its domain: the backward), otherwise the
// compiler's division (the forward, where div_rn measured slower).
template <bool NEWTON>
__device__ __forceinline__ float quotient(float u, float d) {
    if constexpr (NEWTON) return div_rn(u, d);
    else return u / d;
}

struct Geometry {
    float pc[3];
    float scale[3];
    float q[4];
    float q_length;
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

// quaternion_to_matrix (common.wgsl:92-103).
__device__ __forceinline__ void rotation_of(float r, float x, float y, float z, float R[3][3]) {
    R[0][0] = 1.0f - 2.0f * (y * y + z * z);
    R[1][0] = 2.0f * (x * y + r * z);
    R[2][0] = 2.0f * (x * z - r * y);
    R[0][1] = 2.0f * (x * y - r * z);
    R[1][1] = 1.0f - 2.0f * (x * x + z * z);
    R[2][1] = 2.0f * (y * z + r * x);
    R[0][2] = 2.0f * (x * z + r * y);
    R[1][2] = 2.0f * (y * z - r * x);
    R[2][2] = 1.0f - 2.0f * (x * x + y * y);
}

template <bool NEWTON = false>
__device__ __forceinline__ void geometry(const float* p, const sp_camera_uniform& cam, Geometry& g) {
    const float (*rows)[4] = cam.world_to_camera_rows;
    g.pc[0] = row_dot(rows[0], p[0], p[1], p[2]);
    g.pc[1] = row_dot(rows[1], p[0], p[1], p[2]);
    g.pc[2] = row_dot(rows[2], p[0], p[1], p[2]);
#pragma unroll
    for (int k = 0; k < 3; ++k) g.scale[k] = sp_expf(p[SP_SLOT_LOG_SCALE + k]);
    const float* qr = p + SP_SLOT_ROTATION;
    g.q_length = __fsqrt_rn(qr[0] * qr[0] + qr[1] * qr[1] + qr[2] * qr[2] + qr[3] * qr[3]);
#pragma unroll
    for (int k = 0; k < 4; ++k) g.q[k] = quotient<NEWTON>(qr[k], g.q_length);
    rotation_of(g.q[0], g.q[1], g.q[2], g.q[3], g.R);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k) g.M[i][k] = g.R[i][k] * g.scale[k];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            g.Sigma[i][j] = g.M[i][0] * g.M[j][0] + g.M[i][1] * g.M[j][1] + g.M[i][2] * g.M[j][2];
    const float fx = cam.focal[0], fy = cam.focal[1];
    g.limit[0] = quotient<NEWTON>(SP_VIEW_LIMIT_FACTOR * (float)cam.width, 2.0f * fx);
    g.limit[1] = quotient<NEWTON>(SP_VIEW_LIMIT_FACTOR * (float)cam.height, 2.0f * fy);
    const float xz = quotient<NEWTON>(g.pc[0], g.pc[2]);
    const float yz = quotient<NEWTON>(g.pc[1], g.pc[2]);
    g.clamped[0] = fabsf(xz) > g.limit[0];
    g.clamped[1] = fabsf(yz) > g.limit[1];
    g.tx = min_of(max_of(xz, -g.limit[0]), g.limit[0]) * g.pc[2];
    g.ty = min_of(max_of(yz, -g.limit[1]), g.limit[1]) * g.pc[2];
    g.z2 = g.pc[2] * g.pc[2];
    g.J[0][0] = quotient<NEWTON>(fx, g.pc[2]);
    g.J[0][1] = 0.0f;
    g.J[0][2] = quotient<NEWTON>(-fx * g.tx, g.z2);
    g.J[1][0] = 0.0f;
    g.J[1][1] = quotient<NEWTON>(fy, g.pc[2]);
    g.J[1][2] = quotient<NEWTON>(-fy * g.ty, g.z2);
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int j = 0; j < 3; ++j) g.W[k][j] = rows[k][j];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            g.T[r][j] = g.J[r][0] * g.W[0][j] + g.J[r][1] * g.W[1][j] + g.J[r][2] * g.W[2][j];
    float TS[2][3];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            TS[r][j] = g.T[r][0] * g.Sigma[0][j] + g.T[r][1] * g.Sigma[1][j] + g.T[r][2] * g.Sigma[2][j];
    float cov[2][2];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int s = 0; s < 2; ++s) cov[r][s] = TS[r][0] * g.T[s][0] + TS[r][1] * g.T[s][1] + TS[r][2] * g.T[s][2];
    g.a = cov[0][0] + SP_COVARIANCE_BLUR;
    g.b = cov[0][1];
    g.c = cov[1][1] + SP_COVARIANCE_BLUR;
    g.det = g.a * g.c - g.b * g.b;
}

// Camera centre -W^T t and the unit direction from it to `pos` (SH degree >= 1).
template <bool NEWTON = false>
__device__ __forceinline__ void view_direction(const sp_camera_uniform& cam, const float* pos, float dir[3],
                                               float* length) {
    const float (*r)[4] = cam.world_to_camera_rows;
    float c[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) c[j] = -(r[0][j] * r[0][3] + r[1][j] * r[1][3] + r[2][j] * r[2][3]);
    const float v[3] = {pos[0] - c[0], pos[1] - c[1], pos[2] - c[2]};
    const float len = __fsqrt_rn(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    dir[0] = quotient<NEWTON>(v[0], len);
    dir[1] = quotient<NEWTON>(v[1], len);
    dir[2] = quotient<NEWTON>(v[2], len);
    *length = len;
}

template <int DEG>
__device__ __forceinline__ void sh_basis(float x, float y, float z, float* b) {
    b[0] = SP_SH_C0;
    if (DEG < 1) return;
    b[1] = -SP_SH_C1 * y;
    b[2] = SP_SH_C1 * z;
    b[3] = -SP_SH_C1 * x;
    if (DEG < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
    b[4] = SP_SH_C2_0 * xy;
    b[5] = SP_SH_C2_1 * yz;
    b[6] = SP_SH_C2_2 * (2.0f * zz - xx - yy);
    b[7] = SP_SH_C2_3 * xz;
    b[8] = SP_SH_C2_4 * (xx - yy);
    if (DEG < 3) return;
    b[9] = SP_SH_C3_0 * y * (3.0f * xx - yy);
    b[10] = SP_SH_C3_1 * xy * z;
    b[11] = SP_SH_C3_2 * y * (4.0f * zz - xx - yy);
    b[12] = SP_SH_C3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    b[13] = SP_SH_C3_4 * x * (4.0f * zz - xx - yy);
    b[14] = SP_SH_C3_5 * z * (xx - yy);
    b[15] = SP_SH_C3_6 * x * (xx - 3.0f * yy);
}

// d basis_k / d(x, y, z) for one k (the rows of sh_basis_gradient), so that a caller
// looping over k need not hold the whole table.
template <int DEG>
__device__ __forceinline__ void sh_basis_gradient_of(int k, float x, float y, float z, float g[3]) {
    g[0] = g[1] = g[2] = 0.0f;
    const float xx = x * x, yy = y * y, zz = z * z;
    switch (k) {
        case 1: g[1] = -SP_SH_C1; break;
        case 2: g[2] = SP_SH_C1; break;
        case 3: g[0] = -SP_SH_C1; break;
        case 4: g[0] = SP_SH_C2_0 * y; g[1] = SP_SH_C2_0 * x; break;
        case 5: g[1] = SP_SH_C2_1 * z; g[2] = SP_SH_C2_1 * y; break;
        case 6: g[0] = -2.0f * SP_SH_C2_2 * x; g[1] = -2.0f * SP_SH_C2_2 * y; g[2] = 4.0f * SP_SH_C2_2 * z; break;
        case 7: g[0] = SP_SH_C2_3 * z; g[2] = SP_SH_C2_3 * x; break;
        case 8: g[0] = 2.0f * SP_SH_C2_4 * x; g[1] = -2.0f * SP_SH_C2_4 * y; break;
        case 9: g[0] = SP_SH_C3_0 * 6.0f * x * y; g[1] = SP_SH_C3_0 * (3.0f * xx - 3.0f * yy); break;
        case 10: g[0] = SP_SH_C3_1 * y * z; g[1] = SP_SH_C3_1 * x * z; g[2] = SP_SH_C3_1 * x * y; break;
        case 11:
            g[0] = SP_SH_C3_2 * -2.0f * x * y;
            g[1] = SP_SH_C3_2 * (4.0f * zz - xx - 3.0f * yy);
            g[2] = SP_SH_C3_2 * 8.0f * y * z;
            break;
        case 12:
            g[0] = SP_SH_C3_3 * -6.0f * x * z;
            g[1] = SP_SH_C3_3 * -6.0f * y * z;
            g[2] = SP_SH_C3_3 * (6.0f * zz - 3.0f * xx - 3.0f * yy);
            break;
        case 13:
            g[0] = SP_SH_C3_4 * (4.0f * zz - 3.0f * xx - yy);
            g[1] = SP_SH_C3_4 * -2.0f * x * y;
            g[2] = SP_SH_C3_4 * 8.0f * x * z;
            break;
        case 14: g[0] = SP_SH_C3_5 * 2.0f * x * z; g[1] = SP_SH_C3_5 * -2.0f * y * z; g[2] = SP_SH_C3_5 * (xx - yy); break;
        case 15: g[0] = SP_SH_C3_6 * (3.0f * xx - 3.0f * yy); g[1] = SP_SH_C3_6 * -6.0f * x * y; break;
        default: break;
    }
}

// Colour before the clamp at zero (project_forward.wgsl:83-86 at degree 0): `params` holds
// at least the position, `sh` the SH coefficients.
template <int DEG>
__device__ __forceinline__ void raw_color(const float* params, const float* sh, const sp_camera_uniform& cam,
                                          float out[3]) {
    if (DEG == 0) {
#pragma unroll
        for (int c = 0; c < 3; ++c) out[c] = SP_SH_C0 * sh[c] + 0.5f;
        return;
    }
    float dir[3], len;
    view_direction(cam, params, dir, &len);
    float b[16];
    sh_basis<DEG>(dir[0], dir[1], dir[2], b);
    constexpr int kCount = (DEG + 1) * (DEG + 1);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        float s = b[0] * sh[c];
#pragma unroll
        for (int k = 1; k < kCount; ++k) s = s + b[k] * sh[3 * k + c];
        out[c] = s + 0.5f;
    }
}

}  // namespace splat
