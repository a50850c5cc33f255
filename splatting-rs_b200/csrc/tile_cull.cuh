// Tile culling by the Gaussian's ellipse (sp_options.tile_culling = 1): of the tiles of a
// Gaussian's bounding rectangle (project_forward.wgsl:76-83, the reference emits all of them),
// only those where its alpha can reach 1/255 at a pixel centre get a key. The others would be
// skipped at every pixel by the blend's own test (rasterize_forward.wgsl:60-62), so images,
// contributions to the loss and gradients are unchanged; the intersection lists are shorter.
//
// "Can reach" is the blend kernels' conservative test: inside the ellipse d^T C d <= q of the
// conic C, q = 2.02 ln(255 opacity) + 0.02 (1 % above the exact level), and within 0.05 px of
// the tile's rectangle of pixel centres. Per tile row the ellipse's x-extent over the row's
// band is exact: its right end is the concave x_max(y) = (-b y + sqrt(a q - det y^2)) / a at
// its stationary point y = -b sqrt(q / (det c)) clamped to the band, the left end likewise.
// The hardware's approximate sqrt, reciprocal and log2 (relative errors near 2^-22) are far
// inside that padding.
//
// The projection counts the tiles (for the tile offsets) and the emission enumerates them with
// these same functions; every operation is an explicit instruction (rounded multiplies and
// adds, PTX approximations), so both translation units, one of them built with -fmad=false,
// get the same spans.
#pragma once

#include "common.cuh"

namespace splat {
namespace cull {

__device__ __forceinline__ float sqrt_approx(float x) {
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float lg2_approx(float x) {
    float r;
    asm("lg2.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

}  // namespace cull

// A Gaussian's culling ellipse, relative to its mean: a x^2 + 2 b x y + c y^2 <= q.
struct CullEllipse {
    float mx, my;        // mean
    float b, inv_a;      // conic b, 1 / a
    float qa, det;       // a q, a c - b^2 (half width at height y: sqrt(a q - det y^2) / a)
    float ey;            // vertical half extent; < 0: reaches no pixel; inf: keep every tile
    float stationary;    // b sqrt(q / (det c)): x_max peaks at -stationary, x_min bottoms at +stationary
};

// The ellipse of record (a, b): mean = (a.x, a.y), conic = (a.z, a.w, b.x), opacity = b.y.
__device__ __forceinline__ CullEllipse cull_ellipse(float4 a, float4 b) {
    CullEllipse e;
    e.mx = a.x;
    e.my = a.y;
    e.b = a.w;
    e.inv_a = 0.0f;
    e.qa = 0.0f;
    e.det = 0.0f;
    e.stationary = 0.0f;
    const float level = __fmul_rn(b.y, 255.0f);
    if (!(level > 1.0f)) {  // alpha below 1/255 everywhere
        e.ey = -1.0f;
        return e;
    }
    const float ca = a.z, cb = a.w, cc = b.x;
    const float det = __fsub_rn(__fmul_rn(ca, cc), __fmul_rn(cb, cb));
    if (!(det > 0.0f) || !(ca > 0.0f) || !(cc > 0.0f)) {  // degenerate conic: never culled
        e.ey = INFINITY;
        return e;
    }
    // q = 2.02 ln(level) + 0.02 = 2.02 ln(2) log2(level) + 0.02.
    const float q = __fadd_rn(__fmul_rn(1.40015730f, cull::lg2_approx(level)), 0.02f);
    const float inv_det = cull::rcp_approx(det);
    e.inv_a = cull::rcp_approx(ca);
    e.qa = __fmul_rn(q, ca);
    e.det = det;
    e.ey = cull::sqrt_approx(__fmul_rn(e.qa, inv_det));
    e.stationary = __fmul_rn(cb, cull::sqrt_approx(__fmul_rn(__fmul_rn(q, inv_det), cull::rcp_approx(cc))));
    return e;
}

// The ellipse's x-extent [left, right] (relative to its mean) over the band of pixel-centre
// rows [first_row, first_row + rows - 1], padded by 0.05 px; false when the band misses it.
// The ellipse must be neither culled (ey >= 0) nor degenerate (ey finite).
__device__ __forceinline__ bool band_extent(const CullEllipse& e, uint32_t first_row, uint32_t rows, float& left,
                                            float& right) {
    const float lo = __fsub_rn(__fsub_rn((float)first_row, e.my), 0.05f);
    const float hi = __fadd_rn(lo, (float)(rows - 1) + 0.1f);
    const float y0 = fmaxf(lo, -e.ey), y1 = fminf(hi, e.ey);
    if (!(y0 <= y1)) return false;
    const float yr = fminf(fmaxf(-e.stationary, y0), y1);  // where x_max peaks
    const float yl = fminf(fmaxf(e.stationary, y0), y1);   // where x_min bottoms
    const float wr = cull::sqrt_approx(fmaxf(0.0f, __fsub_rn(e.qa, __fmul_rn(e.det, __fmul_rn(yr, yr)))));
    const float wl = cull::sqrt_approx(fmaxf(0.0f, __fsub_rn(e.qa, __fmul_rn(e.det, __fmul_rn(yl, yl)))));
    right = __fmul_rn(__fsub_rn(wr, __fmul_rn(e.b, yr)), e.inv_a);
    left = __fmul_rn(__fadd_rn(wl, __fmul_rn(e.b, yl)), -e.inv_a);
    return true;
}

// Which of the two 8-pixel halves of tile column `column` (bit 0: x offset 0, bit 1: offset 8)
// have a pixel centre within 0.05 px of the absolute x-extent [left, right].
__device__ __forceinline__ uint32_t half_columns(float left, float right, uint32_t column) {
    const float x = (float)(column * SP_TILE);
    uint32_t bits = 0;
    if (left <= __fadd_rn(x, 7.05f) && right >= __fsub_rn(x, 0.05f)) bits |= 1u;
    if (left <= __fadd_rn(x, 15.05f) && right >= __fadd_rn(x, 7.95f)) bits |= 2u;
    return bits;
}

// The columns [first, end) of tile row `row` the ellipse reaches, within the rectangle's
// columns [x0, x1).
__device__ __forceinline__ uint2 tile_row_span(const CullEllipse& e, uint32_t row, uint32_t x0, uint32_t x1) {
    if (!(e.ey >= 0.0f)) return make_uint2(x0, x0);
    if (!(e.ey < INFINITY)) return make_uint2(x0, x1);
    // The row's band of pixel centres, padded by 0.05 px, clamped to the ellipse's extent.
    float left, right;
    if (!band_extent(e, row * SP_TILE, SP_TILE, left, right)) return make_uint2(x0, x0);
    // Columns whose pixel centres [16 t, 16 t + 15] come within 0.05 px of [left, right]
    // (1 / 16 is exact).
    constexpr float kInvTile = 1.0f / (float)SP_TILE;
    const float first = ceilf(__fmul_rn(__fsub_rn(__fadd_rn(left, e.mx), (float)(SP_TILE - 1) + 0.05f), kInvTile));
    const float last = floorf(__fmul_rn(__fadd_rn(__fadd_rn(right, e.mx), 0.05f), kInvTile));
    const float c0 = fmaxf(first, (float)x0), c1 = fminf(__fadd_rn(last, 1.0f), (float)x1);
    if (!(c0 < c1)) return make_uint2(x0, x0);
    return make_uint2((uint32_t)c0, (uint32_t)c1);
}

// The number of tiles of the rectangle [x0, x1) x [y0, y1) the ellipse reaches.
__device__ __forceinline__ uint32_t culled_tile_count(const CullEllipse& e, uint32_t x0, uint32_t y0, uint32_t x1,
                                                      uint32_t y1) {
    if (!(e.ey >= 0.0f)) return 0u;
    uint32_t count = 0;
    for (uint32_t row = y0; row < y1; ++row) {
        const uint2 span = tile_row_span(e, row, x0, x1);
        count += span.y - span.x;
    }
    return count;
}

// Whether the ellipse a x^2 + 2 b x y + c y^2 <= q meets the rectangle [x0, x1] x [y0, y1]
// (coordinates relative to its centre), with kx = -b/c and ky = -b/a precomputed: as
// ellipse_meets_rect, the minima along the edges at the clamped stationary points.
__device__ __forceinline__ bool ellipse_meets_rect_k(float a, float b, float c, float kx, float ky, float q, float x0,
                                                     float x1, float y0, float y1) {
    if (x0 <= 0.0f && x1 >= 0.0f && y0 <= 0.0f && y1 >= 0.0f) return true;
    float best = INFINITY;
    const float xs[2] = {x0, x1}, ys[2] = {y0, y1};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float x = xs[e];
        const float y = fminf(fmaxf(kx * x, y0), y1);
        best = fminf(best, a * x * x + 2.0f * b * x * y + c * y * y);
        const float yy = ys[e];
        const float xx = fminf(fmaxf(ky * yy, x0), x1);
        best = fminf(best, a * xx * xx + 2.0f * b * xx * yy + c * yy * yy);
    }
    return best <= q;
}

// Whether a Gaussian can reach the rectangle of pixel centres [x0, x0 + 7] x [y0, y0 + ROWS - 1]:
// op * exp(power) >= 1/255 somewhere in it, i.e. the ellipse d^T C d <= 2 ln(255 op) of the
// conic C (padded by 1 % in the level) meets the rectangle (padded by 0.05 px). `r` holds the
// projection's constants of the Gaussian (its half extents and slopes, reach_of in
// project.cu); a bounding-box test first, then the exact one.
template <int ROWS>
__device__ __forceinline__ bool reaches(float4 a, float4 b, float4 r, float x0, float y0) {
    if (!(r.x >= 0.0f)) return false;        // the opacity keeps alpha below 1/255
    if (!(r.x < INFINITY)) return true;      // degenerate conic: never culled
    const float lo_x = x0 - a.x - 0.05f, hi_x = lo_x + 7.1f;
    const float lo_y = y0 - a.y - 0.05f, hi_y = lo_y + (float)(ROWS - 1) + 0.1f;
    if (r.x < lo_x || -r.x > hi_x || r.y < lo_y || -r.y > hi_y) return false;
    const float q = 2.02f * __logf(b.y * 255.0f) + 0.02f;
    return ellipse_meets_rect_k(a.z, a.w, b.x, r.z, r.w, q, lo_x, hi_x, lo_y, hi_y);
}

// Which of tile (tx, ty)'s four 8 x 8 pixel blocks a Gaussian can reach (bit w: the block at
// x offset 8 (w & 1), y offset 8 (w >> 1)), by `reaches` with the blend kernels' warp layout.
__device__ __forceinline__ uint32_t block_mask(float4 a, float4 b, float4 r, uint32_t tx, uint32_t ty) {
    uint32_t mask = 0;
#pragma unroll
    for (uint32_t w = 0; w < 4; ++w)
        if (reaches<8>(a, b, r, (float)(tx * SP_TILE + ((w & 1u) << 3)), (float)(ty * SP_TILE + ((w >> 1) << 3))))
            mask |= 1u << w;
    return mask;
}

}  // namespace splat
