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
//
// The projection counts the tiles (for the tile offsets) and the emission enumerates them
// with this same function; every operation has an explicit rounding, so both translation units
// (one built with -fmad=false) get the same spans.
#pragma once

#include "common.cuh"

namespace splat {

// The columns [first, end) of tile row `row` that the Gaussian of record (a, b) reaches,
// within its rectangle's columns [x0, x1). mean = (a.x, a.y), conic = (a.z, a.w, b.x),
// opacity = b.y.
__device__ __forceinline__ uint2 tile_row_span(float4 a, float4 b, uint32_t row, uint32_t x0, uint32_t x1) {
    const float level = __fmul_rn(b.y, 255.0f);
    if (!(level > 1.0f)) return make_uint2(x0, x0);  // alpha below 1/255 everywhere
    const float ca = a.z, cb = a.w, cc = b.x;
    const float det = __fsub_rn(__fmul_rn(ca, cc), __fmul_rn(cb, cb));
    if (!(det > 0.0f) || !(ca > 0.0f) || !(cc > 0.0f)) return make_uint2(x0, x1);  // degenerate: keep all
    const float q = __fadd_rn(__fmul_rn(2.02f, __logf(level)), 0.02f);
    // The ellipse's vertical half extent, and the row's band of pixel centres (padded).
    const float ey = __fsqrt_rn(__fdiv_rn(__fmul_rn(q, ca), det));
    const float lo = __fsub_rn(__fsub_rn((float)(row * SP_TILE), a.y), 0.05f);
    const float hi = __fadd_rn(lo, (float)(SP_TILE - 1) + 0.1f);
    const float y0 = fmaxf(lo, -ey), y1 = fminf(hi, ey);
    if (!(y0 <= y1)) return make_uint2(x0, x0);
    const float stationary = __fmul_rn(cb, __fsqrt_rn(__fdiv_rn(q, __fmul_rn(det, cc))));
    auto half_width = [&](float y) {
        return __fsqrt_rn(fmaxf(0.0f, __fsub_rn(__fmul_rn(ca, q), __fmul_rn(det, __fmul_rn(y, y)))));
    };
    const float yr = fminf(fmaxf(-stationary, y0), y1);  // where x_max peaks
    const float yl = fminf(fmaxf(stationary, y0), y1);   // where x_min bottoms
    const float right = __fdiv_rn(__fadd_rn(-__fmul_rn(cb, yr), half_width(yr)), ca);
    const float left = __fdiv_rn(__fsub_rn(-__fmul_rn(cb, yl), half_width(yl)), ca);
    // Columns whose pixel centres [16 t, 16 t + 15] come within 0.05 px of [left, right].
    const float first = ceilf(__fdiv_rn(__fsub_rn(__fadd_rn(left, a.x), (float)(SP_TILE - 1) + 0.05f), (float)SP_TILE));
    const float last = floorf(__fdiv_rn(__fadd_rn(__fadd_rn(right, a.x), 0.05f), (float)SP_TILE));
    const float c0 = fmaxf(first, (float)x0), c1 = fminf(last + 1.0f, (float)x1);
    if (!(c0 < c1)) return make_uint2(x0, x0);
    return make_uint2((uint32_t)c0, (uint32_t)c1);
}

// The number of tiles of the rectangle [x0, x1) x [y0, y1) the Gaussian reaches.
__device__ __forceinline__ uint32_t culled_tile_count(float4 a, float4 b, uint32_t x0, uint32_t y0, uint32_t x1,
                                                      uint32_t y1) {
    uint32_t count = 0;
    for (uint32_t row = y0; row < y1; ++row) {
        const uint2 span = tile_row_span(a, b, row, x0, x1);
        count += span.y - span.x;
    }
    return count;
}

}  // namespace splat
