// Tile-rectangle arithmetic shared by the 2D projection and binning kernels.
//
// A primitive centred at pixel `center` with pixel radius `radius` covers the
// tiles [x0, x1) x [y0, y1): the centre and radius are divided by the 16-pixel
// tile size, truncated toward zero and clamped to the tile grid
// (reference gsplat/cuda/csrc/helpers.cuh:11-43).
#pragma once

namespace hx {

struct TileRect {
    unsigned x0, y0, x1, y1;
};

__device__ __forceinline__ unsigned clamp_tile(float v, int bound) {
    int t = (int)v;
    t = t < 0 ? 0 : t;
    return (unsigned)(t < bound ? t : bound);
}

__device__ __forceinline__ TileRect tile_rect(float2 center, float radius, int tiles_x,
                                              int tiles_y) {
    const float cx = center.x / 16.f;
    const float cy = center.y / 16.f;
    const float rx = radius / 16.f;
    const float ry = radius / 16.f;
    TileRect r;
    r.x0 = clamp_tile(cx - rx, tiles_x);
    r.x1 = clamp_tile(cx + rx + 1, tiles_x);
    r.y0 = clamp_tile(cy - ry, tiles_y);
    r.y1 = clamp_tile(cy + ry + 1, tiles_y);
    return r;
}

}  // namespace hx
