// Per-pixel math of the 3D hexel compositing kernels (forward and backward),
// restating gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:260-371,1030-1067.
#pragma once

#include "hx_hexels3d.cuh"

namespace hx {

// Per-surfel record staged in shared memory by the compositing kernels
// (128 bytes).
struct __align__(16) Surfel3D {
    float tu[3], tv[3], tw[3];
    float opacity;
    float s0, s1, s2;
    float cb[3];     // base colour
    float cv[3];     // view_dir . view_grads (linear view model), else 0
    float gu[3], gv[3];
    float n[3];      // viewer-facing normal (surface outputs), else 0
    union {
        float2 ctr;  // prefilter centre (prefilter on)
        short4 box;  // pixel box [x, z] x [y, w] holding every pixel with alpha >= 1/255
    } q;
    float nsign;     // the sign applied to that normal
    int id;
};
static_assert(sizeof(Surfel3D) == 128, "a staged surfel is eight 16-byte chunks");

// The staged surfel's pixel box: the screen bounds of the hexagon outside
// which its alpha is below 1/255 (the bound the reference's preprocess uses
// to pick the surfel's tiles), rounded outwards.  When the bound cannot be
// formed the box is unbounded, so nothing is skipped.
__device__ __forceinline__ short4 surfel_pixel_box(const Surfel3D& s, int W, int H) {
    const float smin = fminf(s.s0, fminf(s.s1, s.s2));
    const float smax = fmaxf(s.s0, fmaxf(s.s1, s.s2));
    float lox, loy, hix, hiy;
    if (!hex_screen_box(s.tu, s.tv, s.tw, hex_alpha_apothem(s.opacity, smin, smax), W, H, lox,
                        loy, hix, hiy))
        return make_short4(-32768, -32768, 32767, 32767);
    return make_short4((short)floorf(lox), (short)floorf(loy), (short)ceilf(hix),
                       (short)ceilf(hiy));
}

// Warp-uniform: does the box miss the warp's pixel block [x0, x1] x [y0, y1]?
__device__ __forceinline__ bool box_misses(const short4 b, int x0, int y0, int x1, int y1) {
    return b.x > x1 || b.z < x0 || b.y > y1 || b.w < y0;
}

// Pixel of thread `tr` within a 16x16 tile: each warp covers an 8x4 block
// (two blocks across, four down), so a small surfel's footprint meets fewer
// warps than with 16x2 rows.
__device__ __forceinline__ int2 tile_pixel(int tr) {
    const int warp = tr >> 5, lane = tr & 31;
    return make_int2(((warp & 1) << 3) + (lane & 7), ((warp >> 1) << 2) + (lane >> 3));
}

__device__ __forceinline__ float3 cross3(const float3 a, const float3 b) {
    return make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}

__device__ __forceinline__ float sigmoid_neg(const float dist, const float softness) {
    const float x = dist * softness;
    return 1.f / (1.f + __expf(x));
}

// Hexagon SDF max(|v|, |a u + b v|, |a u - b v|) - 1 without the edge: the
// same value as hex_sdf3 (for surfels whose three edges share one softness).
__device__ __forceinline__ float hex_sdf_value(const float u, const float v) {
    constexpr float k = 1.7320508f;
    constexpr float a = 0.5f * k;
    constexpr float b = 0.5f;
    return fmaxf(fmaxf(fabsf(a * u + b * v), fabsf(a * u - b * v)), fabsf(v)) - 1.f;
}

// Hexagon SDF max(|v|, |a u + b v|, |a u - b v|) - 1 and the active edge;
// slanted edges win ties with |v|, edge 2 wins ties with edge 1.
__device__ __forceinline__ float hex_sdf3(const float u, const float v, int& edge) {
    constexpr float k = 1.7320508f;
    constexpr float a = 0.5f * k;
    constexpr float b = 0.5f;
    const float d0 = fabsf(v);
    const float t1 = a * u + b * v;
    const float t2 = a * u - b * v;
    const float d1 = fabsf(t1);
    const float d2 = fabsf(t2);
    float m = d1;
    edge = 1;
    if (d2 >= m) {
        m = d2;
        edge = 2;
    }
    if (d0 > m) {
        edge = 0;
        return d0 - 1.f;
    }
    return m - 1.f;
}

// SDF with its (sub)gradient; here |x| uses sign(0) = +1.
__device__ __forceinline__ void hex_sdf3_grad(const float u, const float v, float& dist,
                                              float& ddu, float& ddv, int& edge) {
    constexpr float k = 1.7320508f;
    constexpr float a = 0.5f * k;
    constexpr float b = 0.5f;
    const float d0 = fabsf(v);
    const float t1 = a * u + b * v;
    const float t2 = a * u - b * v;
    const float d1 = fabsf(t1);
    const float d2 = fabsf(t2);
    float m = d1;
    edge = 1;
    if (d2 >= m) {
        m = d2;
        edge = 2;
    }
    if (d0 > m) {
        edge = 0;
        dist = d0 - 1.f;
        ddu = 0.f;
        ddv = (v >= 0.f) ? 1.f : -1.f;
        return;
    }
    dist = m - 1.f;
    if (edge == 1) {
        const float s = (t1 >= 0.f) ? 1.f : -1.f;
        ddu = a * s;
        ddv = b * s;
        return;
    }
    const float s = (t2 >= 0.f) ? 1.f : -1.f;
    ddu = a * s;
    ddv = -b * s;
}

// (u, v) scaled back onto the hexagon when outside it (quadratic_bounded).
__device__ __forceinline__ void bounded_coords(const float u, const float v, float& ub,
                                               float& vb) {
    int edge;
    const float rho = hex_sdf3(u, v, edge) + 1.f;
    const float inv = (rho > 1.f) ? (1.f / rho) : 1.f;
    ub = u * inv;
    vb = v * inv;
}

__device__ __forceinline__ void bounded_coords_vjp(const float u, const float v, const float gub,
                                                   const float gvb, float& gu, float& gv) {
    float dist, dru, drv;
    int edge;
    hex_sdf3_grad(u, v, dist, dru, drv, edge);
    const float rho = dist + 1.f;
    if (rho <= 1.f) {
        gu += gub;
        gv += gvb;
        return;
    }
    const float inv = 1.f / rho;
    const float radial = (gub * u + gvb * v) * inv * inv;
    gu += gub * inv - radial * dru;
    gv += gvb * inv - radial * drv;
}

__device__ __forceinline__ float normal_sign(const float3 n, const float* vd) {
    return n.x * vd[0] + n.y * vd[1] + n.z * vd[2] > 0.f ? -1.f : 1.f;
}

// Stages surfel g into its shared-memory row `row` (the per-surfel terms of
// both compositing kernels) and returns its pixel box (unbounded with the
// prefilter).  The record is written as eight 16-byte chunks, each as soon as
// its fields are loaded: a quarter-warp of such stores (one record per lane)
// is 8-way bank conflicted where field-by-field stores were 32-way, and the
// record is never held in registers whole.
template <bool SURF, bool PREFILTER, typename Args>
__device__ __forceinline__ short4 stage_surfel(const Args& a, int g, int W, int H,
                                               Surfel3D* row) {
    float4* dst = reinterpret_cast<float4*>(row);
    Surfel3D s;  // the fields the box needs
    const float* Tm = a.transMats + 9 * g;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        s.tu[c] = Tm[c];
        s.tv[c] = Tm[3 + c];
        s.tw[c] = Tm[6 + c];
    }
    s.opacity = a.opacities[g];
    if (a.softness_stride == 3) {
        s.s0 = a.softnesses[3 * g];
        s.s1 = a.softnesses[3 * g + 1];
        s.s2 = a.softnesses[3 * g + 2];
    } else {
        s.s0 = s.s1 = s.s2 = a.softnesses[g];
    }
    dst[0] = make_float4(s.tu[0], s.tu[1], s.tu[2], s.tv[0]);
    dst[1] = make_float4(s.tv[1], s.tv[2], s.tw[0], s.tw[1]);
    dst[2] = make_float4(s.tw[2], s.opacity, s.s0, s.s1);
    union {
        short4 box;
        float2 f;
    } q;
    short4 box;
    if (PREFILTER) {
        q.f = a.points_xy_center[g];
        box = make_short4(-32768, -32768, 32767, 32767);
    } else {
        box = surfel_pixel_box(s, W, H);
        q.box = box;
    }
    dst[3] = make_float4(s.s2, a.colors[3 * g], a.colors[3 * g + 1], a.colors[3 * g + 2]);
    float cv0 = 0.f, cv1 = 0.f, cv2 = 0.f;
    if (a.use_view_grads) {
        const float* vd = a.view_dirs + 3 * g;
        const float* vg = a.view_grads + 9 * g;
        cv0 = vd[0] * vg[0] + vd[1] * vg[1] + vd[2] * vg[2];
        cv1 = vd[0] * vg[3] + vd[1] * vg[4] + vd[2] * vg[5];
        cv2 = vd[0] * vg[6] + vd[1] * vg[7] + vd[2] * vg[8];
    }
    float gu[3] = {0.f, 0.f, 0.f}, gv[3] = {0.f, 0.f, 0.f};
    if (a.color_model >= kColorLinear) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            gu[c] = a.color_grads[6 * g + c];
            gv[c] = a.color_grads[6 * g + 3 + c];
        }
    }
    dst[4] = make_float4(cv0, cv1, cv2, gu[0]);
    dst[5] = make_float4(gu[1], gu[2], gv[0], gv[1]);
    float3 n = {0.f, 0.f, 0.f};
    float nsign = 1.f;
    if (SURF && a.normals) {
        n = {a.normals[3 * g], a.normals[3 * g + 1], a.normals[3 * g + 2]};
        nsign = normal_sign(n, a.view_dirs + 3 * g);
        n = {nsign * n.x, nsign * n.y, nsign * n.z};
    }
    dst[6] = make_float4(gv[2], n.x, n.y, n.z);
    dst[7] = make_float4(q.f.x, q.f.y, nsign, __int_as_float(g));
    return box;
}

// Copies surfel g's 128-byte record (written once per view by
// hx_hexels3d_surfel_records with the same layout stage_surfel produces)
// into the shared row `row` as eight 16-byte asynchronous copies that bypass
// L1; the issuing thread completes them with cp_async_wait_all() before it
// or, after a barrier, any other thread reads the row.
__device__ __forceinline__ void stage_record_async(const Surfel3D* records, int g,
                                                   Surfel3D* row) {
    const char* src = reinterpret_cast<const char*>(records + g);
    const unsigned dst = (unsigned)__cvta_generic_to_shared(row);
#pragma unroll
    for (int c = 0; c < 8; ++c)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst + 16 * c),
                     "l"(src + 16 * c)
                     : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// Ray-splat intersection of pixel (px, py) with a surfel of transform rows
// Tu, Tv, Tw: returns false when the ray is parallel or the hit is in front
// of the near plane; otherwise (u, v), depth, SDF, boundary weight and alpha.
// With one_softness (all edges share soft3.x) the active edge is not
// computed and h.edge is 0.
struct HexHit {
    float u, v, depth, dist, soft, boundary, alpha_raw, alpha;
    int edge;
    bool clamped;
};

__device__ __forceinline__ bool hexel_hit(const float px, const float py, const float3 Tu,
                                          const float3 Tv, const float3 Tw, const float opacity,
                                          const float3 soft3, const bool one_softness, HexHit& h) {
    const float3 k = {px * Tw.x - Tu.x, px * Tw.y - Tu.y, px * Tw.z - Tu.z};
    const float3 l = {py * Tw.x - Tv.x, py * Tw.y - Tv.y, py * Tw.z - Tv.z};
    const float3 p = cross3(k, l);
    if (p.z == 0.0f) return false;
    h.u = p.x / p.z;
    h.v = p.y / p.z;
    h.depth = (h.u * Tw.x + h.v * Tw.y) + Tw.z;
    if (h.depth < k3NearPlane) return false;
    if (one_softness) {  // the edge only selects a softness; not needed here
        h.dist = hex_sdf_value(h.u, h.v);
        h.edge = 0;
        h.soft = soft3.x;
    } else {
        h.dist = hex_sdf3(h.u, h.v, h.edge);
        h.soft = (h.edge == 0) ? soft3.x : ((h.edge == 1) ? soft3.y : soft3.z);
    }
    h.boundary = sigmoid_neg(h.dist, h.soft);
    h.alpha_raw = opacity * h.boundary;
    h.clamped = h.alpha_raw > 0.99f;
    h.alpha = h.clamped ? 0.99f : h.alpha_raw;
    return true;
}

}  // namespace hx
