// S11 diagnostics: the "exact sort" and "pixel risk" forwards of the 3D hexel
// rasteriser (reference gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:
// 1069-1489 kernels, 4217-4880 host).  The training forward composites each
// tile's list in the order of the surfels' centre depths; these passes
// re-sort each pixel's hits (alpha >= 1/255) by the depth at the pixel and
// composite them in that order, reporting where the two orders differ, and
// score how much an inversion of neighbouring hits can matter (risk map).
//
// Schedule: one CTA per 16x16 tile inside the crop; the tile's list is
// staged 256 records at a time (stage_surfel, the compositing kernels'
// staging) for the per-pixel hit tests; each pixel's hit records
// (pixel << 32 | depth bits, surfel) are then sorted by the library's stable
// radix sort, which keeps the centre-depth order of equal keys as the
// reference's stable CUB sort does, and composited one pixel per thread.
#include <float.h>

#include "hx_hexmath3d.cuh"
#include "hx_sort.cuh"

namespace hx {

// exact_mode values (hexels3d_forward.cu:36-41)
constexpr int kExactCenterReplay = 0;
constexpr int kExactHybrid = 1;
constexpr int kExactSelectedAll = 2;
constexpr int kExactCropAll = 3;
constexpr int kExactBoundaryTail = 4;
constexpr int kExactPixelMask = 5;

struct ExactArgs {
    Render3DArgs r;       // surfel arrays, colour and view models (staging)
    int crop_x0, crop_y0, crop_x1, crop_y1;
    const float* center_depths;
    const unsigned char* selected;  // (P,) or null
    const unsigned char* pixel_mask;  // (H,W) or null
    int mode;
};

namespace {

// Colour of a hit at (u, v): base, linear and quadratic colour terms, the
// linear view term, the specular lobe -- the forward's order
// (hexels3d_forward.cu:1069-1131).
__device__ __forceinline__ float3 hit_color(const Render3DArgs& a, const Surfel3D& s, int g,
                                            float u, float v) {
    float cx = s.cb[0], cy = s.cb[1], cz = s.cb[2];
    if (a.color_model >= kColorLinear) {
        cx += u * s.gu[0] + v * s.gv[0];
        cy += u * s.gu[1] + v * s.gv[1];
        cz += u * s.gu[2] + v * s.gv[2];
    }
    if (a.color_model == kColorQuadratic || a.color_model == kColorQuadBounded) {
        const float* cq = a.color_quads + 9 * g;
        float uu = u, vv = v;
        if (a.color_model == kColorQuadBounded) bounded_coords(u, v, uu, vv);
        const float u2 = uu * uu, uv = uu * vv, v2 = vv * vv;
        cx += u2 * cq[0] + uv * cq[3] + v2 * cq[6];
        cy += u2 * cq[1] + uv * cq[4] + v2 * cq[7];
        cz += u2 * cq[2] + uv * cq[5] + v2 * cq[8];
    }
    if (a.use_view_grads) {
        cx += s.cv[0];
        cy += s.cv[1];
        cz += s.cv[2];
    }
    if (a.view_model == kViewLobe) {
        const float* vd = a.view_dirs + 3 * g;
        const float* nr = a.normals + 3 * g;
        const float cos_nv = fmaxf(-(nr[0] * vd[0] + nr[1] * vd[1] + nr[2] * vd[2]), 0.f);
        const float s_exp = __expf(fminf(fmaxf(a.specular_log_s[g], 0.f), 5.0f));
        const float spec = (cos_nv > 0.f) ? __powf(cos_nv, s_exp) : 0.f;
        cx += a.specular_ks[3 * g] * spec;
        cy += a.specular_ks[3 * g + 1] * spec;
        cz += a.specular_ks[3 * g + 2] * spec;
    }
    return make_float3(cx, cy, cz);
}

// How close pixel (px, py) lies to the surfel's alpha = 1/255 contour along
// the active edge: 1 on the contour, falling to 0 one pixel away
// (hexels3d_forward.cu:1133-1186).  The contour is the line of the local
// hexagon at SDF level ln((o - a0) / a0) / softness across the edge's
// outward normal, mapped to the screen by the transform.
__device__ __forceinline__ float contour_proximity(float px, float py, float u, float v, int edge,
                                                  float opacity, float soft, const float3 Tu,
                                                  const float3 Tv, const float3 Tw) {
    constexpr float a0 = 1.f / 255.f;
    if (opacity <= a0) return 0.f;
    constexpr float ka = 0.8660254f, kb = 0.5f;
    float nu, nv;
    if (edge == 0) {
        nu = 0.f;
        nv = v >= 0.f ? 1.f : -1.f;
    } else if (edge == 1) {
        const float sg = (ka * u + kb * v >= 0.f) ? 1.f : -1.f;
        nu = sg * ka;
        nv = sg * kb;
    } else {
        const float sg = (ka * u - kb * v >= 0.f) ? 1.f : -1.f;
        nu = sg * ka;
        nv = -sg * kb;
    }
    const float level = 1.f + logf((opacity - a0) / a0) / soft;
    // a point of the contour and its direction, in homogeneous screen space
    const float3 pt = {Tu.x * (nu * level) + Tu.y * (nv * level) + Tu.z,
                       Tv.x * (nu * level) + Tv.y * (nv * level) + Tv.z,
                       Tw.x * (nu * level) + Tw.y * (nv * level) + Tw.z};
    const float3 dir = {Tu.x * (-nv) + Tu.y * nu, Tv.x * (-nv) + Tv.y * nu,
                        Tw.x * (-nv) + Tw.y * nu};
    const float3 line = cross3(pt, dir);
    const float len = sqrtf(line.x * line.x + line.y * line.y);
    if (len == 0.f) return 0.f;
    return fmaxf(0.f, 1.f - fabsf(line.x * px + line.y * py + line.z) / len);
}

struct ExactPixel {
    int x, y, pix;
    bool inside;
};

__device__ __forceinline__ ExactPixel exact_pixel(const ExactArgs& e) {
    ExactPixel p;
    p.x = (int)(blockIdx.x * k3BlockX + threadIdx.x % k3BlockX);
    p.y = (int)(blockIdx.y * k3BlockY + threadIdx.x / k3BlockX);
    p.pix = p.y * e.r.W + p.x;
    p.inside = p.x < e.r.W && p.y < e.r.H && p.x >= e.crop_x0 && p.x < e.crop_x1 &&
               p.y >= e.crop_y0 && p.y < e.crop_y1;
    return p;
}

__device__ __forceinline__ bool tile_outside_crop(const ExactArgs& e) {
    const int x0 = (int)(blockIdx.x * k3BlockX), y0 = (int)(blockIdx.y * k3BlockY);
    return x0 >= e.crop_x1 || y0 >= e.crop_y1 || x0 + k3BlockX <= e.crop_x0 ||
           y0 + k3BlockY <= e.crop_y0;
}

// The hit test of the compositing (alpha >= 1/255 at a valid intersection).
__device__ __forceinline__ bool exact_hit(const Surfel3D& s, float px, float py, HexHit& h) {
    const float3 Tu = {s.tu[0], s.tu[1], s.tu[2]};
    const float3 Tv = {s.tv[0], s.tv[1], s.tv[2]};
    const float3 Tw = {s.tw[0], s.tw[1], s.tw[2]};
    const float3 soft3 = {s.s0, s.s1, s.s2};
    if (!hexel_hit(px, py, Tu, Tv, Tw, s.opacity, soft3, false, h)) return false;
    return h.alpha >= 1.0f / 255.0f;
}

// Stages batch `round` of the tile's list into s_prim (and the selected
// flags); returns the batch size.
template <typename Body>
__device__ __forceinline__ void for_each_batch(const ExactArgs& e, uint2 range, Surfel3D* s_prim,
                                               unsigned char* s_sel, Body body) {
    const int len = (int)(range.y - range.x);
    for (int base = 0; base < len; base += k3BlockSize) {
        __syncthreads();
        const int t = threadIdx.x;
        if (base + t < len) {
            const int g = min(max(e.r.point_list[range.x + base + t], 0), e.r.P - 1);
            stage_surfel<false, false>(e.r, g, e.r.W, e.r.H, &s_prim[t]);
            s_sel[t] = e.selected ? e.selected[g] : (unsigned char)0;
        }
        __syncthreads();
        if (!body(base, min(k3BlockSize, len - base))) break;
    }
}

__device__ __forceinline__ uint2 tile_range(const ExactArgs& e) {
    const unsigned hblocks = (unsigned)((e.r.W + k3BlockX - 1) / k3BlockX);
    uint2 range = e.r.ranges[blockIdx.y * hblocks + blockIdx.x];
    range.y = min(range.y, (unsigned)e.r.num_rendered);
    range.x = min(range.x, range.y);
    return range;
}

}  // namespace

// Per pixel of the crop: hits, records to sort (the hits of enabled
// pixels), enabled flag (hexels3d_forward.cu:1384-1489).
__global__ void __launch_bounds__(k3BlockSize) exact_count_kernel(const ExactArgs e,
                                                                  int* __restrict__ hit_counts,
                                                                  int* __restrict__ record_counts,
                                                                  unsigned char* __restrict__ enabled) {
    __shared__ Surfel3D s_prim[k3BlockSize];
    __shared__ unsigned char s_sel[k3BlockSize];
    if (tile_outside_crop(e)) return;
    const ExactPixel p = exact_pixel(e);
    int hits = 0;
    bool touched_selected = false;
    for_each_batch(e, tile_range(e), s_prim, s_sel, [&](int, int n) {
        if (p.inside) {
            for (int j = 0; j < n; ++j) {
                HexHit h;
                if (!exact_hit(s_prim[j], (float)p.x, (float)p.y, h)) continue;
                ++hits;
                touched_selected = touched_selected || s_sel[j];
            }
        }
        return true;
    });
    if (!p.inside) return;
    const bool on = e.mode == kExactPixelMask ? e.pixel_mask[p.pix] != 0
                    : (e.mode == kExactCenterReplay || e.mode == kExactCropAll ||
                       e.mode == kExactBoundaryTail || touched_selected);
    hit_counts[p.pix] = hits;
    record_counts[p.pix] = on ? hits : 0;
    enabled[p.pix] = on ? 1 : 0;
}

// The hit records of enabled pixels, in list (centre-depth) order: key
// pixel << 32 | bits of the sort depth -- the hit's own depth where the mode
// asks for it, else the surfel's centre depth (hexels3d_forward.cu:1490-1600).
__global__ void __launch_bounds__(k3BlockSize) exact_fill_kernel(
    const ExactArgs e, const unsigned char* __restrict__ enabled,
    const int* __restrict__ record_offsets, unsigned long long* __restrict__ keys,
    int* __restrict__ vals) {
    __shared__ Surfel3D s_prim[k3BlockSize];
    __shared__ unsigned char s_sel[k3BlockSize];
    if (tile_outside_crop(e)) return;
    const ExactPixel p = exact_pixel(e);
    const bool on = p.inside && enabled[p.pix];
    int w = on ? (p.pix == 0 ? 0 : record_offsets[p.pix - 1]) : 0;
    for_each_batch(e, tile_range(e), s_prim, s_sel, [&](int, int n) {
        if (on) {
            for (int j = 0; j < n; ++j) {
                HexHit h;
                if (!exact_hit(s_prim[j], (float)p.x, (float)p.y, h)) continue;
                const int g = s_prim[j].id;
                const bool own_depth = e.mode == kExactSelectedAll || e.mode == kExactCropAll ||
                                       e.mode == kExactPixelMask ||
                                       (e.mode == kExactHybrid && s_sel[j]) ||
                                       (e.mode == kExactBoundaryTail && h.dist >= 0.f);
                const float d = own_depth ? h.depth : e.center_depths[g];
                keys[w] = ((unsigned long long)(unsigned)p.pix << 32) | __float_as_uint(d);
                vals[w] = g;
                ++w;
            }
        }
        return true;
    });
}

// Inversion risk of each crop pixel over its list in compositing order:
// for consecutive blended hits whose pixel depths are out of order, the
// largest T_prev alpha_prev alpha contrast max(contour proximities)
// (hexels3d_forward.cu:1188-1383).
__global__ void __launch_bounds__(k3BlockSize) exact_risk_kernel(const ExactArgs e,
                                                                 float* __restrict__ risk_map) {
    __shared__ Surfel3D s_prim[k3BlockSize];
    __shared__ unsigned char s_sel[k3BlockSize];
    __shared__ int s_done;
    if (tile_outside_crop(e)) return;
    const ExactPixel p = exact_pixel(e);
    bool done = !p.inside;
    float T = 1.f, risk = 0.f;
    bool have_prev = false;
    float prev_depth = 0.f, prev_alpha = 0.f, prev_T = 1.f, prev_contour = 0.f;
    float3 prev_c = {0.f, 0.f, 0.f};
    for_each_batch(e, tile_range(e), s_prim, s_sel, [&](int, int n) {
        for (int j = 0; !done && j < n; ++j) {
            HexHit h;
            if (!exact_hit(s_prim[j], (float)p.x, (float)p.y, h)) continue;
            const float alpha = h.alpha;
            const float test_T = T * (1.f - alpha);
            if (test_T < 0.0001f) {
                done = true;
                continue;
            }
            const Surfel3D& s = s_prim[j];
            const float3 c = hit_color(e.r, s, s.id, h.u, h.v);
            const float contour = contour_proximity(
                (float)p.x, (float)p.y, h.u, h.v, h.edge, s.opacity, h.soft,
                make_float3(s.tu[0], s.tu[1], s.tu[2]), make_float3(s.tv[0], s.tv[1], s.tv[2]),
                make_float3(s.tw[0], s.tw[1], s.tw[2]));
            if (have_prev) {
                const float tol = 8.f * FLT_EPSILON * fmaxf(1.f, fmaxf(fabsf(prev_depth),
                                                                       fabsf(h.depth)));
                if (prev_depth > h.depth + tol) {
                    const float contrast = fminf(
                        1.f, fmaxf(fabsf(prev_c.x - c.x),
                                   fmaxf(fabsf(prev_c.y - c.y), fabsf(prev_c.z - c.z))));
                    risk = fmaxf(risk, prev_T * prev_alpha * alpha * contrast *
                                           fmaxf(prev_contour, contour));
                }
            }
            have_prev = true;
            prev_depth = h.depth;
            prev_alpha = alpha;
            prev_T = T;
            prev_contour = contour;
            prev_c = c;
            T = test_T;
        }
        // the whole tile stops once every pixel is done
        if (threadIdx.x == 0) s_done = 0;
        __syncthreads();
        if (!done) atomicAdd(&s_done, 1);
        __syncthreads();
        return s_done > 0;
    });
    if (p.inside) risk_map[p.pix] = risk;
}

}  // namespace hx

namespace hx {

// Per enabled crop pixel: whether the sorted record order differs from the
// list order, and the colour composited front to back in the sorted order
// (hexels3d_forward.cu:1601-1747); other pixels keep the caller's image.
__global__ void __launch_bounds__(k3BlockSize) exact_composite_kernel(
    const ExactArgs e, const unsigned char* __restrict__ enabled,
    const int* __restrict__ record_counts, const int* __restrict__ record_offsets,
    const int* __restrict__ vals_unsorted, const int* __restrict__ vals_sorted,
    float* __restrict__ out_color, unsigned char* __restrict__ order_changed) {
    if (tile_outside_crop(e)) return;
    const ExactPixel p = exact_pixel(e);
    if (!p.inside || !enabled[p.pix]) return;
    const int count = record_counts[p.pix];
    const int start = p.pix == 0 ? 0 : record_offsets[p.pix - 1];
    bool changed = false;
    for (int i = 0; i < count; ++i) changed |= vals_unsorted[start + i] != vals_sorted[start + i];
    order_changed[p.pix] = changed ? 1 : 0;
    float T = 1.f, cx = 0.f, cy = 0.f, cz = 0.f;
    for (int i = 0; i < count; ++i) {
        const int g = min(max(vals_sorted[start + i], 0), e.r.P - 1);
        Surfel3D s;
        stage_surfel<false, false>(e.r, g, e.r.W, e.r.H, &s);
        HexHit h;
        if (!exact_hit(s, (float)p.x, (float)p.y, h)) continue;
        const float test_T = T * (1.f - h.alpha);
        if (test_T < 0.0001f) break;
        const float w = h.alpha * T;
        const float3 c = hit_color(e.r, s, g, h.u, h.v);
        cx += c.x * w;
        cy += c.y * w;
        cz += c.z * w;
        T = test_T;
    }
    const int HW = e.r.W * e.r.H;
    out_color[p.pix] = cx + T * e.r.bg[0];
    out_color[HW + p.pix] = cy + T * e.r.bg[1];
    out_color[2 * HW + p.pix] = cz + T * e.r.bg[2];
}

namespace {

int exact_args(ExactArgs& e, int P, int num_rendered, const int32_t* ranges,
               const int32_t* point_list, int W, int H, const float* colors,
               const float* color_grads, const float* color_quads, const float* view_grads,
               const float* specular_ks, const float* specular_log_s, const float* view_dirs,
               const float* normals, const float* transMats, const float* opacities,
               const float* softnesses, int softness_stride, const float* background,
               const float* center_depths, const uint8_t* selected, const uint8_t* pixel_mask,
               int color_model, int view_model, int use_view_grads, int mode, int cx0, int cy0,
               int cx1, int cy1) {
    HX_REQUIRE(W > 0 && H > 0, "invalid image dimensions");
    HX_REQUIRE((long long)W * H <= 0x7fffffffLL, "image has too many pixels for exact-sort keys");
    HX_REQUIRE(mode >= kExactCenterReplay && mode <= kExactPixelMask, "invalid exact sort mode");
    HX_REQUIRE(cx0 >= 0 && cy0 >= 0 && cx0 < cx1 && cy0 < cy1 && cx1 <= W && cy1 <= H,
               "crop must satisfy 0 <= x0 < x1 <= W and 0 <= y0 < y1 <= H");
    HX_REQUIRE(softness_stride == 1 || softness_stride == 3, "softness_stride must be 1 or 3");
    HX_REQUIRE(color_model >= 0 && color_model <= 3, "color_model must be 0..3");
    HX_REQUIRE(view_model >= 0 && view_model <= 2, "view_model must be 0..2");
    HX_REQUIRE(ranges && background, "hexels3d_exact: null pointer");
    HX_REQUIRE(num_rendered == 0 || (point_list && transMats && opacities && softnesses &&
                                     colors && view_dirs && center_depths && P > 0),
               "hexels3d_exact: null pointer");
    HX_REQUIRE(color_model < 1 || color_grads, "color_grads required for color_model >= 1");
    HX_REQUIRE(color_model < 2 || color_quads, "color_quads required for quadratic models");
    HX_REQUIRE(!use_view_grads || view_grads, "view_grads required with use_view_grads");
    HX_REQUIRE(view_model != 2 || (specular_ks && specular_log_s && normals),
               "lobe view model needs specular_ks, specular_log_s and normals");
    HX_REQUIRE(mode != kExactPixelMask || pixel_mask, "pixel-mask mode needs pixel_mask");
    e = ExactArgs{};
    Render3DArgs& a = e.r;
    a.ranges = (const uint2*)ranges;
    a.point_list = point_list;
    a.num_rendered = num_rendered;
    a.P = P;
    a.W = W;
    a.H = H;
    a.colors = colors;
    a.color_grads = color_grads;
    a.color_quads = color_quads;
    a.view_grads = view_grads;
    a.specular_ks = specular_ks;
    a.specular_log_s = specular_log_s;
    a.view_dirs = view_dirs;
    a.normals = normals;
    a.transMats = transMats;
    a.opacities = opacities;
    a.softnesses = softnesses;
    a.softness_stride = softness_stride;
    a.bg = background;
    a.color_model = color_model;
    a.view_model = view_model;
    a.use_view_grads = use_view_grads != 0;
    e.crop_x0 = cx0;
    e.crop_y0 = cy0;
    e.crop_x1 = cx1;
    e.crop_y1 = cy1;
    e.center_depths = center_depths;
    e.selected = selected;
    e.pixel_mask = pixel_mask;
    e.mode = mode;
    return HX_OK;
}

}  // namespace
}  // namespace hx

using namespace hx;

#define HX_EXACT_PARAMS                                                                          \
    int P, int num_rendered, const int32_t *ranges, const int32_t *point_list, int image_width,  \
        int image_height, const float *colors, const float *color_grads,                         \
        const float *color_quads, const float *view_grads, const float *specular_ks,             \
        const float *specular_log_s, const float *view_dirs, const float *normals,               \
        const float *transMats, const float *opacities, const float *softnesses,                 \
        int softness_stride, const float *background, const float *center_depths,                \
        const uint8_t *selected_mask, const uint8_t *pixel_mask, int color_model, int view_model, \
        int use_view_grads, int exact_mode, int crop_x0, int crop_y0, int crop_x1, int crop_y1
#define HX_EXACT_ARGS                                                                           \
    P, num_rendered, ranges, point_list, image_width, image_height, colors, color_grads,         \
        color_quads, view_grads, specular_ks, specular_log_s, view_dirs, normals, transMats,     \
        opacities, softnesses, softness_stride, background, center_depths, selected_mask,        \
        pixel_mask, color_model, view_model, use_view_grads, exact_mode, crop_x0, crop_y0,       \
        crop_x1, crop_y1

extern "C" int hx_hexels3d_exact_count(HX_EXACT_PARAMS, int32_t* hit_counts,
                                       int32_t* record_counts, uint8_t* enabled, float* risk_map,
                                       cudaStream_t stream) {
    ExactArgs e;
    const int rc = exact_args(e, HX_EXACT_ARGS);
    if (rc != HX_OK) return rc;
    HX_REQUIRE(hit_counts && record_counts && enabled, "hexels3d_exact_count: null pointer");
    const dim3 grid(ceil_div(image_width, k3BlockX), ceil_div(image_height, k3BlockY));
    if (risk_map) {
        exact_risk_kernel<<<grid, k3BlockSize, 0, stream>>>(e, risk_map);
        HX_LAUNCH_CHECK("exact_risk_kernel");
    }
    exact_count_kernel<<<grid, k3BlockSize, 0, stream>>>(e, hit_counts, record_counts, enabled);
    HX_LAUNCH_CHECK("exact_count_kernel");
    return HX_OK;
}

extern "C" size_t hx_hexels3d_exact_resolve_workspace_bytes(int num_records) {
    const size_t n = num_records > 0 ? (size_t)num_records : 1;
    return 2 * align256(sizeof(unsigned long long) * n) + 2 * align256(sizeof(int) * n) +
           sort_workspace_bytes<unsigned long long>((int)n);
}

extern "C" int hx_hexels3d_exact_resolve(HX_EXACT_PARAMS, const uint8_t* enabled,
                                         const int32_t* record_counts,
                                         const int32_t* record_offsets, int num_records,
                                         float* out_color, uint8_t* order_changed,
                                         void* workspace, size_t workspace_bytes,
                                         cudaStream_t stream) {
    ExactArgs e;
    const int rc = exact_args(e, HX_EXACT_ARGS);
    if (rc != HX_OK) return rc;
    HX_REQUIRE(num_records >= 0, "hexels3d_exact_resolve: bad num_records");
    HX_REQUIRE(enabled && record_counts && record_offsets && out_color && order_changed,
               "hexels3d_exact_resolve: null pointer");
    const size_t need = hx_hexels3d_exact_resolve_workspace_bytes(num_records);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE, "hexels3d_exact_resolve: workspace of %zu bytes needed",
                         need);
    char* p = (char*)workspace;
    const size_t n = num_records > 0 ? (size_t)num_records : 1;
    unsigned long long* keys = (unsigned long long*)p;
    p += align256(sizeof(unsigned long long) * n);
    unsigned long long* keys_sorted = (unsigned long long*)p;
    p += align256(sizeof(unsigned long long) * n);
    int* vals = (int*)p;
    p += align256(sizeof(int) * n);
    int* vals_sorted = (int*)p;
    p += align256(sizeof(int) * n);
    const dim3 grid(ceil_div(image_width, k3BlockX), ceil_div(image_height, k3BlockY));
    if (num_records > 0) {
        exact_fill_kernel<<<grid, k3BlockSize, 0, stream>>>(e, enabled, record_offsets, keys,
                                                            vals);
        HX_LAUNCH_CHECK("exact_fill_kernel");
        // stable: equal pixel-depth keys keep the list (centre-depth) order
        const int pix_bits = tile_bits(image_width * image_height);
        const int r2 = sort_pairs<unsigned long long>(keys, vals, keys_sorted, vals_sorted,
                                                      num_records, 0, 32 + pix_bits, p,
                                                      sort_workspace_bytes<unsigned long long>(
                                                          num_records),
                                                      stream);
        if (r2 != HX_OK) return r2;
    }
    exact_composite_kernel<<<grid, k3BlockSize, 0, stream>>>(e, enabled, record_counts,
                                                             record_offsets, vals, vals_sorted,
                                                             out_color, order_changed);
    HX_LAUNCH_CHECK("exact_composite_kernel");
    return HX_OK;
}
