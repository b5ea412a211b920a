// Shared definitions of the 3D hexel surfel kernels.
#pragma once

#include <float.h>

#include "hx_common.cuh"

namespace hx {

// Constants of the reference 3D rasteriser
// (gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:19-41).
constexpr int k3BlockX = 16;
constexpr int k3BlockY = 16;
constexpr int k3BlockSize = k3BlockX * k3BlockY;
constexpr float k3NearPlane = 0.2f;
constexpr float k3FarPlane = 100.0f;
constexpr float k3FilterSize = 0.707106f;
constexpr float k3FilterInvSquare = 2.0f;
constexpr float k3HexRadius = 1.15470053838f;
constexpr float k3Log254 = 5.537334267f;
// alpha from which the forward marks a (pixel block, list entry) pair as
// blending: 1/255 lowered by a relative 1e-4, far more than the few ulp by
// which the forward's and the backward's alpha of a pair can differ
constexpr float k3BlendMarkAlpha = (1.0f / 255.0f) * (1.0f - 1e-4f);

// Bits of the forward's blend mask covered by the warp `warp` of a CTA whose
// warps cover 8 x (4 ppt) pixel blocks, two across: bit 2 q + x-half for each
// 4-row quarter q of the 16x16 tile the warp's rows span.
__host__ __device__ constexpr unsigned blend_bits(int warp, int ppt) {
    unsigned bits = 0u;
    for (int k = 0; k < ppt; ++k) bits |= 1u << (2 * ((warp >> 1) * ppt + k) + (warp & 1));
    return bits;
}

// min/max with the reference's matrix-library semantics (ties and NaN pick x).
__device__ __forceinline__ float glm_min(float x, float y) { return (y < x) ? y : x; }
__device__ __forceinline__ float glm_max(float x, float y) { return (x < y) ? y : x; }

// Apothem, in surfel units, of the hexagon outside which the SDF alpha of a
// surfel with this opacity and softness range is below 1/255
// (hexels3d_forward.cu:479-487): 1 + ln(255 (1 + 8 eps) o - 1) / softness,
// with the smallest softness for a positive log and the largest for a
// negative one.
__device__ __forceinline__ float hex_alpha_apothem(float opacity, float softness_min,
                                                   float softness_max) {
    float margin = k3Log254 / softness_min;
    if (opacity > 1.f / 255.f) {
        const float log_cutoff = logf((255.f * (1.f + 8.f * FLT_EPSILON)) * opacity - 1.f);
        margin = log_cutoff / (log_cutoff < 0.f ? softness_max : softness_min);
    }
    return 1.f + margin;
}

__device__ __forceinline__ float dot3p(const float (&a)[3], const float* b) {
    return a[0] * b[0] + a[1] * b[1] + a[2] * b[2];
}

// Screen bounds [lo, hi] of the hexagon of the given apothem on the surfel
// plane, clipped at the near plane, padded by one pixel and clamped to one
// tile outside the image (hexels3d_forward.cu:221-258).  Tu, Tv, Tw are the
// transform's pixel-x, pixel-y and depth rows.  False when the hexagon does
// not reach the image.
__device__ __forceinline__ bool hex_screen_box(const float* Tu, const float* Tv, const float* Tw,
                                               float apothem, int W, int H, float& lox,
                                               float& loy, float& hix, float& hiy) {
    apothem += 4e-5f * fmaxf(1.f, fabsf(apothem));
    if (apothem <= 0.f) return false;
    const float r = k3HexRadius * apothem;
    const float vx[6] = {r, 0.5f * r, -0.5f * r, -r, -0.5f * r, 0.5f * r};
    const float vy[6] = {0.f, apothem, apothem, 0.f, -apothem, -apothem};
    lox = FLT_MAX;
    loy = FLT_MAX;
    hix = -FLT_MAX;
    hiy = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        const int i2 = (i + 1) % 6;
        const float a[3] = {vx[i], vy[i], 1.f};
        const float b[3] = {vx[i2], vy[i2], 1.f};
        const float za = dot3p(a, Tw);
        const float zb = dot3p(b, Tw);
        if (za >= k3NearPlane) {
            const float qx = dot3p(a, Tu) / za;
            const float qy = dot3p(a, Tv) / za;
            lox = glm_min(lox, qx);
            loy = glm_min(loy, qy);
            hix = glm_max(hix, qx);
            hiy = glm_max(hiy, qy);
        }
        if ((za < k3NearPlane) != (zb < k3NearPlane)) {
            const float s = (k3NearPlane - za) / (zb - za);
            const float e[3] = {a[0] + s * (b[0] - a[0]), a[1] + s * (b[1] - a[1]),
                                a[2] + s * (b[2] - a[2])};
            const float qx = dot3p(e, Tu) / k3NearPlane;
            const float qy = dot3p(e, Tv) / k3NearPlane;
            lox = glm_min(lox, qx);
            loy = glm_min(loy, qy);
            hix = glm_max(hix, qx);
            hiy = glm_max(hiy, qy);
        }
    }
    if (lox > W || loy > H || hix < -1.f || hiy < -1.f) return false;
    lox = glm_max(lox - 1.f, (float)-k3BlockX);
    loy = glm_max(loy - 1.f, (float)-k3BlockY);
    hix = glm_min(hix + 1.f, (float)(W + k3BlockX));
    hiy = glm_min(hiy + 1.f, (float)(H + k3BlockY));
    return true;
}

enum ColorModel { kColorFlat = 0, kColorLinear = 1, kColorQuadratic = 2, kColorQuadBounded = 3 };
enum ViewModel { kViewNone = 0, kViewLinear = 1, kViewLobe = 2 };

struct Prep3DArgs {
    int P;
    const float* means3d;
    const float2* scales;
    float scale_modifier;
    const float4* rotations;
    const float* opacities;
    const float* softnesses_in;
    float softness_default;
    int softness_stride;
    const float* viewmatrix;
    const float* projmatrix;
    const float* campos;
    int W, H;
    bool prefilter;
    bool conservative;
    int* radii;
    int2* tile_radii;
    float2* points_xy_image;
    float2* points_xy_center;
    float* depths;
    float* transMats;
    int* tiles_touched;
    float* opacities_out;
    float* softnesses_out;
    float* view_dirs;
    float* normals;
    uint2 grid;
};

// Pointers and options of the forward compositing kernel.
struct Surfel3D;  // the staged per-surfel record (hx_hexmath3d.cuh)

struct Render3DArgs {
    const uint2* ranges;
    const int* point_list;
    int num_rendered;
    int P;
    const float2* points_xy_center;
    int W, H;
    const float* colors;
    const float* color_grads;
    const float* color_quads;
    const float* view_grads;
    const float* specular_ks;
    const float* specular_log_s;
    const float* view_dirs;
    const float* transMats;
    const float* opacities;
    const float* softnesses;
    int softness_stride;
    const float* bg;
    const float* normals;
    int overdraw_base;
    int color_model;
    int view_model;
    bool use_view_grads;
    bool median;
    // outputs
    float* out_color;          // (3,H,W)
    float* contrib;            // (P,) or null
    float* overdraw;           // (H,W) or null
    float* overdraw_hits;      // (H,W) or null
    float* out_depth;          // (H,W) surface
    float* out_alpha;          // (H,W) surface
    float* out_surface;        // (4 or 5,H,W) surface
    long long* owner_id;       // (H,W) owner
    float* owner_weight;
    float* owner_uv;           // (2,H,W)
    float* owner_sdf;
    float* owner_depth;
    float* total_alpha;
    float* final_T;            // (H,W) or null
    int* last_index;           // (H,W) or null
    // surface state for the backward (all null or all set)
    float* final_T_surf;
    int* last_index_surf;
    float* m1_surf;
    float* m2_surf;
    int* median_index;
    // optional per-pixel counts (2,H,W) of the blended (contributing) pairs
    // and of the pairs evaluated after the warp's box cull, or null
    int* contrib_count;
    // optional per-intersection mask of the 8x4 pixel blocks that met the
    // surfel with alpha >= kBlendMarkAlpha while compositing, or null
    unsigned char* blend_mask;
    // optional per-surfel staged records (hx_hexels3d_surfel_records), or
    // null: the kernel then gathers each record from the arrays above
    const Surfel3D* records;
};

struct Backward3DArgs {
    const uint2* ranges;
    const int* point_list;
    int num_rendered;
    int P;
    const float2* points_xy_center;
    float2* grad_points_xy_center;
    int W, H;
    const float* colors;
    const float* color_grads;
    const float* color_quads;
    const float* view_grads;
    const float* specular_ks;
    const float* specular_log_s;
    int view_model;
    const float* view_dirs;
    const float* transMats;
    const float* opacities;
    const float* softnesses;
    int softness_stride;
    const float* bg;
    const float* grad_out_color;
    const float* grad_out_overdraw;
    const float* grad_out_surf_depth;
    const float* grad_out_surf_alpha;
    const float* grad_out_surf_normals;
    bool has_median_grad;
    const float* normals;
    float* grad_colors;
    float* grad_color_grads;
    float* grad_color_quads;
    float* grad_view_grads;
    float* grad_specular_ks;
    float* grad_specular_log_s;
    float* grad_opacities;
    float* grad_softnesses;
    float* grad_transMats;
    float* abs_means2d;
    float* grad_view_dirs;
    float* grad_normals;
    int overdraw_base;
    int color_model;
    bool use_view_grads;
    const float* final_T;
    const int* last_index;
    const float* final_T_surf;
    const int* last_index_surf;
    const float* m1_surf;
    const float* m2_surf;
    const int* median_index;
    // the forward's blend_mask, or null (no list entry skipped)
    const unsigned char* blend_mask;
    // optional per-surfel staged records (hx_hexels3d_surfel_records), or null
    const Surfel3D* records;
};

}  // namespace hx
