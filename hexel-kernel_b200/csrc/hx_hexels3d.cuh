// Shared definitions of the 3D hexel surfel kernels.
#pragma once

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
    // optional per-pixel count of blended (contributing) pairs, or null
    int* contrib_count;
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
};

}  // namespace hx
