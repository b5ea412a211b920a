// S1: per-Gaussian 2D projection (scale/rotation -> conic, radius, tile count)
// and its vector-Jacobian product.
//
// Follows gsplat/cuda/csrc/foward2d.cu:9-59, backward2d.cu:53-100 and
// helpers.cuh:11-82 of the reference.  The arithmetic is written in the same
// order (and compiled with the same fast-math flags) so that radii and tile
// counts are bit-identical; the kernels additionally write every output
// element, so callers need no zero fill.
#include "hx_common.cuh"
#include "hx_mat.cuh"
#include "hx_tiles.cuh"

namespace hx {

// Conic (inverse covariance) and 3-sigma radius of a 2D covariance given by
// its upper triangle; false for a singular matrix (helpers.cuh:45-68).
__device__ __forceinline__ bool cov2d_bounds(const float3 cov2d, float3& conic, float& radius) {
    float det = cov2d.x * cov2d.z - cov2d.y * cov2d.y;
    if (det == 0.f) return false;
    float inv_det = 1.f / det;
    conic.x = cov2d.z * inv_det;
    conic.y = -cov2d.y * inv_det;
    conic.z = cov2d.x * inv_det;
    float b = 0.5f * (cov2d.x + cov2d.z);
    float v1 = b + sqrt(max(0.1f, b * b - det));
    float v2 = b - sqrt(max(0.1f, b * b - det));
    radius = ceil(3.f * sqrt(max(v1, v2)));
    return true;
}

__global__ void __launch_bounds__(256) project2d_fwd_kernel(
    int n, const float2* __restrict__ means2d, const float2* __restrict__ scales2d,
    const float* __restrict__ rotation, unsigned img_w, unsigned img_h, int tiles_x, int tiles_y,
    float2* __restrict__ xys, int* __restrict__ radii, float3* __restrict__ conics,
    int* __restrict__ num_tiles_hit) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    const float2 m = means2d[idx];
    const float2 center = {m.x * img_w, m.y * img_h};
    const float2 s = scales2d[idx];

    const Mat2 R = rot2(rotation[idx]);
    const Mat2 S = scale2(s.x, s.y);
    const Mat2 M = mul(R, S);
    const Mat2 cov = mul(M, transpose(M));
    const float3 cov2d = make_float3(cov.m[0][0], cov.m[0][1], cov.m[1][1]);

    float3 conic;
    float radius;
    if (!cov2d_bounds(cov2d, conic, radius)) {
        xys[idx] = make_float2(0.f, 0.f);
        conics[idx] = make_float3(0.f, 0.f, 0.f);
        radii[idx] = 0;
        num_tiles_hit[idx] = 0;
        return;
    }
    conics[idx] = conic;
    xys[idx] = center;
    radii[idx] = (int)radius;
    TileRect r = tile_rect(center, radius, tiles_x, tiles_y);
    const int area = (int)((r.x1 - r.x0) * (r.y1 - r.y0));
    num_tiles_hit[idx] = area > 0 ? area : 0;
}

__global__ void __launch_bounds__(256) project2d_bwd_kernel(
    int n, const float2* __restrict__ scales2d, const float* __restrict__ rotation,
    unsigned img_w, unsigned img_h, const int* __restrict__ radii,
    const float3* __restrict__ conics, const float2* __restrict__ v_xy,
    const float3* __restrict__ v_conic, float3* __restrict__ v_cov2d,
    float2* __restrict__ v_mean2d, float2* __restrict__ v_scale, float* __restrict__ v_rot) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    if (radii[idx] <= 0) {
        v_cov2d[idx] = make_float3(0.f, 0.f, 0.f);
        v_mean2d[idx] = make_float2(0.f, 0.f);
        v_scale[idx] = make_float2(0.f, 0.f);
        v_rot[idx] = 0.f;
        return;
    }
    // d(loss)/d(cov2d) = -conic * d(loss)/d(conic) * conic (helpers.cuh:71-82)
    const float3 c = conics[idx];
    const float3 vc = v_conic[idx];
    const Mat2 X = mat2(c.x, c.y, c.y, c.z);
    const Mat2 G = mat2(vc.x, vc.y, vc.y, vc.z);
    const Mat2 vS = mul(mul(neg(X), G), X);
    const float G11 = vS.m[0][0];
    const float G12 = vS.m[1][0] + vS.m[0][1];
    const float G22 = vS.m[1][1];
    v_cov2d[idx] = make_float3(G11, G12, G22);

    const float rot = rotation[idx];
    const float2 s = scales2d[idx];
    const Mat2 R = rot2(rot);
    const Mat2 Rg = rot2_grad(rot);
    const Mat2 S = scale2(s.x, s.y);
    const Mat2 M = mul(R, S);
    const Mat2 theta_g =
        add(mul(mul(Rg, S), transpose(M)), mul(mul(M, transpose(S)), transpose(Rg)));
    Mat2 sxg = mat2_diag(0.f);
    sxg.m[0][0] = 2.f * s.x;
    Mat2 syg = mat2_diag(0.f);
    syg.m[1][1] = 2.f * s.y;
    const Mat2 sig_x = mul(mul(R, sxg), transpose(R));
    const Mat2 sig_y = mul(mul(R, syg), transpose(R));

    float2 vs;
    vs.x = G11 * sig_x.m[0][0] + 2 * G12 * sig_x.m[0][1] + G22 * sig_x.m[1][1];
    vs.y = G11 * sig_y.m[0][0] + 2 * G12 * sig_y.m[0][1] + G22 * sig_y.m[1][1];
    v_scale[idx] = vs;
    v_rot[idx] = G11 * theta_g.m[0][0] + 2 * G12 * theta_g.m[0][1] + G22 * theta_g.m[1][1];
    const float2 vxy = v_xy[idx];
    v_mean2d[idx] = make_float2(vxy.x * img_w, vxy.y * img_h);
}

__global__ void __launch_bounds__(256) cov2d_bounds_kernel(int n, const float* __restrict__ covs,
                                                           float* __restrict__ conics,
                                                           float* __restrict__ radii) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= n) return;
    const float3 cov = make_float3(covs[3 * row], covs[3 * row + 1], covs[3 * row + 2]);
    float3 conic = make_float3(0.f, 0.f, 0.f);
    float radius = 0.f;
    if (!cov2d_bounds(cov, conic, radius)) {
        conic = make_float3(0.f, 0.f, 0.f);
        radius = 0.f;
    }
    conics[3 * row] = conic.x;
    conics[3 * row + 1] = conic.y;
    conics[3 * row + 2] = conic.z;
    radii[row] = radius;
}

}  // namespace hx

using namespace hx;

extern "C" int hx_project_gaussians_2d_scale_rot_forward(
    int num_points, const float* means2d, const float* scales2d, const float* rotation,
    unsigned img_height, unsigned img_width, int tiles_x, int tiles_y, float* xys,
    int32_t* radii, float* conics, int32_t* num_tiles_hit, cudaStream_t stream) {
    HX_REQUIRE(num_points >= 0, "num_points must be non-negative (got %d)", num_points);
    if (num_points == 0) return HX_OK;
    HX_REQUIRE(means2d && scales2d && rotation && xys && radii && conics && num_tiles_hit,
               "project_gaussians_2d_scale_rot_forward: null pointer");
    HX_REQUIRE(tiles_x > 0 && tiles_y > 0, "tile bounds must be positive");
    project2d_fwd_kernel<<<ceil_div(num_points, 256), 256, 0, stream>>>(
        num_points, (const float2*)means2d, (const float2*)scales2d, rotation, img_width,
        img_height, tiles_x, tiles_y, (float2*)xys, radii, (float3*)conics, num_tiles_hit);
    HX_LAUNCH_CHECK("project2d_fwd_kernel");
    return HX_OK;
}

extern "C" int hx_project_gaussians_2d_scale_rot_backward(
    int num_points, const float* means2d, const float* scales2d, const float* rotation,
    unsigned img_height, unsigned img_width, const int32_t* radii, const float* conics,
    const float* v_xy, const float* v_conic, float* v_cov2d, float* v_mean2d, float* v_scale,
    float* v_rot, cudaStream_t stream) {
    (void)means2d;
    HX_REQUIRE(num_points >= 0, "num_points must be non-negative (got %d)", num_points);
    if (num_points == 0) return HX_OK;
    HX_REQUIRE(scales2d && rotation && radii && conics && v_xy && v_conic && v_cov2d && v_mean2d &&
                   v_scale && v_rot,
               "project_gaussians_2d_scale_rot_backward: null pointer");
    project2d_bwd_kernel<<<ceil_div(num_points, 256), 256, 0, stream>>>(
        num_points, (const float2*)scales2d, rotation, img_width, img_height, radii,
        (const float3*)conics, (const float2*)v_xy, (const float3*)v_conic, (float3*)v_cov2d,
        (float2*)v_mean2d, (float2*)v_scale, v_rot);
    HX_LAUNCH_CHECK("project2d_bwd_kernel");
    return HX_OK;
}

extern "C" int hx_compute_cov2d_bounds(int num_points, const float* covs2d, float* conics,
                                       float* radii, cudaStream_t stream) {
    HX_REQUIRE(num_points >= 0, "num_points must be non-negative (got %d)", num_points);
    if (num_points == 0) return HX_OK;
    HX_REQUIRE(covs2d && conics && radii, "compute_cov2d_bounds: null pointer");
    cov2d_bounds_kernel<<<ceil_div(num_points, 256), 256, 0, stream>>>(num_points, covs2d, conics,
                                                                       radii);
    HX_LAUNCH_CHECK("cov2d_bounds_kernel");
    return HX_OK;
}
