// S6 / S7: 3D hexel surfel preprocessing and binning.
//
// preprocess: per surfel, the ray-splat transform T (3x3), the screen-space
// bounding box at the alpha cutoff, the hexagon-polygon tile bounds with
// near-plane clipping, depth, tile count, view direction and normal
// (reference gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:57-551).  The
// arithmetic is written in the reference's order and compiled with the same
// fast-math flags, so tile counts, radii, rectangles and T are bit-identical.
// Every output element is written (zeros for culled surfels).
//
// binning: (tile << 32 | depth bits) keys emitted surfel-major, tile rows then
// columns (hexels3d_forward.cu:553-584), a stable radix sort on bits
// [0, 32 + bits(tiles)) and tile ranges — same sorted lists as the
// reference's CUB stable sort.
#include <float.h>

#include "hx_cmat.cuh"
#include "hx_common.cuh"
#include "hx_hexels3d.cuh"
#include "hx_sort.cuh"

namespace hx {

namespace {

__device__ __forceinline__ float3 transform_point_4x3(const float3 p, const float* m) {
    return {m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12],
            m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13],
            m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14]};
}

__device__ __forceinline__ float gmax(float x, float y) { return (x < y) ? y : x; }

// Tile rectangle [min, max) of a box centred at p with half extents r, in
// tiles (hexels3d_forward.cu:80-91).
__device__ __forceinline__ void get_rect(const float2 p, const int2 r, uint2& rmin, uint2& rmax,
                                         const uint2 grid) {
    rmin = {min(grid.x, (unsigned)max(0, (int)((p.x - (float)r.x) / (float)k3BlockX))),
            min(grid.y, (unsigned)max(0, (int)((p.y - (float)r.y) / (float)k3BlockY)))};
    rmax = {min(grid.x, (unsigned)max(0, (int)((p.x + (float)r.x + (float)k3BlockX - 1.f) /
                                               (float)k3BlockX))),
            min(grid.y, (unsigned)max(0, (int)((p.y + (float)r.y + (float)k3BlockY - 1.f) /
                                               (float)k3BlockY)))};
}

// world -> NDC matrix from the transposed projection matrix.
__device__ __forceinline__ Cmat<4, 4> world2ndc_of(const float* pm) {
    Cmat<4, 4> m;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) m.m[c][r] = pm[4 * r + c];
    return m;
}

__device__ __forceinline__ Cmat<3, 4> ndc2pix_of(int W, int H) {
    Cmat<3, 4> m;
    m.m[0][0] = (float)W / 2.0f; m.m[0][1] = 0.0f; m.m[0][2] = 0.0f;
    m.m[0][3] = ((float)W - 1.0f) / 2.0f;
    m.m[1][0] = 0.0f; m.m[1][1] = (float)H / 2.0f; m.m[1][2] = 0.0f;
    m.m[1][3] = ((float)H - 1.0f) / 2.0f;
    m.m[2][0] = 0.0f; m.m[2][1] = 0.0f; m.m[2][2] = 0.0f; m.m[2][3] = 1.0f;
    return m;
}

// Surfel-to-world columns (scaled tangent axes and centre).
__device__ __forceinline__ Cmat<3, 4> splat2world_of(const Cmat<3, 3>& R, float sx, float sy,
                                                     float mod, const float3 p) {
    Cmat<3, 3> S;
    S.m[0][0] = 1.f; S.m[0][1] = 0.f; S.m[0][2] = 0.f;
    S.m[1][0] = 0.f; S.m[1][1] = 1.f; S.m[1][2] = 0.f;
    S.m[2][0] = 0.f; S.m[2][1] = 0.f; S.m[2][2] = 1.f;
    S.m[0][0] = mod * sx;
    S.m[1][1] = mod * sy;
    const Cmat<3, 3> L = mmul<3, 3, 3>(R, S);
    Cmat<3, 4> s2w;
    s2w.m[0][0] = L.m[0][0]; s2w.m[0][1] = L.m[0][1]; s2w.m[0][2] = L.m[0][2]; s2w.m[0][3] = 0.0f;
    s2w.m[1][0] = L.m[1][0]; s2w.m[1][1] = L.m[1][1]; s2w.m[1][2] = L.m[1][2]; s2w.m[1][3] = 0.0f;
    s2w.m[2][0] = p.x; s2w.m[2][1] = p.y; s2w.m[2][2] = p.z; s2w.m[2][3] = 1.0f;
    return s2w;
}

// T = splat2world^T * world2ndc * ndc2pix (hexels3d_forward.cu:156-202).
__device__ __forceinline__ Cmat<3, 3> compute_transmat(const float3 p, float sx, float sy,
                                                       float mod, const float4 rot,
                                                       const float* projmatrix, int W, int H) {
    const Cmat<3, 3> R = quat_to_rotmat_wxyz(rot);
    const Cmat<3, 4> s2w = splat2world_of(R, sx, sy, mod, p);
    const Cmat<4, 3> s2wT = mtranspose<3, 4>(s2w);
    const Cmat<4, 3> a = mmul<4, 4, 3>(s2wT, world2ndc_of(projmatrix));
    return mmul<3, 4, 3>(a, ndc2pix_of(W, H));
}

__device__ __forceinline__ float dot_sq(const float* t, const float* a, const float* b) {
    // dot(t, a * b) with the product taken first, summed x, y, z.
    return t[0] * (a[0] * b[0]) + t[1] * (a[1] * b[1]) + t[2] * (a[2] * b[2]);
}

// Screen-space centre and half extents of the surfel at the cutoff
// (hexels3d_forward.cu:204-219).
__device__ __forceinline__ bool compute_aabb(const Cmat<3, 3>& T, float cutoff, float2& point,
                                             float2& extent, bool& bounded) {
    const float t[3] = {cutoff * cutoff, cutoff * cutoff, -1.0f};
    const float d = dot_sq(t, T.m[2], T.m[2]);
    bounded = d < 0.0f;
    if (d == 0.0f) return false;
    const float inv = 1.0f / d;
    const float f[3] = {inv * t[0], inv * t[1], inv * t[2]};
    const float px = dot_sq(f, T.m[0], T.m[2]);
    const float py = dot_sq(f, T.m[1], T.m[2]);
    const float h0x = px * px - dot_sq(f, T.m[0], T.m[0]);
    const float h0y = py * py - dot_sq(f, T.m[1], T.m[1]);
    point = {px, py};
    extent = {sqrt(gmax(1e-4f, h0x)), sqrt(gmax(1e-4f, h0y))};
    return true;
}

// Centre and half extents of the projected hexagon of apothem `apothem` (in
// surfel units), clipped at the near plane (hexels3d_forward.cu:221-258).
__device__ __forceinline__ bool compute_hex_bounds(const Cmat<3, 3>& T, float apothem, int W,
                                                   int H, float2& center, int2& radius) {
    float lox, loy, hix, hiy;
    if (!hex_screen_box(T.m[0], T.m[1], T.m[2], apothem, W, H, lox, loy, hix, hiy)) return false;
    center = {(lox + hix) * 0.5f, (loy + hiy) * 0.5f};
    radius = {(int)ceilf((hix - lox) * 0.5f) + 1, (int)ceilf((hiy - loy) * 0.5f) + 1};
    return true;
}

}  // namespace

__global__ void __launch_bounds__(256) preprocess3d_kernel(const Prep3DArgs a) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= a.P) return;
    const float3 p = {a.means3d[3 * idx], a.means3d[3 * idx + 1], a.means3d[3 * idx + 2]};
    const float3 c = {a.campos[0], a.campos[1], a.campos[2]};
    const float3 d = {p.x - c.x, p.y - c.y, p.z - c.z};
    const float inv_norm = rsqrtf(d.x * d.x + d.y * d.y + d.z * d.z + 1e-8f);
    a.view_dirs[3 * idx + 0] = d.x * inv_norm;
    a.view_dirs[3 * idx + 1] = d.y * inv_norm;
    a.view_dirs[3 * idx + 2] = d.z * inv_norm;

    int radius_out = 0;
    int2 tile_radius_out = {0, 0};
    int touched = 0;
    bool write = false;
    float2 point_image = {0.f, 0.f};
    float depth = 0.f;
    Cmat<3, 3> T;
    float3 softness3 = {0.f, 0.f, 0.f};
    float4 rot = {0.f, 0.f, 0.f, 0.f};

    const float3 p_view = transform_point_4x3(p, a.viewmatrix);
    do {
        if (!(p_view.z > k3NearPlane)) break;
        rot = a.rotations[idx];
        const float2 sc = a.scales[idx];
        T = compute_transmat(p, sc.x, sc.y, a.scale_modifier, rot, a.projmatrix, a.W, a.H);
        softness3 = {a.softness_default, a.softness_default, a.softness_default};
        if (a.softnesses_in != nullptr) {
            if (a.softness_stride == 1) {
                const float s = a.softnesses_in[idx];
                softness3 = {s, s, s};
            } else if (a.softness_stride == 3) {
                const float* s = a.softnesses_in + idx * 3;
                softness3 = {s[0], s[1], s[2]};
            }
        }
        softness3.x = fmaxf(softness3.x, 1e-4f);
        softness3.y = fmaxf(softness3.y, 1e-4f);
        softness3.z = fmaxf(softness3.z, 1e-4f);
        const float softness_min = fminf(softness3.x, fminf(softness3.y, softness3.z));
        const float cutoff = k3HexRadius * (1.0f + (k3Log254 / softness_min));

        float2 extent = {0.f, 0.f};
        bool bounded;
        const bool old_bound = compute_aabb(T, cutoff, point_image, extent, bounded);
        float radius_base = fmaxf(fmaxf(extent.x, extent.y), cutoff * k3FilterSize);
        if (a.prefilter) radius_base = fmaxf(radius_base, 3.f * k3FilterSize);
        const int radius = old_bound ? (int)ceilf(radius_base) : 0;
        uint2 rmin, rmax;
        get_rect(point_image, {radius, radius}, rmin, rmax, a.grid);
        const bool old_visible = old_bound && rmin.x < rmax.x && rmin.y < rmax.y;
        const bool corrected = a.conservative && !a.prefilter;
        if (!old_visible && !corrected) break;
        radius_out = old_visible ? radius : 0;

        int2 tile_radius = {radius, radius};
        const float opacity = a.opacities[idx];
        if (!a.prefilter && bounded && opacity <= 1.f) {
            tile_radius.x = min(radius, (int)ceilf(fmaxf(extent.x, cutoff * k3FilterSize)) + 1);
            tile_radius.y = min(radius, (int)ceilf(fmaxf(extent.y, cutoff * k3FilterSize)) + 1);
            get_rect(point_image, tile_radius, rmin, rmax, a.grid);
        }
        const uint2 legacy_min = rmin, legacy_max = rmax;
        if (!a.prefilter) {
            if (opacity < 1.f / 255.f) break;
            const float softness_max = fmaxf(softness3.x, fmaxf(softness3.y, softness3.z));
            const float apothem = hex_alpha_apothem(opacity, softness_min, softness_max);
            if (!compute_hex_bounds(T, apothem, a.W, a.H, point_image, tile_radius)) break;
            get_rect(point_image, tile_radius, rmin, rmax, a.grid);
            if (!corrected) {
                rmin = {max(rmin.x, legacy_min.x), max(rmin.y, legacy_min.y)};
                rmax = {min(rmax.x, legacy_max.x), min(rmax.y, legacy_max.y)};
                if (rmin.x >= rmax.x || rmin.y >= rmax.y) break;
                point_image = {(rmin.x + rmax.x) * (k3BlockX * 0.5f),
                               (rmin.y + rmax.y) * (k3BlockY * 0.5f)};
                tile_radius = {(int)(rmax.x - rmin.x) * (k3BlockX / 2),
                               (int)(rmax.y - rmin.y) * (k3BlockY / 2)};
            }
            if (corrected && !old_visible) radius_out = max(tile_radius.x, tile_radius.y);
        }
        tile_radius_out = tile_radius;
        depth = p_view.z;
        touched = (int)((rmax.y - rmin.y) * (rmax.x - rmin.x));
        write = true;
    } while (false);

    a.radii[idx] = radius_out;
    a.tiles_touched[idx] = touched;
    if (!write) {
        a.tile_radii[idx] = {0, 0};
        a.points_xy_image[idx] = {0.f, 0.f};
        a.depths[idx] = 0.f;
        if (a.points_xy_center) a.points_xy_center[idx] = {0.f, 0.f};
        a.opacities_out[idx] = 0.f;
        if (a.softness_stride == 3) {
            a.softnesses_out[3 * idx] = 0.f;
            a.softnesses_out[3 * idx + 1] = 0.f;
            a.softnesses_out[3 * idx + 2] = 0.f;
        } else {
            a.softnesses_out[idx] = 0.f;
        }
#pragma unroll
        for (int q = 0; q < 9; ++q) a.transMats[9 * idx + q] = 0.f;
        if (a.normals) {
            a.normals[3 * idx] = 0.f;
            a.normals[3 * idx + 1] = 0.f;
            a.normals[3 * idx + 2] = 0.f;
        }
        return;
    }
    a.tile_radii[idx] = tile_radius_out;
    a.depths[idx] = depth;
    a.points_xy_image[idx] = point_image;
    if (a.points_xy_center) {
        const Cmat<4, 4> w2n = world2ndc_of(a.projmatrix);
        const float v[4] = {p.x, p.y, p.z, 1.0f};
        float clip[4];
        vmat<4, 4>(v, w2n, clip);
        const float inv_w = 1.0f / (clip[3] + 1e-8f);
        const float x_pix = ((float)a.W / 2.0f) * (clip[0] * inv_w) + ((float)a.W - 1.0f) / 2.0f;
        const float y_pix = ((float)a.H / 2.0f) * (clip[1] * inv_w) + ((float)a.H - 1.0f) / 2.0f;
        a.points_xy_center[idx] = {x_pix, y_pix};
    }
    a.opacities_out[idx] = a.opacities[idx];
    if (a.softness_stride == 3) {
        a.softnesses_out[3 * idx] = softness3.x;
        a.softnesses_out[3 * idx + 1] = softness3.y;
        a.softnesses_out[3 * idx + 2] = softness3.z;
    } else {
        a.softnesses_out[idx] = softness3.x;
    }
    float* Tp = a.transMats + 9 * idx;
    Tp[0] = T.m[0][0]; Tp[1] = T.m[0][1]; Tp[2] = T.m[0][2];
    Tp[3] = T.m[1][0]; Tp[4] = T.m[1][1]; Tp[5] = T.m[1][2];
    Tp[6] = T.m[2][0]; Tp[7] = T.m[2][1]; Tp[8] = T.m[2][2];
    if (a.normals) {
        const Cmat<3, 3> R = quat_to_rotmat_wxyz(rot);
        a.normals[3 * idx] = R.m[2][0];
        a.normals[3 * idx + 1] = R.m[2][1];
        a.normals[3 * idx + 2] = R.m[2][2];
    }
}

// (tile << 32 | depth bits) keys and surfel ids for every tile of each
// surfel's rectangle; a warp writes 32 surfels' rectangles cooperatively.
__global__ void __launch_bounds__(256) emit3d_kernel(
    int P, int num_rendered, const float2* __restrict__ points_xy,
    const float* __restrict__ depths, const int* __restrict__ offsets,
    const int* __restrict__ radii, const int2* __restrict__ tile_radii, uint2 grid,
    unsigned long long* __restrict__ keys, int* __restrict__ vals) {
    const int lane = threadIdx.x & 31;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    bool valid = false;
    uint2 rmin = {0, 0}, rmax = {0, 0};
    int off = 0;
    unsigned depth_bits = 0;
    if (idx < P) {
        const int2 tr = tile_radii[idx];
        if (radii[idx] > 0 && tr.x > 0 && tr.y > 0) {
            get_rect(points_xy[idx], tr, rmin, rmax, grid);
            valid = rmax.x > rmin.x && rmax.y > rmin.y;
            off = idx == 0 ? 0 : offsets[idx - 1];
            depth_bits = __float_as_uint(depths[idx]);
        }
    }
    unsigned todo = __ballot_sync(0xffffffffu, valid);
    const int warp_base = idx - lane;
    while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1;
        const unsigned x0 = __shfl_sync(0xffffffffu, rmin.x, j);
        const unsigned y0 = __shfl_sync(0xffffffffu, rmin.y, j);
        const unsigned x1 = __shfl_sync(0xffffffffu, rmax.x, j);
        const unsigned y1 = __shfl_sync(0xffffffffu, rmax.y, j);
        const int base = __shfl_sync(0xffffffffu, off, j);
        const unsigned db = __shfl_sync(0xffffffffu, depth_bits, j);
        const int w = (int)(x1 - x0);
        const int area = w * (int)(y1 - y0);
        for (int e = lane; e < area; e += 32) {
            const int pos = base + e;
            if (pos < 0 || pos >= num_rendered) continue;
            const unsigned ty = y0 + (unsigned)(e / w);
            const unsigned tx = x0 + (unsigned)(e % w);
            keys[pos] = ((unsigned long long)(ty * grid.x + tx) << 32) | db;
            vals[pos] = warp_base + j;
        }
    }
}

// ranges[t] = [first, last + 1) of tile t in the sorted keys; ranges must be
// zeroed beforehand.
__global__ void __launch_bounds__(256) ranges3d_kernel(int L, int num_tiles,
                                                       const unsigned long long* __restrict__ keys,
                                                       uint2* __restrict__ ranges) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= L) return;
    const unsigned cur = (unsigned)(keys[idx] >> 32);
    if (cur >= (unsigned)num_tiles) return;
    if (idx == 0) {
        ranges[cur].x = 0;
    } else {
        const unsigned prev = (unsigned)(keys[idx - 1] >> 32);
        if (cur != prev) {
            if (prev < (unsigned)num_tiles) ranges[prev].y = (unsigned)idx;
            ranges[cur].x = (unsigned)idx;
        }
    }
    if (idx == L - 1) ranges[cur].y = (unsigned)L;
}

}  // namespace hx

using namespace hx;

extern "C" int hx_hexels3d_preprocess(
    int P, const float* means3d, const float* scales, float scale_modifier,
    const float* rotations, const float* opacities, const float* softnesses,
    float softness_default, int softness_stride, const float* viewmatrix,
    const float* projmatrix, const float* campos, int image_width, int image_height,
    int prefilter_edge_on, int conservative_bounds, int32_t* radii, int32_t* tile_radii,
    float* points_xy_image, float* points_xy_center, float* depths, float* transMats,
    int32_t* tiles_touched, float* opacities_out, float* softnesses_out, float* view_dirs,
    float* normals, cudaStream_t stream) {
    HX_REQUIRE(P >= 0, "hexels3d_preprocess: P must be non-negative");
    HX_REQUIRE(image_width > 0 && image_height > 0, "invalid image dimensions");
    HX_REQUIRE(softness_stride == 1 || softness_stride == 3,
               "hexels3d_preprocess: softness_stride must be 1 or 3");
    if (P == 0) return HX_OK;
    HX_REQUIRE(means3d && scales && rotations && opacities && viewmatrix && projmatrix && campos &&
                   radii && tile_radii && points_xy_image && depths && transMats &&
                   tiles_touched && opacities_out && softnesses_out && view_dirs,
               "hexels3d_preprocess: null pointer");
    HX_REQUIRE(!prefilter_edge_on || points_xy_center,
               "hexels3d_preprocess: points_xy_center is required with prefilter_edge_on");
    Prep3DArgs a;
    a.P = P;
    a.means3d = means3d;
    a.scales = (const float2*)scales;
    a.scale_modifier = scale_modifier;
    a.rotations = (const float4*)rotations;
    a.opacities = opacities;
    a.softnesses_in = softnesses;
    a.softness_default = softness_default;
    a.softness_stride = softness_stride;
    a.viewmatrix = viewmatrix;
    a.projmatrix = projmatrix;
    a.campos = campos;
    a.W = image_width;
    a.H = image_height;
    a.prefilter = prefilter_edge_on != 0;
    a.conservative = conservative_bounds != 0;
    a.radii = radii;
    a.tile_radii = (int2*)tile_radii;
    a.points_xy_image = (float2*)points_xy_image;
    a.points_xy_center = (float2*)points_xy_center;
    a.depths = depths;
    a.transMats = transMats;
    a.tiles_touched = tiles_touched;
    a.opacities_out = opacities_out;
    a.softnesses_out = softnesses_out;
    a.view_dirs = view_dirs;
    a.normals = normals;
    a.grid = {(unsigned)ceil_div(image_width, k3BlockX), (unsigned)ceil_div(image_height, k3BlockY)};
    preprocess3d_kernel<<<ceil_div(P, 256), 256, 0, stream>>>(a);
    HX_LAUNCH_CHECK("preprocess3d_kernel");
    return HX_OK;
}

extern "C" size_t hx_hexels3d_bin_workspace_bytes(int num_rendered) {
    const size_t n = num_rendered > 0 ? (size_t)num_rendered : 1;
    return align256(sizeof(unsigned long long) * n) + align256(sizeof(int) * n) +
           sort_workspace_bytes<unsigned long long>((int)n);
}

extern "C" int hx_hexels3d_bin(int P, int num_rendered, int image_width, int image_height,
                               const float* points_xy_image, const float* depths,
                               const int32_t* offsets, const int32_t* radii,
                               const int32_t* tile_radii, int64_t* keys_sorted,
                               int32_t* point_list, int32_t* ranges, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream) {
    HX_REQUIRE(P >= 0 && num_rendered >= 0, "hexels3d_bin: bad sizes");
    const uint2 grid = {(unsigned)ceil_div(image_width, k3BlockX),
                        (unsigned)ceil_div(image_height, k3BlockY)};
    const int num_tiles = (int)(grid.x * grid.y);
    HX_REQUIRE(ranges, "hexels3d_bin: null ranges");
    HX_CUDA_TRY(cudaMemsetAsync(ranges, 0, sizeof(uint2) * (size_t)num_tiles, stream));
    if (P == 0 || num_rendered == 0) return HX_OK;
    HX_REQUIRE(points_xy_image && depths && offsets && radii && tile_radii && keys_sorted &&
                   point_list,
               "hexels3d_bin: null pointer");
    const size_t need = hx_hexels3d_bin_workspace_bytes(num_rendered);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE, "hexels3d_bin: workspace of %zu bytes needed", need);
    char* p = (char*)workspace;
    unsigned long long* keys = (unsigned long long*)p;
    p += align256(sizeof(unsigned long long) * (size_t)num_rendered);
    int* vals = (int*)p;
    p += align256(sizeof(int) * (size_t)num_rendered);
    emit3d_kernel<<<ceil_div(P, 256), 256, 0, stream>>>(
        P, num_rendered, (const float2*)points_xy_image, depths, offsets, radii,
        (const int2*)tile_radii, grid, keys, vals);
    HX_LAUNCH_CHECK("emit3d_kernel");
    int bits = 0;
    while (bits < 31 && (1u << bits) <= (unsigned)num_tiles) ++bits;
    int rc = sort_pairs<unsigned long long>(keys, vals, (unsigned long long*)keys_sorted,
                                            point_list, num_rendered, 0, 32 + bits, p,
                                            sort_workspace_bytes<unsigned long long>(num_rendered),
                                            stream);
    if (rc != HX_OK) return rc;
    ranges3d_kernel<<<ceil_div(num_rendered, 256), 256, 0, stream>>>(
        num_rendered, num_tiles, (const unsigned long long*)keys_sorted, (uint2*)ranges);
    HX_LAUNCH_CHECK("ranges3d_kernel");
    return HX_OK;
}

// ---------------------------------------------------------------------------
// Depth-ordered binning.  Sorting the surfels once by depth (32-bit keys,
// stable) and emitting their tiles in that order leaves only the tile index
// to sort per intersection: bits [0, bits(tiles)) instead of
// [0, 32 + bits(tiles)).  Within a tile the entries end up ordered by depth
// bits, then surfel index -- the order of the stable sort of
// (tile << 32 | depth bits) over surfel-major emission.
// ---------------------------------------------------------------------------
namespace hx {

__global__ void __launch_bounds__(256) iota_kernel(int n, int* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = i;
}

__global__ void __launch_bounds__(256) gather_counts_kernel(int n, const int* __restrict__ order,
                                                            const int* __restrict__ counts,
                                                            int* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = counts[min(max(order[i], 0), n - 1)];
}

// Tile keys and surfel ids for every tile of each surfel's rectangle, surfels
// in depth order.  A warp takes 32 consecutive surfels, whose entries are one
// contiguous run of the output: it scans their tile counts and then writes
// the run 32 consecutive entries at a time, each lane finding the surfel
// that owns its entry by a binary search over the warp's prefix sums.  With
// several views (P = views x P_view entries, view-major), entry order[i] =
// view * P_view + surfel, the key is view * tiles + tile and the value the
// surfel index within its view.
__global__ void __launch_bounds__(256) emit3d_ordered_kernel(
    int P, int num_rendered, const int* __restrict__ order, const float2* __restrict__ points_xy,
    const int* __restrict__ offsets, const int* __restrict__ radii,
    const int2* __restrict__ tile_radii, uint2 grid, unsigned* __restrict__ keys,
    int* __restrict__ vals, int P_view) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned tiles = grid.x * grid.y;
    int cnt = 0, x0 = 0, y0 = 0, w = 1, sid = 0, off = 0, lid = 0;
    unsigned key_base = 0;
    if (i < P) {
        sid = min(max(order[i], 0), P - 1);
        const int2 tr = tile_radii[sid];
        if (radii[sid] > 0 && tr.x > 0 && tr.y > 0) {
            uint2 rmin, rmax;
            get_rect(points_xy[sid], tr, rmin, rmax, grid);
            if (rmax.x > rmin.x && rmax.y > rmin.y) {
                x0 = (int)rmin.x;
                y0 = (int)rmin.y;
                w = (int)(rmax.x - rmin.x);
                cnt = w * (int)(rmax.y - rmin.y);
            }
        }
        off = i == 0 ? 0 : offsets[i - 1];
        const int view = sid / P_view;
        key_base = (unsigned)view * tiles;
        lid = sid - view * P_view;
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(full, incl, o);
        if (lane >= o) incl += t;
    }
    const int excl = incl - cnt;
    const int total = __shfl_sync(full, incl, 31);
    const int base = __shfl_sync(full, off, 0);  // first entry of the warp's run
    for (int e0 = 0; e0 < total; e0 += 32) {
        const int e = e0 + lane;
        // owner: the last lane whose exclusive prefix is <= e
        int j = 0;
#pragma unroll
        for (int step = 16; step >= 1; step >>= 1) {
            const int ex = __shfl_sync(full, excl, j + step);
            if (ex <= e) j += step;
        }
        const int jx0 = __shfl_sync(full, x0, j);
        const int jy0 = __shfl_sync(full, y0, j);
        const int jw = __shfl_sync(full, w, j);
        const int jid = __shfl_sync(full, lid, j);
        const int jex = __shfl_sync(full, excl, j);
        const unsigned jkb = __shfl_sync(full, key_base, j);
        const int pos = base + e;
        if (e < total && pos >= 0 && pos < num_rendered) {
            const int local = e - jex;
            const unsigned ty = (unsigned)(jy0 + local / jw);
            const unsigned tx = (unsigned)(jx0 + local % jw);
            keys[pos] = jkb + ty * grid.x + tx;
            vals[pos] = jid;
        }
    }
}

// ranges[t] = [first, last + 1) of tile t in the sorted tile keys; ranges
// must be zeroed beforehand.
__global__ void __launch_bounds__(256) ranges3d_u32_kernel(int L, int num_tiles,
                                                           const unsigned* __restrict__ keys,
                                                           uint2* __restrict__ ranges) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= L) return;
    const unsigned cur = keys[idx];
    if (cur >= (unsigned)num_tiles) return;
    if (idx == 0) {
        ranges[cur].x = 0;
    } else {
        const unsigned prev = keys[idx - 1];
        if (cur != prev) {
            if (prev < (unsigned)num_tiles) ranges[prev].y = (unsigned)idx;
            ranges[cur].x = (unsigned)idx;
        }
    }
    if (idx == L - 1) ranges[cur].y = (unsigned)L;
}

// The reference's 64-bit keys of the sorted list, (tile << 32) | depth bits.
__global__ void __launch_bounds__(256) full_keys_kernel(int L, int P,
                                                        const unsigned* __restrict__ tiles,
                                                        const int* __restrict__ ids,
                                                        const float* __restrict__ depths,
                                                        unsigned long long* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L) return;
    const int id = min(max(ids[i], 0), P - 1);
    out[i] = ((unsigned long long)tiles[i] << 32) | __float_as_uint(depths[id]);
}

}  // namespace hx

extern "C" size_t hx_hexels3d_depth_order_workspace_bytes(int P) {
    const size_t n = P > 0 ? (size_t)P : 1;
    return align256(sizeof(unsigned) * n) + align256(sizeof(int) * n) +
           align256(sizeof(int) * n) + hx_scan_workspace_bytes((int)n) +
           sort_workspace_bytes<uint32_t>((int)n);
}

extern "C" int hx_hexels3d_depth_order(int P, const float* depths, const int32_t* tiles_touched,
                                       int32_t* order, int32_t* offsets, int64_t* total_out,
                                       void* workspace, size_t workspace_bytes,
                                       cudaStream_t stream) {
    HX_REQUIRE(P >= 0, "hexels3d_depth_order: bad P");
    if (P == 0) {
        if (total_out) HX_CUDA_TRY(cudaMemsetAsync(total_out, 0, sizeof(int64_t), stream));
        return HX_OK;
    }
    HX_REQUIRE(depths && tiles_touched && order && offsets, "hexels3d_depth_order: null pointer");
    const size_t need = hx_hexels3d_depth_order_workspace_bytes(P);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE, "hexels3d_depth_order: workspace of %zu bytes needed",
                         need);
    char* p = (char*)workspace;
    unsigned* keys_sorted = (unsigned*)p;
    p += align256(sizeof(unsigned) * (size_t)P);
    int* ids = (int*)p;
    p += align256(sizeof(int) * (size_t)P);
    int* counts = (int*)p;
    p += align256(sizeof(int) * (size_t)P);
    void* scan_ws = p;
    const size_t scan_bytes = hx_scan_workspace_bytes(P);
    p += scan_bytes;
    iota_kernel<<<ceil_div(P, 256), 256, 0, stream>>>(P, ids);
    HX_LAUNCH_CHECK("iota_kernel");
    // depths are >= the near plane (> 0) for every surfel that touches a
    // tile, so their bit patterns order like the values
    int rc = sort_pairs<uint32_t>((const uint32_t*)depths, ids, keys_sorted, order, P, 0, 32, p,
                                  sort_workspace_bytes<uint32_t>(P), stream);
    if (rc != HX_OK) return rc;
    gather_counts_kernel<<<ceil_div(P, 256), 256, 0, stream>>>(P, order, tiles_touched, counts);
    HX_LAUNCH_CHECK("gather_counts_kernel");
    return hx_inclusive_scan_i32(counts, offsets, P, total_out, scan_ws, scan_bytes, stream);
}

extern "C" size_t hx_hexels3d_bin_ordered_workspace_bytes(int num_rendered) {
    const size_t n = num_rendered > 0 ? (size_t)num_rendered : 1;
    return align256(sizeof(unsigned) * n) * 2 + align256(sizeof(int) * n) +
           sort_workspace_bytes<uint32_t>((int)n);
}

extern "C" int hx_hexels3d_bin_ordered(int P, int num_rendered, int image_width,
                                       int image_height, const float* points_xy_image,
                                       const int32_t* order, const int32_t* offsets,
                                       const int32_t* radii, const int32_t* tile_radii,
                                       const float* depths, int64_t* keys_sorted,
                                       int32_t* point_list, int32_t* ranges, void* workspace,
                                       size_t workspace_bytes, cudaStream_t stream) {
    HX_REQUIRE(P >= 0 && num_rendered >= 0, "hexels3d_bin_ordered: bad sizes");
    HX_REQUIRE(image_width > 0 && image_height > 0, "invalid image dimensions");
    const uint2 grid = {(unsigned)ceil_div(image_width, k3BlockX),
                        (unsigned)ceil_div(image_height, k3BlockY)};
    const int num_tiles = (int)(grid.x * grid.y);
    HX_REQUIRE(ranges, "hexels3d_bin_ordered: null ranges");
    HX_CUDA_TRY(cudaMemsetAsync(ranges, 0, sizeof(uint2) * (size_t)num_tiles, stream));
    if (P == 0 || num_rendered == 0) return HX_OK;
    HX_REQUIRE(points_xy_image && order && offsets && radii && tile_radii && point_list,
               "hexels3d_bin_ordered: null pointer");
    HX_REQUIRE(!keys_sorted || depths, "hexels3d_bin_ordered: keys_sorted needs depths");
    const size_t need = hx_hexels3d_bin_ordered_workspace_bytes(num_rendered);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE, "hexels3d_bin_ordered: workspace of %zu bytes needed",
                         need);
    char* p = (char*)workspace;
    unsigned* keys = (unsigned*)p;
    p += align256(sizeof(unsigned) * (size_t)num_rendered);
    unsigned* keys_out = (unsigned*)p;
    p += align256(sizeof(unsigned) * (size_t)num_rendered);
    int* vals = (int*)p;
    p += align256(sizeof(int) * (size_t)num_rendered);
    emit3d_ordered_kernel<<<ceil_div(P, 256), 256, 0, stream>>>(
        P, num_rendered, order, (const float2*)points_xy_image, offsets, radii,
        (const int2*)tile_radii, grid, keys, vals, P);
    HX_LAUNCH_CHECK("emit3d_ordered_kernel");
    int rc = sort_pairs<uint32_t>(keys, vals, keys_out, point_list, num_rendered, 0,
                                  tile_bits(num_tiles), p,
                                  sort_workspace_bytes<uint32_t>(num_rendered), stream);
    if (rc != HX_OK) return rc;
    ranges3d_u32_kernel<<<ceil_div(num_rendered, 256), 256, 0, stream>>>(
        num_rendered, num_tiles, keys_out, (uint2*)ranges);
    HX_LAUNCH_CHECK("ranges3d_u32_kernel");
    if (keys_sorted) {
        full_keys_kernel<<<ceil_div(num_rendered, 256), 256, 0, stream>>>(
            num_rendered, P, keys_out, point_list, depths, (unsigned long long*)keys_sorted);
        HX_LAUNCH_CHECK("full_keys_kernel");
    }
    return HX_OK;
}

// ---------------------------------------------------------------------------
// Several views of one scene binned together (view-major (views, P) arrays).
// ---------------------------------------------------------------------------
namespace hx {
namespace {

// (view << 32) | depth bits of each (view, surfel) entry, and its index.
__global__ void __launch_bounds__(256) view_depth_keys_kernel(int n, int P_view,
                                                              const float* __restrict__ depths,
                                                              unsigned long long* __restrict__ keys,
                                                              int* __restrict__ ids) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    keys[i] = ((unsigned long long)(i / P_view) << 32) | __float_as_uint(depths[i]);
    ids[i] = i;
}

}  // namespace
}  // namespace hx

extern "C" size_t hx_hexels3d_depth_order_views_workspace_bytes(int views, int P) {
    const size_t n = (views > 0 && P > 0) ? (size_t)views * P : 1;
    return 2 * align256(sizeof(unsigned long long) * n) + align256(sizeof(int) * n) +
           align256(sizeof(int) * n) + hx_scan_workspace_bytes((int)n) +
           sort_workspace_bytes<unsigned long long>((int)n);
}

extern "C" int hx_hexels3d_depth_order_views(int views, int P, const float* depths,
                                             const int32_t* tiles_touched, int32_t* order,
                                             int32_t* offsets, int64_t* total_out,
                                             void* workspace, size_t workspace_bytes,
                                             cudaStream_t stream) {
    HX_REQUIRE(views >= 1 && P >= 0, "hexels3d_depth_order_views: bad sizes");
    HX_REQUIRE((long long)views * P <= 0x7fffffffLL,
               "hexels3d_depth_order_views: views x P overflows int32");
    const int n = views * P;
    if (n == 0) {
        if (total_out) HX_CUDA_TRY(cudaMemsetAsync(total_out, 0, sizeof(int64_t), stream));
        return HX_OK;
    }
    HX_REQUIRE(depths && tiles_touched && order && offsets,
               "hexels3d_depth_order_views: null pointer");
    const size_t need = hx_hexels3d_depth_order_views_workspace_bytes(views, P);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE,
                         "hexels3d_depth_order_views: workspace of %zu bytes needed", need);
    char* p = (char*)workspace;
    unsigned long long* keys = (unsigned long long*)p;
    p += align256(sizeof(unsigned long long) * (size_t)n);
    unsigned long long* keys_sorted = (unsigned long long*)p;
    p += align256(sizeof(unsigned long long) * (size_t)n);
    int* ids = (int*)p;
    p += align256(sizeof(int) * (size_t)n);
    int* counts = (int*)p;
    p += align256(sizeof(int) * (size_t)n);
    void* scan_ws = p;
    const size_t scan_bytes = hx_scan_workspace_bytes(n);
    p += scan_bytes;
    view_depth_keys_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(n, P, depths, keys, ids);
    HX_LAUNCH_CHECK("view_depth_keys_kernel");
    // per view, depths are >= the near plane (> 0) for every surfel that
    // touches a tile, so their bit patterns order like the values; the view
    // in the high bits keeps each view's entries contiguous and in its own
    // stable depth order
    int rc = sort_pairs<unsigned long long>(keys, ids, keys_sorted, order, n, 0,
                                            32 + tile_bits(views), p,
                                            sort_workspace_bytes<unsigned long long>(n), stream);
    if (rc != HX_OK) return rc;
    gather_counts_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(n, order, tiles_touched, counts);
    HX_LAUNCH_CHECK("gather_counts_kernel");
    return hx_inclusive_scan_i32(counts, offsets, n, total_out, scan_ws, scan_bytes, stream);
}

extern "C" size_t hx_hexels3d_bin_views_workspace_bytes(int num_rendered) {
    return hx_hexels3d_bin_ordered_workspace_bytes(num_rendered);
}

extern "C" int hx_hexels3d_bin_views(int views, int P, int num_rendered, int image_width,
                                     int image_height, const float* points_xy_image,
                                     const int32_t* order, const int32_t* offsets,
                                     const int32_t* radii, const int32_t* tile_radii,
                                     int32_t* point_list, int32_t* ranges, void* workspace,
                                     size_t workspace_bytes, cudaStream_t stream) {
    HX_REQUIRE(views >= 1 && P >= 0 && num_rendered >= 0, "hexels3d_bin_views: bad sizes");
    HX_REQUIRE(image_width > 0 && image_height > 0, "invalid image dimensions");
    HX_REQUIRE((long long)views * P <= 0x7fffffffLL, "hexels3d_bin_views: views x P overflows");
    const uint2 grid = {(unsigned)ceil_div(image_width, k3BlockX),
                        (unsigned)ceil_div(image_height, k3BlockY)};
    const long long all_tiles = (long long)views * grid.x * grid.y;
    HX_REQUIRE(all_tiles <= 0x7fffffffLL, "hexels3d_bin_views: views x tiles overflows");
    const int num_tiles = (int)all_tiles;
    HX_REQUIRE(ranges, "hexels3d_bin_views: null ranges");
    HX_CUDA_TRY(cudaMemsetAsync(ranges, 0, sizeof(uint2) * (size_t)num_tiles, stream));
    const int n = views * P;
    if (n == 0 || num_rendered == 0) return HX_OK;
    HX_REQUIRE(points_xy_image && order && offsets && radii && tile_radii && point_list,
               "hexels3d_bin_views: null pointer");
    const size_t need = hx_hexels3d_bin_views_workspace_bytes(num_rendered);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE, "hexels3d_bin_views: workspace of %zu bytes needed",
                         need);
    char* p = (char*)workspace;
    unsigned* keys = (unsigned*)p;
    p += align256(sizeof(unsigned) * (size_t)num_rendered);
    unsigned* keys_out = (unsigned*)p;
    p += align256(sizeof(unsigned) * (size_t)num_rendered);
    int* vals = (int*)p;
    p += align256(sizeof(int) * (size_t)num_rendered);
    emit3d_ordered_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(
        n, num_rendered, order, (const float2*)points_xy_image, offsets, radii,
        (const int2*)tile_radii, grid, keys, vals, P);
    HX_LAUNCH_CHECK("emit3d_ordered_kernel");
    int rc = sort_pairs<uint32_t>(keys, vals, keys_out, point_list, num_rendered, 0,
                                  tile_bits(num_tiles), p,
                                  sort_workspace_bytes<uint32_t>(num_rendered), stream);
    if (rc != HX_OK) return rc;
    ranges3d_u32_kernel<<<ceil_div(num_rendered, 256), 256, 0, stream>>>(
        num_rendered, num_tiles, keys_out, (uint2*)ranges);
    HX_LAUNCH_CHECK("ranges3d_u32_kernel");
    return HX_OK;
}
