// S8 forward: front-to-back alpha compositing of hexagon-SDF surfels, one
// 16x16 tile per CTA (reference gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:
// 610-1011).  Per-pixel arithmetic is the reference's, in its order.
//
// Schedule changes:
//   * per-surfel terms that do not depend on the pixel are computed once while
//     staging a batch: the linear view-dependent colour term
//     (view_dir . view_grads, added to the pixel colour in the same position
//     of the sum as in the reference) and the viewer-facing normal;
//   * the staged record is a packed struct (one 16-byte aligned row per
//     surfel) instead of sixteen separate shared arrays;
//   * with surface outputs the per-pixel state the backward needs (surface
//     transmittance, last index, distortion moments, median index) is saved,
//     so the backward never re-walks or re-bins.
#include "hx_hexmath3d.cuh"

namespace hx {

template <bool SURF, bool PREFILTER, bool OWNER>
__global__ void __launch_bounds__(256) render3d_fwd_kernel(const Render3DArgs a) {
    __shared__ Surfel3D s_prim[k3BlockSize];
    __shared__ float s_contrib[k3BlockSize];

    const int W = a.W, H = a.H;
    const unsigned hblocks = (W + k3BlockX - 1) / k3BlockX;
    const int tr = threadIdx.y * k3BlockX + threadIdx.x;
    const int2 lp = tile_pixel(tr);
    const unsigned px_i = blockIdx.x * k3BlockX + lp.x;
    const unsigned py_i = blockIdx.y * k3BlockY + lp.y;
    const unsigned pix_id = (unsigned)(W * (int)py_i + (int)px_i);
    // this warp's 8x4 pixel block
    const int wx0 = (int)(blockIdx.x * k3BlockX) + (((tr >> 5) & 1) << 3);
    const int wy0 = (int)(blockIdx.y * k3BlockY) + ((tr >> 6) << 2);
    const float px = (float)px_i;
    const float py = (float)py_i;
    const bool inside = px_i < (unsigned)W && py_i < (unsigned)H;
    bool done_color = !inside;
    bool done_surf = SURF ? !inside : true;
    bool done = SURF ? (done_color && done_surf) : done_color;

    uint2 range = a.ranges[blockIdx.y * hblocks + blockIdx.x];
    range.y = min(range.y, (unsigned)a.num_rendered);
    range.x = min(range.x, range.y);
    const int rounds = (int)((range.y - range.x + k3BlockSize - 1) / k3BlockSize);
    int to_do = (int)(range.y - range.x);

    int n_visited = 0;
    int n_blended = 0;
    float T = 1.0f;
    float C0 = 0.f, C1 = 0.f, C2 = 0.f;
    float overdraw = 0.f, overdraw_hits = 0.f;
    float T_surf = 1.0f, D_surf = 0.f, median_depth = 0.f, M1 = 0.f, M2 = 0.f, distortion = 0.f;
    float3 N_surf = {0.f, 0.f, 0.f};
    int n_visited_surf = 0;
    int median_idx = -1;
    long long owner_id = -1;
    float owner_weight = 0.f, owner_sdf = 0.f, owner_depth = 0.f;
    float2 owner_uv = {0.f, 0.f};

    for (int i = 0; i < rounds; ++i, to_do -= k3BlockSize) {
        if (__syncthreads_count(done) == k3BlockSize) break;
        const int progress = i * k3BlockSize + tr;
        s_contrib[tr] = 0.f;
        if ((int)range.x + progress < (int)range.y) {
            int g = a.point_list[range.x + progress];
            g = min(max(g, 0), a.P - 1);
            Surfel3D& s = s_prim[tr];
            s.id = g;
            const float* Tm = a.transMats + 9 * g;
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                s.tu[q] = Tm[q];
                s.tv[q] = Tm[3 + q];
                s.tw[q] = Tm[6 + q];
            }
            s.opacity = a.opacities[g];
            if (a.softness_stride == 3) {
                s.s0 = a.softnesses[3 * g];
                s.s1 = a.softnesses[3 * g + 1];
                s.s2 = a.softnesses[3 * g + 2];
            } else {
                s.s0 = s.s1 = s.s2 = a.softnesses[g];
            }
#pragma unroll
            for (int q = 0; q < 3; ++q) s.cb[q] = a.colors[3 * g + q];
            if (a.color_model >= kColorLinear) {
#pragma unroll
                for (int q = 0; q < 3; ++q) {
                    s.gu[q] = a.color_grads[6 * g + q];
                    s.gv[q] = a.color_grads[6 * g + 3 + q];
                }
            } else {
#pragma unroll
                for (int q = 0; q < 3; ++q) s.gu[q] = s.gv[q] = 0.f;
            }
            if (a.use_view_grads) {
                const float* vd = a.view_dirs + 3 * g;
                const float* vg = a.view_grads + 9 * g;
                s.cv[0] = vd[0] * vg[0] + vd[1] * vg[1] + vd[2] * vg[2];
                s.cv[1] = vd[0] * vg[3] + vd[1] * vg[4] + vd[2] * vg[5];
                s.cv[2] = vd[0] * vg[6] + vd[1] * vg[7] + vd[2] * vg[8];
            } else {
                s.cv[0] = s.cv[1] = s.cv[2] = 0.f;
            }
            if (SURF) {
                float3 n = {a.normals[3 * g], a.normals[3 * g + 1], a.normals[3 * g + 2]};
                const float sg = normal_sign(n, a.view_dirs + 3 * g);
                s.n[0] = sg * n.x;
                s.n[1] = sg * n.y;
                s.n[2] = sg * n.z;
                s.nsign = sg;
            } else {
                s.n[0] = s.n[1] = s.n[2] = 0.f;
                s.nsign = 1.f;
            }
            if (PREFILTER) {
                s.q.ctr = a.points_xy_center[g];
            } else {
                s.q.box = surfel_pixel_box(s, W, H);
            }
        }
        __syncthreads();

        const int batch_size = min(k3BlockSize, to_do);
        for (int j = 0; !done && j < batch_size; ++j) {
            const Surfel3D& s = s_prim[j];
            // every pixel of a warp block the surfel's box misses has alpha < 1/255
            if (!PREFILTER && box_misses(s.q.box, wx0, wy0, wx0 + 7, wy0 + 3)) continue;
            const int g_id = s.id;
            const bool is_base = g_id < a.overdraw_base;
            if (SURF && done_color && !is_base) continue;
            const float3 Tu = {s.tu[0], s.tu[1], s.tu[2]};
            const float3 Tv = {s.tv[0], s.tv[1], s.tv[2]};
            const float3 Tw = {s.tw[0], s.tw[1], s.tw[2]};
            const float3 k = {px * Tw.x - Tu.x, px * Tw.y - Tu.y, px * Tw.z - Tu.z};
            const float3 l = {py * Tw.x - Tv.x, py * Tw.y - Tv.y, py * Tw.z - Tv.z};
            const float3 p = cross3(k, l);
            if (p.z == 0.0f) continue;
            const float sx = p.x / p.z;
            const float sy = p.y / p.z;
            const float depth_sdf = (sx * Tw.x + sy * Tw.y) + Tw.z;
            if (depth_sdf < k3NearPlane) continue;
            int edge;
            const float dist = hex_sdf3(sx, sy, edge);
            const float soft = (edge == 0) ? s.s0 : ((edge == 1) ? s.s1 : s.s2);
            const float boundary = sigmoid_neg(dist, soft);
            const float alpha_raw_sdf = s.opacity * boundary;
            const float alpha_sdf = fminf(alpha_raw_sdf, 0.99f);
            float alpha = alpha_sdf;
            bool use_filter = false;
            if (PREFILTER) {
                const float dx = px - s.q.ctr.x;
                const float dy = py - s.q.ctr.y;
                const float G = __expf(-0.5f * k3FilterInvSquare * (dx * dx + dy * dy));
                const float alpha_filter = fminf(s.opacity * G, 0.99f);
                use_filter = alpha_filter > alpha_sdf;
                alpha = use_filter ? alpha_filter : alpha_sdf;
            }
            if (alpha < 1.0f / 255.0f) continue;
            const float depth = use_filter ? Tw.z : depth_sdf;

            if (!done_color) {
                if (is_base && alpha_sdf >= 1.0f / 255.0f) {
                    if (a.overdraw) overdraw += alpha_raw_sdf;
                    if (a.overdraw_hits) overdraw_hits += 1.0f;
                }
                const float test_T = T * (1.f - alpha);
                if (test_T < 0.0001f) {
                    done_color = true;
                } else {
                    const float w = alpha * T;
                    const float u = use_filter ? 0.f : sx;
                    const float v = use_filter ? 0.f : sy;
                    if (OWNER) {
                        if (w > owner_weight) {
                            owner_id = g_id;
                            owner_weight = w;
                            owner_uv = {sx, sy};
                            owner_sdf = dist;
                            owner_depth = depth;
                        }
                    }
                    float cx = s.cb[0], cy = s.cb[1], cz = s.cb[2];
                    if (a.color_model >= kColorLinear) {
                        cx += u * s.gu[0] + v * s.gv[0];
                        cy += u * s.gu[1] + v * s.gv[1];
                        cz += u * s.gu[2] + v * s.gv[2];
                    }
                    if (a.color_model == kColorQuadratic || a.color_model == kColorQuadBounded) {
                        const float* cq = a.color_quads + 9 * g_id;
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
                        const float* vd = a.view_dirs + 3 * g_id;
                        const float* nr = a.normals + 3 * g_id;
                        const float cos_nv =
                            fmaxf(-(nr[0] * vd[0] + nr[1] * vd[1] + nr[2] * vd[2]), 0.f);
                        const float log_s = a.specular_log_s[g_id];
                        const float s_exp = __expf(fminf(fmaxf(log_s, 0.f), 5.0f));
                        const float spec = (cos_nv > 0.f) ? __powf(cos_nv, s_exp) : 0.f;
                        cx += a.specular_ks[3 * g_id] * spec;
                        cy += a.specular_ks[3 * g_id + 1] * spec;
                        cz += a.specular_ks[3 * g_id + 2] * spec;
                    }
                    C0 += cx * w;
                    C1 += cy * w;
                    C2 += cz * w;
                    T = test_T;
                    n_visited = i * k3BlockSize + j + 1;
                    ++n_blended;
                    if (a.contrib) atomicAdd(&s_contrib[j], w);
                }
            }
            if (SURF) {
                if (!done_surf && is_base) {
                    const float test_T_surf = T_surf * (1.f - alpha);
                    if (test_T_surf < 0.0001f) {
                        done_surf = true;
                    } else {
                        if (a.median && T_surf > 0.5f) {
                            median_depth = depth;
                            median_idx = i * k3BlockSize + j;
                        }
                        const float w_surf = alpha * T_surf;
                        const float m = k3FarPlane / (k3FarPlane - k3NearPlane) *
                                        (1.0f - k3NearPlane / depth);
                        const float acc_alpha = 1.0f - T_surf;
                        distortion += (m * m * acc_alpha + M2 - 2.0f * m * M1) * w_surf;
                        M1 += m * w_surf;
                        M2 += m * m * w_surf;
                        D_surf += depth * w_surf;
                        N_surf.x += s.n[0] * w_surf;
                        N_surf.y += s.n[1] * w_surf;
                        N_surf.z += s.n[2] * w_surf;
                        T_surf = test_T_surf;
                        n_visited_surf = i * k3BlockSize + j + 1;
                    }
                }
                done = done_color && done_surf;
            } else {
                done = done_color;
            }
        }
        if (a.contrib) {
            __syncthreads();
            if (tr < batch_size && s_contrib[tr] != 0.f) atomicAdd(&a.contrib[s_prim[tr].id], s_contrib[tr]);
        }
    }

    if (!inside) return;
    const int HW = H * W;
    if (a.final_T) {
        a.final_T[pix_id] = T;
        a.last_index[pix_id] = n_visited;
    }
    if (a.contrib_count) a.contrib_count[pix_id] = n_blended;
    // With nothing binned every tile range is empty and the pixel is the
    // background, as in the reference (hexels3d_forward.cu:3300-3470).
    a.out_color[pix_id] = C0 + T * a.bg[0];
    a.out_color[HW + pix_id] = C1 + T * a.bg[1];
    a.out_color[2 * HW + pix_id] = C2 + T * a.bg[2];
    if (a.overdraw) a.overdraw[pix_id] = overdraw;
    if (a.overdraw_hits) a.overdraw_hits[pix_id] = overdraw_hits;
    if (SURF) {
        a.out_depth[pix_id] = D_surf;
        a.out_alpha[pix_id] = 1.0f - T_surf;
        a.out_surface[pix_id] = N_surf.x;
        a.out_surface[HW + pix_id] = N_surf.y;
        a.out_surface[2 * HW + pix_id] = N_surf.z;
        a.out_surface[3 * HW + pix_id] = distortion;
        if (a.median) a.out_surface[4 * HW + pix_id] = median_depth;
        if (a.final_T_surf) {
            a.final_T_surf[pix_id] = T_surf;
            a.last_index_surf[pix_id] = n_visited_surf;
            a.m1_surf[pix_id] = M1;
            a.m2_surf[pix_id] = M2;
            a.median_index[pix_id] = median_idx;
        }
    }
    if (OWNER) {
        a.owner_id[pix_id] = owner_id;
        a.owner_weight[pix_id] = owner_weight;
        a.owner_uv[pix_id] = owner_uv.x;
        a.owner_uv[HW + pix_id] = owner_uv.y;
        a.owner_sdf[pix_id] = owner_sdf;
        a.owner_depth[pix_id] = owner_depth;
        a.total_alpha[pix_id] = 1.0f - T;
    }
}

}  // namespace hx

using namespace hx;

namespace {

template <bool SURF, bool PREFILTER, bool OWNER>
int launch_render(const Render3DArgs& a, cudaStream_t stream) {
    dim3 grid(ceil_div(a.W, k3BlockX), ceil_div(a.H, k3BlockY)), block(k3BlockX, k3BlockY);
    render3d_fwd_kernel<SURF, PREFILTER, OWNER><<<grid, block, 0, stream>>>(a);
    HX_LAUNCH_CHECK("render3d_fwd_kernel");
    return HX_OK;
}

}  // namespace

extern "C" int hx_hexels3d_render_forward(
    int P, int num_rendered, const int32_t* ranges, const int32_t* point_list,
    const float* points_xy_center, int image_width, int image_height, const float* colors,
    const float* color_grads, const float* color_quads, const float* view_grads,
    const float* specular_ks, const float* specular_log_s, const float* view_dirs,
    const float* transMats, const float* opacities, const float* softnesses,
    int softness_stride, const float* background, const float* normals, int overdraw_base_count,
    int color_model, int view_model, int use_view_grads, int return_median_depth,
    float* out_color, float* contrib, float* overdraw, float* overdraw_hits, float* out_depth,
    float* out_alpha, float* out_surface, int64_t* owner_id, float* owner_weight,
    float* owner_uv, float* owner_sdf, float* owner_depth, float* total_alpha, float* final_T,
    int32_t* last_index, float* final_T_surf, int32_t* last_index_surf, float* m1_surf,
    float* m2_surf, int32_t* median_index, int32_t* contrib_count, cudaStream_t stream) {
    HX_REQUIRE(image_width > 0 && image_height > 0, "invalid image dimensions");
    HX_REQUIRE(color_model >= 0 && color_model <= 3, "color_model must be 0..3");
    HX_REQUIRE(view_model >= 0 && view_model <= 2, "view_model must be 0..2");
    HX_REQUIRE(softness_stride == 1 || softness_stride == 3, "softness_stride must be 1 or 3");
    HX_REQUIRE(ranges && out_color && background, "hexels3d_render_forward: null pointer");
    const bool surf = out_depth != nullptr;
    const bool owner = owner_id != nullptr;
    const bool prefilter = points_xy_center != nullptr;
    HX_REQUIRE(!surf || (out_alpha && out_surface && normals),
               "surface outputs need out_alpha, out_surface and normals");
    HX_REQUIRE(!owner || (owner_weight && owner_uv && owner_sdf && owner_depth && total_alpha),
               "owner outputs must be given together");
    HX_REQUIRE(!(surf && owner), "surface and owner outputs are separate passes");
    HX_REQUIRE(!(final_T != nullptr) || last_index != nullptr, "final_T needs last_index");
    HX_REQUIRE(num_rendered == 0 || (point_list && transMats && opacities && softnesses &&
                                     colors && view_dirs && P > 0),
               "hexels3d_render_forward: null pointer");
    HX_REQUIRE(color_model < 1 || color_grads, "color_grads required for color_model >= 1");
    HX_REQUIRE(color_model < 2 || color_quads, "color_quads required for quadratic models");
    HX_REQUIRE(!use_view_grads || view_grads, "view_grads required with use_view_grads");
    HX_REQUIRE(view_model != 2 || (specular_ks && specular_log_s && normals),
               "lobe view model needs specular_ks, specular_log_s and normals");
    Render3DArgs a = {};
    a.ranges = (const uint2*)ranges;
    a.point_list = point_list;
    a.num_rendered = num_rendered;
    a.P = P;
    a.points_xy_center = (const float2*)points_xy_center;
    a.W = image_width;
    a.H = image_height;
    a.colors = colors;
    a.color_grads = color_grads;
    a.color_quads = color_quads;
    a.view_grads = view_grads;
    a.specular_ks = specular_ks;
    a.specular_log_s = specular_log_s;
    a.view_dirs = view_dirs;
    a.transMats = transMats;
    a.opacities = opacities;
    a.softnesses = softnesses;
    a.softness_stride = softness_stride;
    a.bg = background;
    a.normals = normals;
    a.overdraw_base = (overdraw_base_count <= 0 || overdraw_base_count > P) ? P : overdraw_base_count;
    a.color_model = color_model;
    a.view_model = view_model;
    a.use_view_grads = use_view_grads != 0;
    a.median = return_median_depth != 0;
    a.out_color = out_color;
    a.contrib = contrib;
    a.overdraw = overdraw;
    a.overdraw_hits = overdraw_hits;
    a.out_depth = out_depth;
    a.out_alpha = out_alpha;
    a.out_surface = out_surface;
    a.owner_id = (long long*)owner_id;
    a.owner_weight = owner_weight;
    a.owner_uv = owner_uv;
    a.owner_sdf = owner_sdf;
    a.owner_depth = owner_depth;
    a.total_alpha = total_alpha;
    a.final_T = final_T;
    a.last_index = last_index;
    a.final_T_surf = final_T_surf;
    a.last_index_surf = last_index_surf;
    a.m1_surf = m1_surf;
    a.m2_surf = m2_surf;
    a.median_index = median_index;
    a.contrib_count = contrib_count;
    if (surf) return prefilter ? launch_render<true, true, false>(a, stream)
                               : launch_render<true, false, false>(a, stream);
    if (owner) return prefilter ? launch_render<false, true, true>(a, stream)
                                : launch_render<false, false, true>(a, stream);
    return prefilter ? launch_render<false, true, false>(a, stream)
                     : launch_render<false, false, false>(a, stream);
}
