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

// Per-pixel state of the front-to-back compositing.  Surface and owner
// fields are dead (and eliminated) in the instantiations without them.
struct FwdPixel {
    float px, py;
    bool done_color, done_surf;
    float T, C0, C1, C2;
    int n_visited, n_blended, n_evaluated;
    float overdraw, overdraw_hits;
    float T_surf, D_surf, median_depth, M1, M2, distortion;
    float3 N_surf;
    int n_visited_surf, median_idx;
    long long owner_id;
    float owner_weight, owner_sdf, owner_depth;
    float2 owner_uv;
};

// One (pixel, surfel) pair at list index `idx` (batch slot j): the
// reference's per-pair arithmetic (hexels3d_forward.cu:690-1000).  Returns
// whether the pair's alpha reached k3BlendMarkAlpha (the blend-mask test).
// PLAIN fixes the training configuration at compile time (linear colour,
// linear view model with view gradients, one softness for all edges, no
// overdraw, contribution or pair-count outputs, every surfel a base surfel;
// with or without the surface outputs):
// the same arithmetic without the per-pair tests of the other options.
template <bool SURF, bool PREFILTER, bool OWNER, bool PLAIN>
__device__ __forceinline__ bool fwd_pair(const Render3DArgs& a, const Surfel3D& s, int idx, int j,
                                         FwdPixel& q, float* s_contrib) {
    const int g_id = s.id;
    const bool is_base = PLAIN || g_id < a.overdraw_base;
    if (SURF && q.done_color && !is_base) return false;
    const float px = q.px, py = q.py;
    const float3 Tu = {s.tu[0], s.tu[1], s.tu[2]};
    const float3 Tv = {s.tv[0], s.tv[1], s.tv[2]};
    const float3 Tw = {s.tw[0], s.tw[1], s.tw[2]};
    const float3 k = {px * Tw.x - Tu.x, px * Tw.y - Tu.y, px * Tw.z - Tu.z};
    const float3 l = {py * Tw.x - Tv.x, py * Tw.y - Tv.y, py * Tw.z - Tv.z};
    const float3 p = cross3(k, l);
    if (p.z == 0.0f) return false;
    const float sx = p.x / p.z;
    const float sy = p.y / p.z;
    const float depth_sdf = (sx * Tw.x + sy * Tw.y) + Tw.z;
    if (depth_sdf < k3NearPlane) return false;
    float dist, soft;
    if (PLAIN || a.softness_stride == 1) {  // one softness for all edges: no edge needed
        dist = hex_sdf_value(sx, sy);
        soft = s.s0;
    } else {
        int edge;
        dist = hex_sdf3(sx, sy, edge);
        soft = (edge == 0) ? s.s0 : ((edge == 1) ? s.s1 : s.s2);
    }
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
    const bool mark = alpha >= k3BlendMarkAlpha;
    if (alpha < 1.0f / 255.0f) return mark;
    const float depth = use_filter ? Tw.z : depth_sdf;

    if (!q.done_color) {
        if (!PLAIN && is_base && alpha_sdf >= 1.0f / 255.0f) {
            if (a.overdraw) q.overdraw += alpha_raw_sdf;
            if (a.overdraw_hits) q.overdraw_hits += 1.0f;
        }
        const float test_T = q.T * (1.f - alpha);
        if (test_T < 0.0001f) {
            q.done_color = true;
        } else {
            const float w = alpha * q.T;
            const float u = use_filter ? 0.f : sx;
            const float v = use_filter ? 0.f : sy;
            if (OWNER) {
                if (w > q.owner_weight) {
                    q.owner_id = g_id;
                    q.owner_weight = w;
                    q.owner_uv = {sx, sy};
                    q.owner_sdf = dist;
                    q.owner_depth = depth;
                }
            }
            float cx = s.cb[0], cy = s.cb[1], cz = s.cb[2];
            if (PLAIN || a.color_model >= kColorLinear) {
                cx += u * s.gu[0] + v * s.gv[0];
                cy += u * s.gu[1] + v * s.gv[1];
                cz += u * s.gu[2] + v * s.gv[2];
            }
            if (!PLAIN &&
                (a.color_model == kColorQuadratic || a.color_model == kColorQuadBounded)) {
                const float* cq = a.color_quads + 9 * g_id;
                float uu = u, vv = v;
                if (a.color_model == kColorQuadBounded) bounded_coords(u, v, uu, vv);
                const float u2 = uu * uu, uv = uu * vv, v2 = vv * vv;
                cx += u2 * cq[0] + uv * cq[3] + v2 * cq[6];
                cy += u2 * cq[1] + uv * cq[4] + v2 * cq[7];
                cz += u2 * cq[2] + uv * cq[5] + v2 * cq[8];
            }
            if (PLAIN || a.use_view_grads) {
                cx += s.cv[0];
                cy += s.cv[1];
                cz += s.cv[2];
            }
            if (!PLAIN && a.view_model == kViewLobe) {
                const float* vd = a.view_dirs + 3 * g_id;
                const float* nr = a.normals + 3 * g_id;
                const float cos_nv = fmaxf(-(nr[0] * vd[0] + nr[1] * vd[1] + nr[2] * vd[2]), 0.f);
                const float log_s = a.specular_log_s[g_id];
                const float s_exp = __expf(fminf(fmaxf(log_s, 0.f), 5.0f));
                const float spec = (cos_nv > 0.f) ? __powf(cos_nv, s_exp) : 0.f;
                cx += a.specular_ks[3 * g_id] * spec;
                cy += a.specular_ks[3 * g_id + 1] * spec;
                cz += a.specular_ks[3 * g_id + 2] * spec;
            }
            q.C0 += cx * w;
            q.C1 += cy * w;
            q.C2 += cz * w;
            q.T = test_T;
            q.n_visited = idx + 1;
            if (!PLAIN) ++q.n_blended;
            if (!PLAIN && a.contrib) atomicAdd(&s_contrib[j], w);
        }
    }
    if (SURF && !q.done_surf && is_base) {
        const float test_T_surf = q.T_surf * (1.f - alpha);
        if (test_T_surf < 0.0001f) {
            q.done_surf = true;
        } else {
            if (a.median && q.T_surf > 0.5f) {
                q.median_depth = depth;
                q.median_idx = idx;
            }
            const float w_surf = alpha * q.T_surf;
            const float m = k3FarPlane / (k3FarPlane - k3NearPlane) * (1.0f - k3NearPlane / depth);
            const float acc_alpha = 1.0f - q.T_surf;
            q.distortion += (m * m * acc_alpha + q.M2 - 2.0f * m * q.M1) * w_surf;
            q.M1 += m * w_surf;
            q.M2 += m * m * w_surf;
            q.D_surf += depth * w_surf;
            q.N_surf.x += s.n[0] * w_surf;
            q.N_surf.y += s.n[1] * w_surf;
            q.N_surf.z += s.n[2] * w_surf;
            q.T_surf = test_T_surf;
            q.n_visited_surf = idx + 1;
        }
    }
    return mark;
}

// One CTA per 16x16 tile, 256 / PPT threads, PPT pixels per thread: warps
// cover 8 x (4 PPT) pixel blocks (two across, 4 / PPT down), lane l owns
// pixels (l % 8, l / 8 + 4 k), k < PPT.  The tile's list is staged 256
// surfels at a time; a warp skips a surfel whose pixel box misses its block.
template <bool SURF, bool PREFILTER, bool OWNER, int PPT, bool PLAIN>
__global__ void __launch_bounds__(k3BlockSize / PPT, PLAIN && !SURF ? 5 : 0)
    render3d_fwd_kernel(const Render3DArgs a) {
    constexpr int kThreads = k3BlockSize / PPT;
    constexpr int kWarpRows = 4 * PPT;
    __shared__ Surfel3D s_prim[k3BlockSize];
    __shared__ float s_contrib[k3BlockSize];
    // per warp: the batch slots whose pixel box meets the warp's block
    __shared__ unsigned char s_list[kThreads / 32][k3BlockSize];
    // per warp and batch slot: whether a pixel of the warp marked the pair
    __shared__ __align__(4) unsigned char s_wmark[kThreads / 32][k3BlockSize];

    const int W = a.W, H = a.H;
    const unsigned hblocks = (W + k3BlockX - 1) / k3BlockX;
    const int tr = threadIdx.x;
    const int lane = tr & 31;
    const int warp = tr >> 5;
    const int wx0 = (int)(blockIdx.x * k3BlockX) + ((warp & 1) << 3);
    const int wy0 = (int)(blockIdx.y * k3BlockY) + (warp >> 1) * kWarpRows;

    FwdPixel q[PPT];
    bool inside[PPT];
    bool thread_done = true;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        const int pxi = wx0 + (lane & 7);
        const int pyi = wy0 + (lane >> 3) + 4 * k;
        inside[k] = pxi < W && pyi < H;
        FwdPixel& p = q[k];
        p.px = (float)pxi;
        p.py = (float)pyi;
        p.done_color = !inside[k];
        p.done_surf = SURF ? !inside[k] : true;
        p.T = 1.0f;
        p.C0 = p.C1 = p.C2 = 0.f;
        p.n_visited = p.n_blended = p.n_evaluated = 0;
        p.overdraw = p.overdraw_hits = 0.f;
        p.T_surf = 1.0f;
        p.D_surf = p.median_depth = p.M1 = p.M2 = p.distortion = 0.f;
        p.N_surf = {0.f, 0.f, 0.f};
        p.n_visited_surf = 0;
        p.median_idx = -1;
        p.owner_id = -1;
        p.owner_weight = p.owner_sdf = p.owner_depth = 0.f;
        p.owner_uv = {0.f, 0.f};
        thread_done = thread_done && p.done_color && p.done_surf;
    }

    uint2 range = a.ranges[blockIdx.y * hblocks + blockIdx.x];
    range.y = min(range.y, (unsigned)a.num_rendered);
    range.x = min(range.x, range.y);
    const int rounds = (int)((range.y - range.x + k3BlockSize - 1) / k3BlockSize);
    int to_do = (int)(range.y - range.x);

    for (int i = 0; i < rounds; ++i, to_do -= k3BlockSize) {
        if (__syncthreads_count(thread_done) == kThreads) break;
        if (a.blend_mask)
            for (int t = tr; t < (kThreads / 32) * k3BlockSize / 4; t += kThreads)
                reinterpret_cast<unsigned*>(&s_wmark[0][0])[t] = 0u;
        for (int t = tr; t < k3BlockSize; t += kThreads) {
            s_contrib[t] = 0.f;
            const int progress = i * k3BlockSize + t;
            if ((int)range.x + progress >= (int)range.y) continue;
            int g = a.point_list[range.x + progress];
            g = min(max(g, 0), a.P - 1);
            if (a.records)
                stage_record_async(a.records, g, &s_prim[t]);
            else
                stage_surfel<SURF, PREFILTER>(a, g, W, H, &s_prim[t]);
        }
        if (a.records) cp_async_wait_all();
        __syncthreads();

        const int batch_size = min(k3BlockSize, to_do);
        // compact the batch to the surfels whose box meets this warp's block
        // (every pixel of a block a box misses has alpha < 1/255)
        int n_mine = 0;
        if (!__all_sync(0xffffffffu, thread_done)) {
            for (int base = 0; base < batch_size; base += 32) {
                const int t = base + lane;
                const bool hit = t < batch_size &&
                                 (PREFILTER || !box_misses(s_prim[t].q.box, wx0, wy0, wx0 + 7,
                                                           wy0 + kWarpRows - 1));
                const unsigned m = __ballot_sync(0xffffffffu, hit);
                if (hit) s_list[warp][n_mine + __popc(m & ((1u << lane) - 1u))] = (unsigned char)t;
                n_mine += __popc(m);
            }
            __syncwarp();
        }
        for (int jj = 0; !thread_done && jj < n_mine; ++jj) {
            const int j = s_list[warp][jj];
            const Surfel3D& s = s_prim[j];
            bool all_done = true, mark = false;
#pragma unroll
            for (int k = 0; k < PPT; ++k) {
                if (!(q[k].done_color && q[k].done_surf)) {
                    mark |= fwd_pair<SURF, PREFILTER, OWNER, PLAIN>(a, s, i * k3BlockSize + j,
                                                                    j, q[k], s_contrib);
                    if (!PLAIN) ++q[k].n_evaluated;
                }
                all_done = all_done && q[k].done_color && q[k].done_surf;
            }
            if (mark) s_wmark[warp][j] = 1;  // same value from every marking lane
            thread_done = all_done;
        }
        if (a.contrib || a.blend_mask) __syncthreads();
        if (a.contrib) {
            for (int t = tr; t < batch_size; t += kThreads)
                if (s_contrib[t] != 0.f) atomicAdd(&a.contrib[s_prim[t].id], s_contrib[t]);
        }
        if (a.blend_mask) {
            for (int t = tr; t < batch_size; t += kThreads) {
                unsigned bits = 0u;
#pragma unroll
                for (int w = 0; w < kThreads / 32; ++w)
                    if (s_wmark[w][t]) bits |= blend_bits(w, PPT);
                a.blend_mask[range.x + i * k3BlockSize + t] = (unsigned char)bits;
            }
        }
    }

    const int HW = H * W;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        if (!inside[k]) continue;
        const FwdPixel& p = q[k];
        const int pix = (int)p.py * W + (int)p.px;
        if (a.final_T) {
            a.final_T[pix] = p.T;
            a.last_index[pix] = p.n_visited;
        }
        if (a.contrib_count) {
            a.contrib_count[pix] = p.n_blended;
            a.contrib_count[HW + pix] = p.n_evaluated;
        }
        // With nothing binned every tile range is empty and the pixel is the
        // background, as in the reference (hexels3d_forward.cu:3300-3470).
        a.out_color[pix] = p.C0 + p.T * a.bg[0];
        a.out_color[HW + pix] = p.C1 + p.T * a.bg[1];
        a.out_color[2 * HW + pix] = p.C2 + p.T * a.bg[2];
        if (a.overdraw) a.overdraw[pix] = p.overdraw;
        if (a.overdraw_hits) a.overdraw_hits[pix] = p.overdraw_hits;
        if (SURF) {
            a.out_depth[pix] = p.D_surf;
            a.out_alpha[pix] = 1.0f - p.T_surf;
            a.out_surface[pix] = p.N_surf.x;
            a.out_surface[HW + pix] = p.N_surf.y;
            a.out_surface[2 * HW + pix] = p.N_surf.z;
            a.out_surface[3 * HW + pix] = p.distortion;
            if (a.median) a.out_surface[4 * HW + pix] = p.median_depth;
            if (a.final_T_surf) {
                a.final_T_surf[pix] = p.T_surf;
                a.last_index_surf[pix] = p.n_visited_surf;
                a.m1_surf[pix] = p.M1;
                a.m2_surf[pix] = p.M2;
                a.median_index[pix] = p.median_idx;
            }
        }
        if (OWNER) {
            a.owner_id[pix] = p.owner_id;
            a.owner_weight[pix] = p.owner_weight;
            a.owner_uv[pix] = p.owner_uv.x;
            a.owner_uv[HW + pix] = p.owner_uv.y;
            a.owner_sdf[pix] = p.owner_sdf;
            a.owner_depth[pix] = p.owner_depth;
            a.total_alpha[pix] = 1.0f - p.T;
        }
    }
}

}  // namespace hx

using namespace hx;

namespace {

template <bool SURF, bool PREFILTER, bool OWNER>
int launch_render(const Render3DArgs& a, cudaStream_t stream) {
    // One pixel per thread: each pixel terminates on its own, and two per
    // thread keep a lane busy until both have (measured slower on B200).
    constexpr int kPPT = 1;
    dim3 grid(ceil_div(a.W, k3BlockX), ceil_div(a.H, k3BlockY));
    if constexpr (!PREFILTER && !OWNER) {
        // (every surfel a base surfel: the surface outputs skip the others)
        if (a.color_model == kColorLinear && a.view_model == kViewLinear && a.use_view_grads &&
            a.softness_stride == 1 && !a.overdraw && !a.overdraw_hits && !a.contrib &&
            !a.contrib_count && a.overdraw_base >= a.P) {
            render3d_fwd_kernel<SURF, false, false, kPPT, true>
                <<<grid, k3BlockSize / kPPT, 0, stream>>>(a);
            HX_LAUNCH_CHECK("render3d_fwd_kernel");
            return HX_OK;
        }
    }
    render3d_fwd_kernel<SURF, PREFILTER, OWNER, kPPT, false>
        <<<grid, k3BlockSize / kPPT, 0, stream>>>(a);
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
    float* m2_surf, int32_t* median_index, int32_t* contrib_count, uint8_t* blend_mask,
    const void* records, cudaStream_t stream) {
    HX_REQUIRE(image_width > 0 && image_height > 0, "invalid image dimensions");
    HX_REQUIRE((uintptr_t)records % 16 == 0, "records must start on a 16-byte boundary");
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
    a.blend_mask = blend_mask;
    a.records = (const Surfel3D*)records;
    if (surf) return prefilter ? launch_render<true, true, false>(a, stream)
                               : launch_render<true, false, false>(a, stream);
    if (owner) return prefilter ? launch_render<false, true, true>(a, stream)
                                : launch_render<false, false, true>(a, stream);
    return prefilter ? launch_render<false, true, false>(a, stream)
                     : launch_render<false, false, false>(a, stream);
}

namespace hx {
namespace {

// One thread per surfel: its record as the compositing kernels stage it,
// assembled in shared memory and written out by the CTA as one contiguous
// run of 16-byte stores (256 records, 32 KB).
template <bool SURF, bool PREFILTER>
__global__ void __launch_bounds__(256) surfel_records_kernel(const Render3DArgs a,
                                                             Surfel3D* __restrict__ out) {
    __shared__ Surfel3D s_rec[256];
    const int g0 = blockIdx.x * 256;
    const int g = g0 + (int)threadIdx.x;
    if (g < a.P) stage_surfel<SURF, PREFILTER>(a, g, a.W, a.H, &s_rec[threadIdx.x]);
    __syncthreads();
    const int n = min(256, a.P - g0) * (int)(sizeof(Surfel3D) / sizeof(float4));
    const float4* src = reinterpret_cast<const float4*>(s_rec);
    float4* dst = reinterpret_cast<float4*>(out + g0);
    for (int i = (int)threadIdx.x; i < n; i += 256) dst[i] = src[i];
}

}  // namespace
}  // namespace hx

extern "C" int hx_hexels3d_surfel_records(
    int P, int image_width, int image_height, const float* transMats, const float* opacities,
    const float* softnesses, int softness_stride, const float* colors, const float* color_grads,
    const float* view_grads, const float* view_dirs, const float* normals,
    const float* points_xy_center, int color_model, int use_view_grads, int surface,
    void* records, cudaStream_t stream) {
    HX_REQUIRE(P >= 0 && image_width > 0 && image_height > 0,
               "hexels3d_surfel_records: bad sizes");
    if (P == 0) return HX_OK;
    HX_REQUIRE(softness_stride == 1 || softness_stride == 3, "softness_stride must be 1 or 3");
    HX_REQUIRE(transMats && opacities && softnesses && colors && view_dirs && records,
               "hexels3d_surfel_records: null pointer");
    HX_REQUIRE((uintptr_t)records % 16 == 0, "records must start on a 16-byte boundary");
    HX_REQUIRE(color_model < 1 || color_grads, "color_grads required for color_model >= 1");
    HX_REQUIRE(!use_view_grads || view_grads, "view_grads required with use_view_grads");
    HX_REQUIRE(!surface || normals, "surface records need normals");
    Render3DArgs a = {};
    a.P = P;
    a.W = image_width;
    a.H = image_height;
    a.transMats = transMats;
    a.opacities = opacities;
    a.softnesses = softnesses;
    a.softness_stride = softness_stride;
    a.colors = colors;
    a.color_grads = color_grads;
    a.view_grads = view_grads;
    a.view_dirs = view_dirs;
    a.normals = normals;
    a.points_xy_center = (const float2*)points_xy_center;
    a.color_model = color_model;
    a.use_view_grads = use_view_grads != 0;
    Surfel3D* out = (Surfel3D*)records;
    const int blocks = ceil_div(P, 256);
    const bool prefilter = points_xy_center != nullptr;
    if (surface) {
        if (prefilter)
            surfel_records_kernel<true, true><<<blocks, 256, 0, stream>>>(a, out);
        else
            surfel_records_kernel<true, false><<<blocks, 256, 0, stream>>>(a, out);
    } else {
        if (prefilter)
            surfel_records_kernel<false, true><<<blocks, 256, 0, stream>>>(a, out);
        else
            surfel_records_kernel<false, false><<<blocks, 256, 0, stream>>>(a, out);
    }
    HX_LAUNCH_CHECK("surfel_records_kernel");
    return HX_OK;
}
