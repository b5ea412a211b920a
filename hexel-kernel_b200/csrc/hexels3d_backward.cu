// S8 backward: reverse traversal of the front-to-back compositing and the VJP
// to the ray-splat transforms and appearance parameters (reference
// gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:1749-2492), and the VJP from
// transforms to geometry (hexels3d_forward.cu:2494-2664).
//
// Per-pixel arithmetic is the reference's.  The schedule is B200-specific:
//   * one CTA per 16x16 tile walks the tile's list back to front in lock step
//     (pixel p is active for list index i < its own last index), with the
//     surfels of each 256-entry batch staged in shared memory instead of
//     re-read from global memory by every pixel;
//   * the per-(pixel, surfel) gradient vector (up to 64 components) is summed
//     over the warp with a butterfly reduce-scatter (N - N/32 shuffles, each
//     lane ends with N/32 component sums), added into a per-batch
//     shared-memory accumulator, and flushed with one global atomic per
//     (surfel, component) per tile — instead of ~33 global atomics per
//     (pixel, surfel);
//   * gradients that factor through per-surfel constants (linear view-model
//     gradients and the matching view-direction gradient) are formed once per
//     surfel at flush time from the accumulated colour gradient;
//   * with surface outputs the forward's saved per-pixel state replaces the
//     reference's forward re-walk.
#include <atomic>

#include "hx_cmat.cuh"
#include "hx_hexmath3d.cuh"

namespace hx {

struct BwdLayout {
    int ncomp;
    int off_cg, off_cq, off_op, off_soft, off_tm, off_vd, off_n, off_ks, off_ls, off_abs, off_ctr;
    bool derive_vg, derive_vd;
};

// Fixed slot layout of the common configurations (flat or linear colour,
// no or linear view model): colour 0-2, colour gradients 3-8, opacity 9,
// softness 10-12, transform 13-21, normal 22-24, screen-gradient norm 25,
// prefilter centre 26-27, explicit view direction 28-30.
constexpr int kFixCg = 3, kFixOp = 9, kFixSoft = 10, kFixTm = 13, kFixN = 22, kFixAbs = 25,
              kFixCtr = 26, kFixVd = 28, kFixComp = 31;

// Lite slot layout of the plain RGB configuration (flat or linear colour, no
// or linear view model, no softness, normal, prefilter or means2d-norm
// gradients): colour 0-2, colour gradients 3-8, opacity 9, transform 10-18;
// padded to 24 slots.
constexpr int kLiteCg = 3, kLiteOp = 9, kLiteTm = 10, kLiteComp = 19;

// Sum of a 24-slot vector over the warp: three reduce-scatter halvings
// (over lane bits 4, 3, 2) leave each lane 3 slots summed over 8 lanes, then
// an all-reduce over lane bits 1 and 0 completes the sums.  Lanes that share
// bits 2-4 hold the same 3 slots, starting at the returned index.
__device__ __forceinline__ int warp_reduce_scatter24(float (&v)[24], const int lane) {
    int start = 0;
#pragma unroll
    for (int o = 16, n = 24; o >= 4; o >>= 1, n >>= 1) {
        const int half = n / 2;
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
        if (upper) start += half;
    }
#pragma unroll
    for (int o = 2; o >= 1; o >>= 1) {
#pragma unroll
        for (int i = 0; i < 3; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
    }
    return start;
}

// Sum of a 24-slot vector over each 16-lane half of the warp (two vectors
// at once): reduce-scatter halvings over lane bits 3, 2, 1 leave each lane 3
// slots summed over 8 lanes, and one exchange over lane bit 0 completes them
// split between the two lanes: the even lane holds slots start, start + 1 in
// v[0], v[1], the odd lane slot start + 2 in v[2].
__device__ __forceinline__ int half_warp_reduce_scatter24(float (&v)[24], const int lane) {
    int start = 0;
#pragma unroll
    for (int o = 8, n = 24; o >= 2; o >>= 1, n >>= 1) {
        const int half = n / 2;
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
        if (upper) start += half;
    }
    const bool odd = (lane & 1) != 0;
    const float r0 = __shfl_xor_sync(0xffffffffu, odd ? v[0] : v[2], 1);
    const float r1 = __shfl_xor_sync(0xffffffffu, v[1], 1);
    if (odd) {
        v[2] += r0;
    } else {
        v[0] += r0;
        v[1] += r1;
    }
    return start;
}

template <int N>
__device__ __forceinline__ int warp_reduce_scatter(float (&v)[N], const int lane) {
    int start = 0;
#pragma unroll
    for (int o = 16, n = N; o >= 1; o >>= 1, n >>= 1) {
        const int half = n / 2;
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
        if (upper) start += half;
    }
    return start;
}

// Per-pixel state of the reverse traversal.  The surface fields are dead
// (and eliminated) in the RGB-only instantiations.
struct BwdPixel {
    float px, py;
    float v_r, v_g, v_b, v_overdraw;
    float T_after;
    float3 behind;
    int n_color;
    float v_depth, v_alpha, v_dist, v_median;
    float3 v_normal;
    float T_after_surf, M1, M2, final_alpha_surf, last_dist_vjp;
    float behind_depth, behind_alpha;
    float3 behind_normal;
    int n_surf, median_index;
};

// Slot offsets of the per-pair gradient vector.
struct BwdSlots {
    int cg, cq, op, soft, tm, vd, n, ks, ls, abs, ctr;
};

// VJP of one (pixel, surfel) pair at list index idx, ADDED into acc; updates
// the pixel's running state (transmittance and "behind" terms).  Returns
// whether the pair blended.  Per-pair arithmetic restates
// hexels3d_forward.cu:1983-2470.  PL fixes the training configuration at
// compile time (linear colour with colour-gradient slots, linear view model
// with view gradients, one softness, every surfel a base surfel, no
// overdraw, softness, quadratic, lobe or explicit view-direction slots): the
// same arithmetic without those per-pair tests.
template <bool SURF, bool PREFILTER, int N, bool PL>
__device__ __forceinline__ bool bwd_pair(const Backward3DArgs& a, const BwdLayout& L,
                                         const BwdSlots& O, const Surfel3D& s, const int idx,
                                         BwdPixel& q, float (&acc)[N]) {
    const int g_id = s.id;
    const bool is_base = PL || g_id < a.overdraw_base;
    const bool active_color = idx < q.n_color;
    const bool active_surf = SURF && is_base && idx < q.n_surf;
    if (!active_color && !active_surf) return false;
    const float px = q.px, py = q.py;
    const float3 Tu = {s.tu[0], s.tu[1], s.tu[2]};
    const float3 Tv = {s.tv[0], s.tv[1], s.tv[2]};
    const float3 Tw = {s.tw[0], s.tw[1], s.tw[2]};
    const float3 soft3 = {s.s0, s.s1, s.s2};
    HexHit h;
    if (!hexel_hit(px, py, Tu, Tv, Tw, s.opacity, soft3, PL || a.softness_stride == 1, h))
        return false;
    float alpha = h.alpha;
    bool use_filter = false, clamped_filter = false;
    float G = 0.f, dxf = 0.f, dyf = 0.f;
    if (PREFILTER) {
        dxf = px - s.q.ctr.x;
        dyf = py - s.q.ctr.y;
        G = __expf(-0.5f * k3FilterInvSquare * (dxf * dxf + dyf * dyf));
        const float arf = s.opacity * G;
        clamped_filter = arf > 0.99f;
        const float af = clamped_filter ? 0.99f : arf;
        use_filter = af > h.alpha;
        alpha = use_filter ? af : h.alpha;
    }
    if (alpha < 1.0f / 255.0f) return false;

    const float u = h.u, v = h.v;
    const float depth = use_filter ? Tw.z : h.depth;
    const float inv_1ma = 1.f / (1.f - alpha);
    float3 c = {0.f, 0.f, 0.f};
    float v_alpha_total = 0.f, v_u = 0.f, v_v = 0.f, v_depth_direct = 0.f;
    float T_before = 0.f;
    const float v_out_r = q.v_r, v_out_g = q.v_g, v_out_b = q.v_b;
    if (active_color) {
        T_before = q.T_after * inv_1ma;
        const float w = alpha * T_before;
        const float ua = use_filter ? 0.f : u;
        const float va = use_filter ? 0.f : v;
        c = {s.cb[0], s.cb[1], s.cb[2]};
        if (PL || a.color_model >= kColorLinear) {
            c.x += ua * s.gu[0] + va * s.gv[0];
            c.y += ua * s.gu[1] + va * s.gv[1];
            c.z += ua * s.gu[2] + va * s.gv[2];
        }
        const float* cq = nullptr;
        float ub = ua, vb = va;
        if (!PL && (a.color_model == kColorQuadratic || a.color_model == kColorQuadBounded)) {
            cq = a.color_quads + 9 * g_id;
            if (a.color_model == kColorQuadBounded) bounded_coords(ua, va, ub, vb);
            const float u2 = ub * ub, uv = ub * vb, v2 = vb * vb;
            c.x += u2 * cq[0] + uv * cq[3] + v2 * cq[6];
            c.y += u2 * cq[1] + uv * cq[4] + v2 * cq[7];
            c.z += u2 * cq[2] + uv * cq[5] + v2 * cq[8];
        }
        if (PL || a.use_view_grads) {
            c.x += s.cv[0];
            c.y += s.cv[1];
            c.z += s.cv[2];
        }
        float spec = 0.f, cos_nv = 0.f, s_exp = 0.f;
        bool log_s_clamped = false;
        const float* vd = a.view_dirs + 3 * g_id;
        float3 nr = {0.f, 0.f, 0.f};
        if (!PL && a.view_model == kViewLobe) {
            if (a.normals)
                nr = {a.normals[3 * g_id], a.normals[3 * g_id + 1], a.normals[3 * g_id + 2]};
            cos_nv = fmaxf(-(nr.x * vd[0] + nr.y * vd[1] + nr.z * vd[2]), 0.f);
            const float log_s = a.specular_log_s[g_id];
            log_s_clamped = (log_s < 0.f) || (log_s > 5.0f);
            s_exp = __expf(fminf(fmaxf(log_s, 0.f), 5.0f));
            spec = (cos_nv > 0.f) ? __powf(cos_nv, s_exp) : 0.f;
            c.x += a.specular_ks[3 * g_id] * spec;
            c.y += a.specular_ks[3 * g_id + 1] * spec;
            c.z += a.specular_ks[3 * g_id + 2] * spec;
        }
        acc[0] += w * v_out_r;
        acc[1] += w * v_out_g;
        acc[2] += w * v_out_b;
        if (PL || L.off_cg >= 0) {
            acc[O.cg + 0] += w * v_out_r * ua;
            acc[O.cg + 1] += w * v_out_g * ua;
            acc[O.cg + 2] += w * v_out_b * ua;
            acc[O.cg + 3] += w * v_out_r * va;
            acc[O.cg + 4] += w * v_out_g * va;
            acc[O.cg + 5] += w * v_out_b * va;
        }
        if (!PL && L.off_cq >= 0 && cq) {
            const float q3[3] = {ub * ub, ub * vb, vb * vb};
#pragma unroll
            for (int r = 0; r < 3; ++r) {
                acc[O.cq + 3 * r + 0] += w * v_out_r * q3[r];
                acc[O.cq + 3 * r + 1] += w * v_out_g * q3[r];
                acc[O.cq + 3 * r + 2] += w * v_out_b * q3[r];
            }
        }
        if (!PL && a.use_view_grads && L.off_vd >= 0 && !use_filter) {
            const float* vg = a.view_grads + 9 * g_id;
            acc[O.vd + 0] += w * (v_out_r * vg[0] + v_out_g * vg[3] + v_out_b * vg[6]);
            acc[O.vd + 1] += w * (v_out_r * vg[1] + v_out_g * vg[4] + v_out_b * vg[7]);
            acc[O.vd + 2] += w * (v_out_r * vg[2] + v_out_g * vg[5] + v_out_b * vg[8]);
        }
        if (!PL && a.view_model == kViewLobe) {
            if (L.off_ks >= 0) {
                acc[O.ks + 0] += w * v_out_r * spec;
                acc[O.ks + 1] += w * v_out_g * spec;
                acc[O.ks + 2] += w * v_out_b * spec;
            }
            const float v_spec = w * (v_out_r * a.specular_ks[3 * g_id] +
                                      v_out_g * a.specular_ks[3 * g_id + 1] +
                                      v_out_b * a.specular_ks[3 * g_id + 2]);
            if (L.off_ls >= 0 && !log_s_clamped && cos_nv > 0.f)
                acc[O.ls] += v_spec * (spec * logf(cos_nv) * s_exp);
            if (!use_filter && v_spec != 0.f && cos_nv > 0.f) {
                const float v_cos = v_spec * (s_exp * spec / cos_nv);
                if (L.off_vd >= 0) {
                    acc[O.vd + 0] += -v_cos * nr.x;
                    acc[O.vd + 1] += -v_cos * nr.y;
                    acc[O.vd + 2] += -v_cos * nr.z;
                }
                if (L.off_n >= 0) {
                    acc[O.n + 0] += -v_cos * vd[0];
                    acc[O.n + 1] += -v_cos * vd[1];
                    acc[O.n + 2] += -v_cos * vd[2];
                }
            }
        }
        v_alpha_total += T_before * (v_out_r * (c.x - q.behind.x) + v_out_g * (c.y - q.behind.y) +
                                     v_out_b * (c.z - q.behind.z));
        if (!use_filter && (PL || a.color_model >= kColorLinear)) {
            v_u += w * (v_out_r * s.gu[0] + v_out_g * s.gu[1] + v_out_b * s.gu[2]);
            v_v += w * (v_out_r * s.gv[0] + v_out_g * s.gv[1] + v_out_b * s.gv[2]);
        }
        if (!PL && !use_filter && a.color_model == kColorQuadratic) {
            const float du_r = 2.f * u * cq[0] + v * cq[3];
            const float du_g = 2.f * u * cq[1] + v * cq[4];
            const float du_b = 2.f * u * cq[2] + v * cq[5];
            const float dv_r = u * cq[3] + 2.f * v * cq[6];
            const float dv_g = u * cq[4] + 2.f * v * cq[7];
            const float dv_b = u * cq[5] + 2.f * v * cq[8];
            v_u += w * (v_out_r * du_r + v_out_g * du_g + v_out_b * du_b);
            v_v += w * (v_out_r * dv_r + v_out_g * dv_g + v_out_b * dv_b);
        } else if (!PL && !use_filter && a.color_model == kColorQuadBounded) {
            float ubb, vbb;
            bounded_coords(u, v, ubb, vbb);
            const float du_r = 2.f * ubb * cq[0] + vbb * cq[3];
            const float du_g = 2.f * ubb * cq[1] + vbb * cq[4];
            const float du_b = 2.f * ubb * cq[2] + vbb * cq[5];
            const float dv_r = ubb * cq[3] + 2.f * vbb * cq[6];
            const float dv_g = ubb * cq[4] + 2.f * vbb * cq[7];
            const float dv_b = ubb * cq[5] + 2.f * vbb * cq[8];
            bounded_coords_vjp(u, v, w * (v_out_r * du_r + v_out_g * du_g + v_out_b * du_b),
                               w * (v_out_r * dv_r + v_out_g * dv_g + v_out_b * dv_b), v_u, v_v);
        }
    }
    float T_before_surf = 0.f;
    float3 n_surf = {0.f, 0.f, 0.f};
    if (SURF && active_surf) {
        T_before_surf = q.T_after_surf * inv_1ma;
        const float w_surf = alpha * T_before_surf;
        if (q.v_depth != 0.f) {
            v_alpha_total += T_before_surf * q.v_depth * (depth - q.behind_depth);
            if (!use_filter) {
                v_depth_direct += w_surf * q.v_depth;
                v_u += v_depth_direct * Tw.x;
                v_v += v_depth_direct * Tw.y;
            }
        }
        if (q.v_dist != 0.f) {
            const float m = k3FarPlane / (k3FarPlane - k3NearPlane) * (1.0f - k3NearPlane / depth);
            const float weight_vjp =
                (q.M2 + m * m * q.final_alpha_surf - 2.0f * m * q.M1) * q.v_dist;
            v_alpha_total += T_before_surf * (weight_vjp - q.last_dist_vjp);
            q.last_dist_vjp = alpha * weight_vjp + (1.0f - alpha) * q.last_dist_vjp;
            if (!use_filter) {
                const float m_vjp = 2.0f * w_surf * (m * q.final_alpha_surf - q.M1) * q.v_dist;
                const float depth_vjp = m_vjp * (k3FarPlane * k3NearPlane) /
                                        ((k3FarPlane - k3NearPlane) * depth * depth);
                v_depth_direct += depth_vjp;
                v_u += depth_vjp * Tw.x;
                v_v += depth_vjp * Tw.y;
            }
        }
        if (idx == q.median_index && q.v_median != 0.f) {
            if (use_filter) {
                acc[O.tm + 8] += q.v_median;
            } else {
                v_depth_direct += q.v_median;
                v_u += q.v_median * Tw.x;
                v_v += q.v_median * Tw.y;
            }
        }
        if (q.v_alpha != 0.f)
            v_alpha_total += T_before_surf * q.v_alpha * (1.f - q.behind_alpha);
        if (a.grad_out_surf_normals && a.normals) {
            n_surf = {s.n[0], s.n[1], s.n[2]};
            v_alpha_total += T_before_surf * (q.v_normal.x * (n_surf.x - q.behind_normal.x) +
                                              q.v_normal.y * (n_surf.y - q.behind_normal.y) +
                                              q.v_normal.z * (n_surf.z - q.behind_normal.z));
            if (!use_filter && L.off_n >= 0) {
                acc[O.n + 0] += s.nsign * w_surf * q.v_normal.x;
                acc[O.n + 1] += s.nsign * w_surf * q.v_normal.y;
                acc[O.n + 2] += s.nsign * w_surf * q.v_normal.z;
            }
        }
    }
    // opacity
    float v_op = 0.f;
    if (use_filter) {
        if (!clamped_filter) {
            v_op += v_alpha_total * G;
            if (PREFILTER && L.off_ctr >= 0) {
                const float factor = v_alpha_total * s.opacity * G * k3FilterInvSquare;
                acc[O.ctr + 0] += factor * dxf;
                acc[O.ctr + 1] += factor * dyf;
            }
        }
    } else if (!h.clamped) {
        v_op += v_alpha_total * h.boundary;
    }
    const bool alpha_sdf_ok = h.alpha >= (1.0f / 255.0f);
    const bool has_overdraw =
        !PL && (q.v_overdraw != 0.f) && active_color && is_base && alpha_sdf_ok;
    if (has_overdraw) v_op += q.v_overdraw * h.boundary;
    acc[O.op] += v_op;
    if (!PL && L.off_soft >= 0) {
        const float sig = h.boundary;
        float v_soft = 0.f;
        if (!use_filter && !h.clamped)
            v_soft += v_alpha_total * s.opacity * (-h.dist) * sig * (1.f - sig);
        if (has_overdraw) v_soft += q.v_overdraw * s.opacity * (-h.dist) * sig * (1.f - sig);
        if (a.softness_stride == 3) {
            acc[O.soft + 0] += h.edge == 0 ? v_soft : 0.f;
            acc[O.soft + 1] += h.edge == 1 ? v_soft : 0.f;
            acc[O.soft + 2] += h.edge == 2 ? v_soft : 0.f;
        } else {
            acc[O.soft] += v_soft;
        }
    }
    if ((!use_filter && !h.clamped) || has_overdraw) {
        float dist_g, ddu, ddv;
        int edge_g;
        hex_sdf3_grad(u, v, dist_g, ddu, ddv, edge_g);
        const float soft_g =
            PL ? soft3.x : ((edge_g == 0) ? soft3.x : ((edge_g == 1) ? soft3.y : soft3.z));
        const float d_sig = -soft_g * h.boundary * (1.f - h.boundary);
        float v_ad = has_overdraw ? (q.v_overdraw * s.opacity * d_sig) : 0.f;
        if (!use_filter && !h.clamped) v_ad += v_alpha_total * s.opacity * d_sig;
        v_u += v_ad * ddu;
        v_v += v_ad * ddv;
    }
    const float3 k = {px * Tw.x - Tu.x, px * Tw.y - Tu.y, px * Tw.z - Tu.z};
    const float3 l = {py * Tw.x - Tv.x, py * Tw.y - Tv.y, py * Tw.z - Tv.z};
    const float3 p = cross3(k, l);
    if (p.z != 0.f) {
        const float inv_pz = 1.f / p.z;
        const float dsx = v_u * inv_pz;
        const float dsy = v_v * inv_pz;
        const float3 v_p = {dsx, dsy, -(dsx * u + dsy * v)};
        const float3 v_k = cross3(l, v_p);
        const float3 v_l = cross3(v_p, k);
        float3 v_Tw = {px * v_k.x + py * v_l.x, px * v_k.y + py * v_l.y,
                       px * v_k.z + py * v_l.z};
        if (SURF && active_surf && v_depth_direct != 0.f) {
            v_Tw.x += u * v_depth_direct;
            v_Tw.y += v * v_depth_direct;
            v_Tw.z += v_depth_direct;
        }
        if (L.off_abs >= 0) {
            const float gx = -v_k.z * Tw.z * 0.5f * (float)a.W;
            const float gy = -v_l.z * Tw.z * 0.5f * (float)a.H;
            acc[O.abs] += sqrtf(gx * gx + gy * gy);
        }
        acc[O.tm + 0] += -v_k.x;
        acc[O.tm + 1] += -v_k.y;
        acc[O.tm + 2] += -v_k.z;
        acc[O.tm + 3] += -v_l.x;
        acc[O.tm + 4] += -v_l.y;
        acc[O.tm + 5] += -v_l.z;
        acc[O.tm + 6] += v_Tw.x;
        acc[O.tm + 7] += v_Tw.y;
        acc[O.tm + 8] += v_Tw.z;
    }
    if (active_color) {
        q.behind = {alpha * c.x + (1.f - alpha) * q.behind.x,
                    alpha * c.y + (1.f - alpha) * q.behind.y,
                    alpha * c.z + (1.f - alpha) * q.behind.z};
        q.T_after = T_before;
    }
    if (SURF && active_surf) {
        q.behind_depth = alpha * depth + (1.f - alpha) * q.behind_depth;
        q.behind_alpha = alpha * 1.0f + (1.f - alpha) * q.behind_alpha;
        if (a.grad_out_surf_normals && a.normals) {
            q.behind_normal = {alpha * n_surf.x + (1.f - alpha) * q.behind_normal.x,
                               alpha * n_surf.y + (1.f - alpha) * q.behind_normal.y,
                               alpha * n_surf.z + (1.f - alpha) * q.behind_normal.z};
        }
        q.T_after_surf = T_before_surf;
    }
    return true;
}

// ---------------------------------------------------------------------------
// Packed plain-RGB pairs.  On the training path (flat or linear colour, no
// or linear view model, no surface, prefilter, overdraw or softness
// gradients) a list entry's work splits into a cheap per-pixel part that
// must run in list order (hit test, alpha, and the reverse recursion of the
// transmittance and the colour behind) and the VJP proper, which depends
// only on a few numbers of the pair.  The warp runs the first part for all
// its pixels, writes each blended pair's numbers into consecutive slots of a
// warp-private shared buffer, and runs the VJP with one pair per lane, so
// that ~17 blended pairs of the 64 pixels take one pass of the VJP instead
// of one per 8x4 half at a quarter of the lanes.
// ---------------------------------------------------------------------------
struct PairRec {
    float4 a;  // w * v_out (3), v_alpha (the alpha VJP of the colour term)
    float4 b;  // u, v, boundary weight (negative: alpha clamped), source lane | half << 5
};

// First part for one pixel: returns whether the pair blends and fills rec.
__device__ __forceinline__ bool rgb_pair_forward(const Backward3DArgs& a, const Surfel3D& s,
                                                 const int idx, BwdPixel& q, PairRec& rec) {
    if (idx >= q.n_color) return false;
    const float3 Tu = {s.tu[0], s.tu[1], s.tu[2]};
    const float3 Tv = {s.tv[0], s.tv[1], s.tv[2]};
    const float3 Tw = {s.tw[0], s.tw[1], s.tw[2]};
    const float3 soft3 = {s.s0, s.s1, s.s2};
    HexHit h;
    if (!hexel_hit(q.px, q.py, Tu, Tv, Tw, s.opacity, soft3, a.softness_stride == 1, h))
        return false;
    const float alpha = h.alpha;
    if (alpha < 1.0f / 255.0f) return false;
    const float u = h.u, v = h.v;
    const float T_before = q.T_after * (1.f / (1.f - alpha));
    const float w = alpha * T_before;
    const float cx = s.cb[0] + u * s.gu[0] + v * s.gv[0] + s.cv[0];
    const float cy = s.cb[1] + u * s.gu[1] + v * s.gv[1] + s.cv[1];
    const float cz = s.cb[2] + u * s.gu[2] + v * s.gv[2] + s.cv[2];
    const float v_alpha = T_before * (q.v_r * (cx - q.behind.x) + q.v_g * (cy - q.behind.y) +
                                      q.v_b * (cz - q.behind.z));
    rec.a = make_float4(w * q.v_r, w * q.v_g, w * q.v_b, v_alpha);
    rec.b = make_float4(u, v, h.clamped ? -1.f : h.boundary, 0.f);
    q.behind = {alpha * cx + (1.f - alpha) * q.behind.x, alpha * cy + (1.f - alpha) * q.behind.y,
                alpha * cz + (1.f - alpha) * q.behind.z};
    q.T_after = T_before;
    return true;
}

// The VJP of one packed pair at pixel (px, py), added into the 24-slot
// plain-RGB vector (colour 0-2, colour gradients 3-8, opacity 9, transform
// 10-18).  Same terms as bwd_pair's for this configuration.
__device__ __forceinline__ void rgb_pair_vjp(const Surfel3D& s, const PairRec& rec,
                                             const float px, const float py, float (&acc)[24]) {
    const float wr = rec.a.x, wg = rec.a.y, wb = rec.a.z, v_alpha = rec.a.w;
    const float u = rec.b.x, v = rec.b.y, bnd = rec.b.z;
    acc[0] += wr;
    acc[1] += wg;
    acc[2] += wb;
    acc[kLiteCg + 0] += wr * u;
    acc[kLiteCg + 1] += wg * u;
    acc[kLiteCg + 2] += wb * u;
    acc[kLiteCg + 3] += wr * v;
    acc[kLiteCg + 4] += wg * v;
    acc[kLiteCg + 5] += wb * v;
    float v_u = wr * s.gu[0] + wg * s.gu[1] + wb * s.gu[2];
    float v_v = wr * s.gv[0] + wg * s.gv[1] + wb * s.gv[2];
    if (bnd >= 0.f) {  // alpha not clamped: opacity and SDF terms
        acc[kLiteOp] += v_alpha * bnd;
        float dist_g, ddu, ddv;
        int edge_g;
        hex_sdf3_grad(u, v, dist_g, ddu, ddv, edge_g);
        const float soft_g = (edge_g == 0) ? s.s0 : ((edge_g == 1) ? s.s1 : s.s2);
        const float v_ad = v_alpha * s.opacity * (-soft_g * bnd * (1.f - bnd));
        v_u += v_ad * ddu;
        v_v += v_ad * ddv;
    }
    const float3 Tu = {s.tu[0], s.tu[1], s.tu[2]};
    const float3 Tv = {s.tv[0], s.tv[1], s.tv[2]};
    const float3 Tw = {s.tw[0], s.tw[1], s.tw[2]};
    const float3 k = {px * Tw.x - Tu.x, px * Tw.y - Tu.y, px * Tw.z - Tu.z};
    const float3 l = {py * Tw.x - Tv.x, py * Tw.y - Tv.y, py * Tw.z - Tv.z};
    const float3 p = cross3(k, l);
    if (p.z != 0.f) {
        const float inv_pz = 1.f / p.z;
        const float dsx = v_u * inv_pz;
        const float dsy = v_v * inv_pz;
        const float3 v_p = {dsx, dsy, -(dsx * u + dsy * v)};
        const float3 v_k = cross3(l, v_p);
        const float3 v_l = cross3(v_p, k);
        acc[kLiteTm + 0] += -v_k.x;
        acc[kLiteTm + 1] += -v_k.y;
        acc[kLiteTm + 2] += -v_k.z;
        acc[kLiteTm + 3] += -v_l.x;
        acc[kLiteTm + 4] += -v_l.y;
        acc[kLiteTm + 5] += -v_l.z;
        acc[kLiteTm + 6] += px * v_k.x + py * v_l.x;
        acc[kLiteTm + 7] += px * v_k.y + py * v_l.y;
        acc[kLiteTm + 8] += px * v_k.z + py * v_l.z;
    }
}

// Packs the blended pairs of the entry in hand (ballots m[k] of the lanes'
// pixel k, records rec[k]) into pairs[0, n) in pixel order.
template <int PPT>
__device__ __forceinline__ void pack_pairs(const unsigned (&m)[PPT], const PairRec (&rec)[PPT],
                                           const int lane, PairRec* pairs) {
    int base = 0;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        if (m[k] & (1u << lane)) pairs[base + __popc(m[k] & ((1u << lane) - 1u))] = rec[k];
        base += __popc(m[k]);
    }
}

// The VJP of a packed pair of the warp whose pixel block starts at (wx0,
// wy0); the pair carries its lane and pixel slot (lane | k << 5).
__device__ __forceinline__ void packed_pair_vjp(const Surfel3D& s, const PairRec& r, const int wx0,
                                                const int wy0, float (&acc)[24]) {
    const int code = __float_as_int(r.b.w);
    const float px = (float)(wx0 + (code & 7));
    const float py = (float)(wy0 + ((code & 31) >> 3) + 4 * (code >> 5));
    rgb_pair_vjp(s, r, px, py, acc);
}

// Adds a warp-reduced 24-slot vector (warp_reduce_scatter24) into the
// entry's shared gradient row.
__device__ __forceinline__ void put_reduced24(float* dst, const float (&acc)[24], const int start,
                                              const int lane) {
    const int c = lane & 3;  // lanes 0-2 of each group of 4 write
    const float val = c == 0 ? acc[0] : (c == 1 ? acc[1] : acc[2]);
    const int comp = start + c;
    if (c < 3 && comp < kLiteComp && val != 0.f) atomicAdd(dst + comp, val);
}

// One CTA per 16x16 tile, 256 / PPT threads, PPT pixels per thread: warps
// cover 8 x (4 PPT) pixel blocks (two across, 4 / PPT down), lane l owns
// pixels (l % 8, l / 8 + 4 k), k < PPT.  Per list index the PPT pairs of a
// thread are added into one gradient vector before the warp reduction.
template <bool SURF, bool PREFILTER, int N, int PPT, bool PACK, bool PL>
__global__ void __launch_bounds__(k3BlockSize / PPT, PPT == 2 ? 5 : 2)
    render3d_bwd_kernel(const Backward3DArgs a, const BwdLayout L) {
    constexpr int kThreads = k3BlockSize / PPT;
    constexpr int kBatch = kThreads;  // surfels staged per batch
    constexpr int kWarpRows = 4 * PPT;
    extern __shared__ __align__(16) unsigned char s_raw[];
    Surfel3D* s_prim = reinterpret_cast<Surfel3D*>(s_raw);
    float* s_acc = reinterpret_cast<float*>(s_raw + sizeof(Surfel3D) * kBatch);
    __shared__ int s_max_visit;
    // the staged records' pixel boxes, packed (the compaction reads one per lane)
    __shared__ short4 s_box[kBatch];
    // per warp: the batch slots whose pixel box meets the warp's block
    __shared__ unsigned char s_list[kThreads / 32][kBatch];
    // the forward's blend-mask bytes of the batch's list entries
    __shared__ unsigned char s_bm[kBatch];
    // per warp: the packed pairs of the list entry in hand (PACK)
    __shared__ PairRec s_pairs[PACK ? kThreads / 32 : 1][PACK ? 32 : 1];
    static_assert(!PACK || (N == 24 && !SURF && !PREFILTER), "packed pairs: plain RGB only");

    // N == 32 uses the fixed slot layout (compile-time indices keep the
    // gradient vector in registers); N == 64 takes the host-computed layout
    // of the quadratic colour and lobe view models.
    constexpr bool FIX = (N == 32);
    constexpr bool LITE = (N == 24);  // lite layout: slots absent from it are never touched
    BwdSlots O;
    O.cg = LITE ? kLiteCg : FIX ? kFixCg : L.off_cg;
    O.cq = (FIX || LITE) ? 0 : L.off_cq;
    O.op = LITE ? kLiteOp : FIX ? kFixOp : L.off_op;
    O.soft = LITE ? 0 : FIX ? kFixSoft : L.off_soft;
    O.tm = LITE ? kLiteTm : FIX ? kFixTm : L.off_tm;
    O.vd = LITE ? 0 : FIX ? kFixVd : L.off_vd;
    O.n = LITE ? 0 : FIX ? kFixN : L.off_n;
    O.ks = (FIX || LITE) ? 0 : L.off_ks;
    O.ls = (FIX || LITE) ? 0 : L.off_ls;
    O.abs = LITE ? 0 : FIX ? kFixAbs : L.off_abs;
    O.ctr = LITE ? 0 : FIX ? kFixCtr : L.off_ctr;

    const int W = a.W, H = a.H;
    const unsigned hblocks = (W + k3BlockX - 1) / k3BlockX;
    const int tr = threadIdx.x;
    const int lane = tr & 31;
    const int warp = tr >> 5;
    const int wx0 = (int)(blockIdx.x * k3BlockX) + ((warp & 1) << 3);
    const int wy0 = (int)(blockIdx.y * k3BlockY) + (warp >> 1) * kWarpRows;
    const int HW = H * W;
    const unsigned my_bits = blend_bits(warp, PPT);

    uint2 range = a.ranges[blockIdx.y * hblocks + blockIdx.x];
    range.y = min(range.y, (unsigned)a.num_rendered);
    range.x = min(range.x, range.y);
    const int range_len = (int)(range.y - range.x);
    if (range_len <= 0) return;  // uniform across the CTA

    BwdPixel q[PPT];
    int n_max = 0;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        const int pxi = wx0 + (lane & 7);
        const int pyi = wy0 + (lane >> 3) + 4 * k;
        const bool inside = pxi < W && pyi < H;
        const int pix = pyi * W + pxi;
        BwdPixel& p = q[k];
        p.px = (float)pxi;
        p.py = (float)pyi;
        p.v_r = p.v_g = p.v_b = p.v_overdraw = 0.f;
        p.T_after = 1.f;
        p.behind = {a.bg[0], a.bg[1], a.bg[2]};
        p.n_color = 0;
        p.v_depth = p.v_alpha = p.v_dist = p.v_median = 0.f;
        p.v_normal = {0.f, 0.f, 0.f};
        p.T_after_surf = 1.f;
        p.M1 = p.M2 = 0.f;
        p.last_dist_vjp = 0.f;
        p.behind_depth = p.behind_alpha = 0.f;
        p.behind_normal = {0.f, 0.f, 0.f};
        p.n_surf = 0;
        p.median_index = -1;
        if (inside) {
            p.v_r = a.grad_out_color[pix];
            p.v_g = a.grad_out_color[HW + pix];
            p.v_b = a.grad_out_color[2 * HW + pix];
            if (a.grad_out_overdraw) p.v_overdraw = a.grad_out_overdraw[pix];
            p.T_after = a.final_T[pix];
            p.n_color = min(a.last_index[pix], range_len);
            if (SURF) {
                if (a.grad_out_surf_depth) p.v_depth = a.grad_out_surf_depth[pix];
                if (a.grad_out_surf_alpha) p.v_alpha = a.grad_out_surf_alpha[pix];
                if (a.grad_out_surf_normals) {
                    p.v_normal = {a.grad_out_surf_normals[pix],
                                  a.grad_out_surf_normals[HW + pix],
                                  a.grad_out_surf_normals[2 * HW + pix]};
                    p.v_dist = a.grad_out_surf_normals[3 * HW + pix];
                    if (a.has_median_grad) p.v_median = a.grad_out_surf_normals[4 * HW + pix];
                }
                p.T_after_surf = a.final_T_surf[pix];
                p.n_surf = min(a.last_index_surf[pix], range_len);
                p.M1 = a.m1_surf[pix];
                p.M2 = a.m2_surf[pix];
                p.median_index = a.median_index[pix];
            }
        }
        p.final_alpha_surf = 1.0f - p.T_after_surf;
        n_max = max(n_max, SURF ? max(p.n_color, p.n_surf) : p.n_color);
    }
    if (tr == 0) s_max_visit = 0;
    __syncthreads();
    if (n_max > 0) atomicMax(&s_max_visit, n_max);
    __syncthreads();
    const int block_max = s_max_visit;
    // list entries at or past every one of this warp's last indices change
    // nothing for the warp: it starts its walk below them
    const int warp_max = __reduce_max_sync(0xffffffffu, n_max);

    const int nb = (block_max + kBatch - 1) / kBatch;
    for (int b = nb - 1; b >= 0; --b) {
        const int bstart = b * kBatch;
        const int bend = min(bstart + kBatch, block_max);
        __syncthreads();
        for (int t = tr; bstart + t < bend; t += kThreads) {
            int g = a.point_list[range.x + bstart + t];
            g = min(max(g, 0), a.P - 1);
            s_bm[t] = a.blend_mask ? a.blend_mask[range.x + bstart + t] : (unsigned char)0xff;
            if (a.records) {
                stage_record_async(a.records, g, &s_prim[t]);
                cp_async_wait_all();  // this thread's own row: its box is read next
                s_box[t] = PREFILTER ? make_short4(-32768, -32768, 32767, 32767)
                                     : s_prim[t].q.box;
            } else {
                s_box[t] = stage_surfel<SURF, PREFILTER>(a, g, W, H, &s_prim[t]);
            }
        }
        for (int t = tr; t < kBatch * L.ncomp; t += kThreads) s_acc[t] = 0.f;
        __syncthreads();

        // compact the batch slots below this warp's pixels' last indices to the
        // surfels whose box meets the warp's block and whose blend-mask bits
        // for the block are set: no pixel of the block blends any other, so
        // nothing of those pairs changes there
        const int n_slots = min(bend, warp_max) - bstart;
        int n_mine = 0;
        for (int base = 0; base < n_slots; base += 32) {
            const int t = base + lane;
            const bool hit = t < n_slots && (s_bm[t] & my_bits) != 0u &&
                             (PREFILTER || !box_misses(s_box[t], wx0, wy0, wx0 + 7,
                                                       wy0 + kWarpRows - 1));
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (hit) s_list[warp][n_mine + __popc(m & ((1u << lane) - 1u))] = (unsigned char)t;
            n_mine += __popc(m);
        }
        __syncwarp();
        // PACK: an entry of at most 16 pairs held in the first half of the
        // pair buffer until the next one (or the end of the batch)
        int pend_idx = -1, pend_n = 0;
        for (int jj = n_mine - 1; jj >= 0; --jj) {
            const int idx = bstart + s_list[warp][jj];
            const Surfel3D& s = s_prim[idx - bstart];
            if constexpr (PACK) {
                // per-pixel part in list order, then the blended pairs packed
                // one per lane for the VJP
                const unsigned bm = s_bm[idx - bstart];
                PairRec rec[PPT];
                unsigned m[PPT];
                int n_pairs = 0;
#pragma unroll
                for (int k = 0; k < PPT; ++k) {
                    bool bl = false;
                    if (bm & (1u << (2 * ((warp >> 1) * PPT + k) + (warp & 1))))
                        bl = rgb_pair_forward(a, s, idx, q[k], rec[k]);
                    m[k] = __ballot_sync(0xffffffffu, bl);
                    rec[k].b.w = __int_as_float(lane | (k << 5));
                    n_pairs += __popc(m[k]);
                }
                if (n_pairs == 0) continue;
                if (n_pairs <= 16) {
                    // packed into one half of the warp's pair buffer; two such
                    // entries share one VJP pass and one half-warp reduction
                    // (the per-pixel part above never reads their result)
                    const int off = pend_idx >= 0 ? 16 : 0;
                    if (off == 0) __syncwarp();  // the buffer's last reads are done
                    pack_pairs<PPT>(m, rec, lane, &s_pairs[warp][off]);
                    if (pend_idx < 0) {
                        pend_idx = idx;
                        pend_n = n_pairs;
                        continue;
                    }
                    __syncwarp();
                    const bool hi = lane >= 16;
                    const int e_idx = hi ? idx : pend_idx;
                    float acc[24];
#pragma unroll
                    for (int c = 0; c < 24; ++c) acc[c] = 0.f;
                    if ((lane & 15) < (hi ? n_pairs : pend_n))
                        packed_pair_vjp(s_prim[e_idx - bstart], s_pairs[warp][lane], wx0, wy0,
                                        acc);
                    const int start = half_warp_reduce_scatter24(acc, lane);
                    float* dst = s_acc + (e_idx - bstart) * kLiteComp;
                    const bool odd = (lane & 1) != 0;
                    const int comp = start + (odd ? 2 : 0);
                    const float val = odd ? acc[2] : acc[0];
                    if (comp < kLiteComp && val != 0.f) atomicAdd(dst + comp, val);
                    if (!odd && start + 1 < kLiteComp && acc[1] != 0.f)
                        atomicAdd(dst + start + 1, acc[1]);
                    pend_idx = -1;
                    continue;
                }
                if (pend_idx >= 0) {  // the held entry goes alone
                    __syncwarp();
                    float acc[24];
#pragma unroll
                    for (int c = 0; c < 24; ++c) acc[c] = 0.f;
                    if (lane < pend_n)
                        packed_pair_vjp(s_prim[pend_idx - bstart], s_pairs[warp][lane], wx0, wy0,
                                        acc);
                    const int start = warp_reduce_scatter24(acc, lane);
                    put_reduced24(s_acc + (pend_idx - bstart) * kLiteComp, acc, start, lane);
                    pend_idx = -1;
                }
                float acc[24];
#pragma unroll
                for (int c = 0; c < 24; ++c) acc[c] = 0.f;
                int halves = 0;
#pragma unroll
                for (int k = 0; k < PPT; ++k) halves += m[k] != 0u;
                if (halves > 1 && n_pairs <= 32) {
                    // pairs of both halves: packed one per lane (one pass)
                    __syncwarp();  // the previous entry's pairs have been read
                    pack_pairs<PPT>(m, rec, lane, &s_pairs[warp][0]);
                    __syncwarp();
                    if (lane < n_pairs)
                        packed_pair_vjp(s, s_pairs[warp][lane], wx0, wy0, acc);
                } else {
                    // more than a warp of pairs, or (never with 16 or fewer)
                    // one half holding every pair: each lane takes its own
#pragma unroll
                    for (int k = 0; k < PPT; ++k)
                        if (m[k] != 0u && (m[k] & (1u << lane)))
                            rgb_pair_vjp(s, rec[k], q[k].px, q[k].py, acc);
                }
                // (shared-memory atomics straight from the few lanes holding
                // pairs measured slower than this reduction even for one pair)
                const int start = warp_reduce_scatter24(acc, lane);
                put_reduced24(s_acc + (idx - bstart) * kLiteComp, acc, start, lane);
            } else {
            float acc[N];
#pragma unroll
            for (int c = 0; c < N; ++c) acc[c] = 0.f;
            bool contributed = false;
            // the mask has one bit per 8x4 half of the block: a half whose
            // bit is clear blends nothing of this entry (warp-uniform skip)
            const unsigned bm = s_bm[idx - bstart];
#pragma unroll
            for (int k = 0; k < PPT; ++k)
                if (bm & (1u << (2 * ((warp >> 1) * PPT + k) + (warp & 1))))
                    contributed |= bwd_pair<SURF, PREFILTER, N, PL>(a, L, O, s, idx, q[k], acc);
            if (__any_sync(0xffffffffu, contributed)) {
                float* dst = s_acc + (idx - bstart) * L.ncomp;
                if constexpr (N == 24) {
                    const int start = warp_reduce_scatter24(acc, lane);
                    const int c = lane & 3;  // lanes 0-2 of each group of 4 write
                    const float val = c == 0 ? acc[0] : (c == 1 ? acc[1] : acc[2]);
                    const int comp = start + c;
                    if (c < 3 && comp < L.ncomp && val != 0.f) atomicAdd(dst + comp, val);
                } else {
                    const int start = warp_reduce_scatter<N>(acc, lane);
#pragma unroll
                    for (int c = 0; c < N / 32; ++c) {
                        const int comp = start + c;
                        if (comp < L.ncomp && acc[c] != 0.f) atomicAdd(dst + comp, acc[c]);
                    }
                }
            }
            }
        }
        if (PACK && pend_idx >= 0) {  // the batch's last held entry goes alone
            __syncwarp();
            float acc[24];
#pragma unroll
            for (int c = 0; c < 24; ++c) acc[c] = 0.f;
            if (lane < pend_n)
                packed_pair_vjp(s_prim[pend_idx - bstart], s_pairs[warp][lane], wx0, wy0, acc);
            const int start = warp_reduce_scatter24(acc, lane);
            put_reduced24(s_acc + (pend_idx - bstart) * kLiteComp, acc, start, lane);
        }
        __syncthreads();
        // Flush this batch: one global atomic per (surfel, non-zero component).
        for (int t = tr; bstart + t < bend; t += kThreads) {
            const Surfel3D& s = s_prim[t];
            const int g = s.id;
            const float* sa = s_acc + t * L.ncomp;
            auto put = [](float* p, float v) {
                if (v != 0.f) atomicAdd(p, v);
            };
            put(a.grad_colors + 3 * g + 0, sa[0]);
            put(a.grad_colors + 3 * g + 1, sa[1]);
            put(a.grad_colors + 3 * g + 2, sa[2]);
            if (L.off_cg >= 0 && a.grad_color_grads)
                for (int c = 0; c < 6; ++c) put(a.grad_color_grads + 6 * g + c, sa[L.off_cg + c]);
            if (L.off_cq >= 0 && a.grad_color_quads)
                for (int c = 0; c < 9; ++c) put(a.grad_color_quads + 9 * g + c, sa[L.off_cq + c]);
            put(a.grad_opacities + g, sa[L.off_op]);
            if (L.off_soft >= 0) {
                if (a.softness_stride == 3)
                    for (int c = 0; c < 3; ++c) put(a.grad_softnesses + 3 * g + c, sa[L.off_soft + c]);
                else
                    put(a.grad_softnesses + g, sa[L.off_soft]);
            }
            for (int c = 0; c < 9; ++c) put(a.grad_transMats + 9 * g + c, sa[L.off_tm + c]);
            if (L.off_n >= 0)
                for (int c = 0; c < 3; ++c) put(a.grad_normals + 3 * g + c, sa[L.off_n + c]);
            if (L.off_ks >= 0)
                for (int c = 0; c < 3; ++c) put(a.grad_specular_ks + 3 * g + c, sa[L.off_ks + c]);
            if (L.off_ls >= 0) put(a.grad_specular_log_s + g, sa[L.off_ls]);
            if (L.off_abs >= 0) put(a.abs_means2d + 4 * g + 3, sa[L.off_abs]);
            if (L.off_ctr >= 0) {
                put(&a.grad_points_xy_center[g].x, sa[L.off_ctr]);
                put(&a.grad_points_xy_center[g].y, sa[L.off_ctr + 1]);
            }
            float vd_acc[3] = {0.f, 0.f, 0.f};
            if (L.off_vd >= 0)
                for (int c = 0; c < 3; ++c) vd_acc[c] = sa[L.off_vd + c];
            if (L.derive_vg || L.derive_vd) {
                const float* vd = a.view_dirs + 3 * g;
                const float* vg = a.view_grads + 9 * g;
                if (L.derive_vg) {
                    for (int c = 0; c < 3; ++c)
                        for (int r = 0; r < 3; ++r)
                            put(a.grad_view_grads + 9 * g + 3 * c + r, sa[c] * vd[r]);
                }
                if (L.derive_vd) {
                    for (int r = 0; r < 3; ++r)
                        vd_acc[r] += sa[0] * vg[r] + sa[1] * vg[3 + r] + sa[2] * vg[6 + r];
                }
            }
            if (L.off_vd >= 0 || L.derive_vd)
                for (int r = 0; r < 3; ++r) put(a.grad_view_dirs + 3 * g + r, vd_acc[r]);
        }
    }
}

// ---------------------------------------------------------------------------
// Geometry VJPs (hexels3d_forward.cu:2494-2664)
// ---------------------------------------------------------------------------
namespace {

__device__ __forceinline__ Cmat<4, 4> w2n_of(const float* pm) {
    Cmat<4, 4> m;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) m.m[c][r] = pm[4 * r + c];
    return m;
}

__device__ __forceinline__ Cmat<3, 4> n2p_of(int W, int H) {
    Cmat<3, 4> m;
    m.m[0][0] = (float)W / 2.0f; m.m[0][1] = 0.0f; m.m[0][2] = 0.0f;
    m.m[0][3] = ((float)W - 1.0f) / 2.0f;
    m.m[1][0] = 0.0f; m.m[1][1] = (float)H / 2.0f; m.m[1][2] = 0.0f;
    m.m[1][3] = ((float)H - 1.0f) / 2.0f;
    m.m[2][0] = 0.0f; m.m[2][1] = 0.0f; m.m[2][2] = 0.0f; m.m[2][3] = 1.0f;
    return m;
}

// Quaternion VJP through the normalised rotation matrix; the result is
// projected onto the tangent space of the normalisation.
__device__ __forceinline__ float4 quat_vjp(const float4 q, const Cmat<3, 3>& vR) {
    const float s = rsqrtf(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    const float w = q.x * s, x = q.y * s, y = q.z * s, z = q.w * s;
    float4 g;
    g.x = 2.f * (x * (vR.m[1][2] - vR.m[2][1]) + y * (vR.m[2][0] - vR.m[0][2]) +
                 z * (vR.m[0][1] - vR.m[1][0]));
    g.y = 2.f * (-2.f * x * (vR.m[1][1] + vR.m[2][2]) + y * (vR.m[0][1] + vR.m[1][0]) +
                 z * (vR.m[0][2] + vR.m[2][0]) + w * (vR.m[1][2] - vR.m[2][1]));
    g.z = 2.f * (x * (vR.m[0][1] + vR.m[1][0]) - 2.f * y * (vR.m[0][0] + vR.m[2][2]) +
                 z * (vR.m[1][2] + vR.m[2][1]) + w * (vR.m[2][0] - vR.m[0][2]));
    g.w = 2.f * (x * (vR.m[0][2] + vR.m[2][0]) + y * (vR.m[1][2] + vR.m[2][1]) -
                 2.f * z * (vR.m[0][0] + vR.m[1][1]) + w * (vR.m[0][1] - vR.m[1][0]));
    const float4 qu = {q.x * s, q.y * s, q.z * s, q.w * s};
    const float dq = qu.x * g.x + qu.y * g.y + qu.z * g.z + qu.w * g.w;
    return {s * (g.x - qu.x * dq), s * (g.y - qu.y * dq), s * (g.z - qu.z * dq),
            s * (g.w - qu.w * dq)};
}

__device__ __forceinline__ float3 dnormvdv3(const float3 v, const float3 dv) {
    const float sum2 = v.x * v.x + v.y * v.y + v.z * v.z + 1e-8f;
    const float invsum32 = rsqrtf(sum2 * sum2 * sum2);
    return {((sum2 - v.x * v.x) * dv.x - v.y * v.x * dv.y - v.z * v.x * dv.z) * invsum32,
            (-v.x * v.y * dv.x + (sum2 - v.y * v.y) * dv.y - v.z * v.y * dv.z) * invsum32,
            (-v.x * v.z * dv.x - v.y * v.z * dv.y + (sum2 - v.z * v.z) * dv.z) * invsum32};
}

}  // namespace

__global__ void __launch_bounds__(256) geometry3d_bwd_kernel(
    int P, const float* __restrict__ means3d, const float2* __restrict__ scales, float mod,
    const float4* __restrict__ rotations, const float* __restrict__ projmatrix,
    const float* __restrict__ campos, int W, int H, const int* __restrict__ radii,
    const float* __restrict__ grad_T, const float* __restrict__ grad_view_dirs,
    const float* __restrict__ grad_normals, float* __restrict__ grad_means3d,
    float2* __restrict__ grad_scales, float4* __restrict__ grad_rotations, bool accumulate) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= P) return;
    if (radii[idx] <= 0) return;
    const float3 p = {means3d[3 * idx], means3d[3 * idx + 1], means3d[3 * idx + 2]};
    const float4 q = rotations[idx];
    const float2 sc = scales[idx];
    const Cmat<3, 3> R = quat_to_rotmat_wxyz(q);
    const Cmat<3, 4> Pm = mmul<3, 4, 4>(w2n_of(projmatrix), n2p_of(W, H));
    Cmat<3, 3> vT;
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int r = 0; r < 3; ++r) vT.m[c][r] = grad_T[9 * idx + 3 * c + r];
    const Cmat<3, 4> vM = mmul<3, 3, 4>(Pm, mtranspose<3, 3>(vT));
    float3 v_mean = {vM.m[2][0], vM.m[2][1], vM.m[2][2]};
    const float3 d = {p.x - campos[0], p.y - campos[1], p.z - campos[2]};
    const float3 vvd = {grad_view_dirs[3 * idx], grad_view_dirs[3 * idx + 1],
                        grad_view_dirs[3 * idx + 2]};
    const float3 v_d = dnormvdv3(d, vvd);
    v_mean.x += v_d.x;
    v_mean.y += v_d.y;
    v_mean.z += v_d.z;
    if (accumulate) {
        grad_means3d[3 * idx] += v_mean.x;
        grad_means3d[3 * idx + 1] += v_mean.y;
        grad_means3d[3 * idx + 2] += v_mean.z;
    } else {
        grad_means3d[3 * idx] = v_mean.x;
        grad_means3d[3 * idx + 1] = v_mean.y;
        grad_means3d[3 * idx + 2] = v_mean.z;
    }
    float3 vR2 = {0.f, 0.f, 0.f};
    if (grad_normals) {
        vR2.x += grad_normals[3 * idx];
        vR2.y += grad_normals[3 * idx + 1];
        vR2.z += grad_normals[3 * idx + 2];
    }
    Cmat<3, 3> vR;
    const float s0 = mod * sc.x, s1 = mod * sc.y;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        vR.m[0][r] = vM.m[0][r] * s0;
        vR.m[1][r] = vM.m[1][r] * s1;
    }
    vR.m[2][0] = vR2.x;
    vR.m[2][1] = vR2.y;
    vR.m[2][2] = vR2.z;
    const float4 v_rot = quat_vjp(q, vR);
    const float2 v_scale = {
        (vM.m[0][0] * R.m[0][0] + vM.m[0][1] * R.m[0][1] + vM.m[0][2] * R.m[0][2]) * mod,
        (vM.m[1][0] * R.m[1][0] + vM.m[1][1] * R.m[1][1] + vM.m[1][2] * R.m[1][2]) * mod};
    if (accumulate) {
        const float4 r0 = grad_rotations[idx];
        const float2 s0 = grad_scales[idx];
        grad_rotations[idx] = {r0.x + v_rot.x, r0.y + v_rot.y, r0.z + v_rot.z, r0.w + v_rot.w};
        grad_scales[idx] = {s0.x + v_scale.x, s0.y + v_scale.y};
    } else {
        grad_rotations[idx] = v_rot;
        grad_scales[idx] = v_scale;
    }
}

__global__ void __launch_bounds__(256) means2d3d_bwd_kernel(int P, int W, int H, int stride,
                                                            const int* __restrict__ radii,
                                                            const float* __restrict__ transMats,
                                                            const float* __restrict__ grad_T,
                                                            float* __restrict__ grad_means2d,
                                                            bool accumulate) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= P) return;
    if (radii[idx] <= 0) return;
    const float depth = transMats[9 * idx + 8];
    const float gx = grad_T[9 * idx + 2] * depth * 0.5f * (float)W;
    const float gy = grad_T[9 * idx + 5] * depth * 0.5f * (float)H;
    if (accumulate) {
        grad_means2d[idx * stride + 0] += gx;
        grad_means2d[idx * stride + 1] += gy;
    } else {
        grad_means2d[idx * stride + 0] = gx;
        grad_means2d[idx * stride + 1] = gy;
        grad_means2d[idx * stride + 2] = 0.f;
    }
}

__global__ void __launch_bounds__(256) center3d_bwd_kernel(int P, const float* __restrict__ means3d,
                                                           const float* __restrict__ pm, int W,
                                                           int H, const float2* __restrict__ gc,
                                                           float* __restrict__ grad_means3d) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= P) return;
    const float2 v_pix = gc[idx];
    if (v_pix.x == 0.f && v_pix.y == 0.f) return;
    const float x = means3d[3 * idx], y = means3d[3 * idx + 1], z = means3d[3 * idx + 2];
    const float clip_x = pm[0] * x + pm[4] * y + pm[8] * z + pm[12];
    const float clip_y = pm[1] * x + pm[5] * y + pm[9] * z + pm[13];
    const float clip_w = pm[3] * x + pm[7] * y + pm[11] * z + pm[15];
    const float inv_w = 1.0f / (clip_w + 1e-8f);
    const float inv_w2 = inv_w * inv_w;
    const float vx = v_pix.x * ((float)W / 2.0f);
    const float vy = v_pix.y * ((float)H / 2.0f);
    const float common = (vx * clip_x + vy * clip_y) * inv_w2;
    grad_means3d[3 * idx + 0] += (vx * inv_w * pm[0]) + (vy * inv_w * pm[1]) - (common * pm[3]);
    grad_means3d[3 * idx + 1] += (vx * inv_w * pm[4]) + (vy * inv_w * pm[5]) - (common * pm[7]);
    grad_means3d[3 * idx + 2] += (vx * inv_w * pm[8]) + (vy * inv_w * pm[9]) - (common * pm[11]);
}

}  // namespace hx

using namespace hx;

namespace {

template <bool SURF, bool PREFILTER, int N, int PPT, bool PACK, bool PL = false>
int launch_bwd3d(const Backward3DArgs& a, const BwdLayout& L, cudaStream_t stream) {
    constexpr int kBatch = k3BlockSize / PPT;
    const size_t smem = sizeof(Surfel3D) * kBatch + sizeof(float) * kBatch * L.ncomp;
    // the dynamic shared-memory limit is raised once per device (host threads
    // may launch concurrently: the flags are atomic)
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        HX_CUDA_TRY(cudaFuncSetAttribute(render3d_bwd_kernel<SURF, PREFILTER, N, PPT, PACK, PL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(sizeof(Surfel3D) * kBatch +
                                               sizeof(float) * kBatch * N)));
        if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    dim3 grid(ceil_div(a.W, k3BlockX), ceil_div(a.H, k3BlockY));
    render3d_bwd_kernel<SURF, PREFILTER, N, PPT, PACK, PL>
        <<<grid, k3BlockSize / PPT, smem, stream>>>(a, L);
    HX_LAUNCH_CHECK("render3d_bwd_kernel");
    return HX_OK;
}

// Two pixels per thread on the RGB path; one with surface gradients, whose
// larger per-pixel state costs more in occupancy (167 registers at two
// pixels) than the shared per-surfel work saves.  The plain-RGB layout
// without overdraw gradients (the training path) takes the packed pairs.
template <bool SURF, bool PREFILTER>
int launch_bwd3d_n(const Backward3DArgs& a, const BwdLayout& L, int slots,
                   cudaStream_t stream) {
    constexpr int kPPT = SURF ? 1 : 2;
    if constexpr (!SURF && !PREFILTER) {
        if (slots == 24 && a.grad_out_overdraw == nullptr)
            return launch_bwd3d<false, false, 24, kPPT, true>(a, L, stream);
        if (slots == 24) return launch_bwd3d<false, false, 24, kPPT, false>(a, L, stream);
    }
    if constexpr (!PREFILTER) {
        if (slots == 32 && a.color_model == kColorLinear && a.view_model == kViewLinear &&
            a.use_view_grads && a.softness_stride == 1 && a.overdraw_base >= a.P &&
            !a.grad_out_overdraw && L.off_cg >= 0 && L.off_cq < 0 && L.off_soft < 0 &&
            L.off_vd < 0 && L.off_ks < 0 && L.off_ls < 0)
            return launch_bwd3d<SURF, false, 32, kPPT, false, true>(a, L, stream);
    }
    if (slots <= 32) return launch_bwd3d<SURF, PREFILTER, 32, kPPT, false>(a, L, stream);
    return launch_bwd3d<SURF, PREFILTER, 64, kPPT, false>(a, L, stream);
}

}  // namespace

extern "C" int hx_hexels3d_render_backward(
    int P, int num_rendered, const int32_t* ranges, const int32_t* point_list,
    const float* points_xy_center, float* grad_points_xy_center, int image_width,
    int image_height, const float* colors, const float* color_grads, const float* color_quads,
    const float* view_grads, const float* specular_ks, const float* specular_log_s,
    int view_model, const float* view_dirs, const float* transMats, const float* opacities,
    const float* softnesses, int softness_stride, const float* background,
    const float* grad_out_color, const float* grad_out_overdraw,
    const float* grad_out_surf_depth, const float* grad_out_surf_alpha,
    const float* grad_out_surf_normals, int has_median_grad, const float* normals,
    float* grad_colors, float* grad_color_grads, float* grad_color_quads, float* grad_view_grads,
    float* grad_specular_ks, float* grad_specular_log_s, float* grad_opacities,
    float* grad_softnesses, float* grad_transMats, float* abs_means2d, float* grad_view_dirs,
    float* grad_normals, int overdraw_base_count, int color_model, int use_view_grads,
    const float* final_T, const int32_t* last_index, const float* final_T_surf,
    const int32_t* last_index_surf, const float* m1_surf, const float* m2_surf,
    const int32_t* median_index, const uint8_t* blend_mask, const void* records,
    cudaStream_t stream) {
    HX_REQUIRE((uintptr_t)records % 16 == 0, "records must start on a 16-byte boundary");
    HX_REQUIRE(image_width > 0 && image_height > 0, "invalid image dimensions");
    HX_REQUIRE(color_model >= 0 && color_model <= 3, "color_model must be 0..3");
    HX_REQUIRE(view_model >= 0 && view_model <= 2, "view_model must be 0..2");
    HX_REQUIRE(softness_stride == 1 || softness_stride == 3, "softness_stride must be 1 or 3");
    if (num_rendered == 0 || P == 0) return HX_OK;
    HX_REQUIRE(ranges && point_list && colors && view_dirs && transMats && opacities &&
                   softnesses && background && grad_out_color && grad_colors &&
                   grad_opacities && grad_transMats && grad_view_dirs && final_T && last_index,
               "hexels3d_render_backward: null pointer");
    const bool surf = grad_out_surf_depth || grad_out_surf_alpha || grad_out_surf_normals;
    HX_REQUIRE(!surf || (final_T_surf && last_index_surf && m1_surf && m2_surf && median_index),
               "surface gradients need the forward's saved surface state");
    const bool prefilter = points_xy_center != nullptr;
    HX_REQUIRE(!prefilter || grad_points_xy_center, "prefilter needs grad_points_xy_center");
    Backward3DArgs a = {};
    a.ranges = (const uint2*)ranges;
    a.point_list = point_list;
    a.num_rendered = num_rendered;
    a.P = P;
    a.points_xy_center = (const float2*)points_xy_center;
    a.grad_points_xy_center = (float2*)grad_points_xy_center;
    a.W = image_width;
    a.H = image_height;
    a.colors = colors;
    a.color_grads = color_grads;
    a.color_quads = color_quads;
    a.view_grads = view_grads;
    a.specular_ks = specular_ks;
    a.specular_log_s = specular_log_s;
    a.view_model = view_model;
    a.view_dirs = view_dirs;
    a.transMats = transMats;
    a.opacities = opacities;
    a.softnesses = softnesses;
    a.softness_stride = softness_stride;
    a.bg = background;
    a.grad_out_color = grad_out_color;
    a.grad_out_overdraw = grad_out_overdraw;
    a.grad_out_surf_depth = grad_out_surf_depth;
    a.grad_out_surf_alpha = grad_out_surf_alpha;
    a.grad_out_surf_normals = grad_out_surf_normals;
    a.has_median_grad = has_median_grad != 0;
    a.normals = normals;
    a.grad_colors = grad_colors;
    a.grad_color_grads = grad_color_grads;
    a.grad_color_quads = grad_color_quads;
    a.grad_view_grads = grad_view_grads;
    a.grad_specular_ks = grad_specular_ks;
    a.grad_specular_log_s = grad_specular_log_s;
    a.grad_opacities = grad_opacities;
    a.grad_softnesses = grad_softnesses;
    a.grad_transMats = grad_transMats;
    a.abs_means2d = abs_means2d;
    a.grad_view_dirs = grad_view_dirs;
    a.grad_normals = grad_normals;
    a.overdraw_base = (overdraw_base_count <= 0 || overdraw_base_count > P) ? P : overdraw_base_count;
    a.color_model = color_model;
    a.use_view_grads = use_view_grads != 0;
    a.final_T = final_T;
    a.last_index = last_index;
    a.final_T_surf = final_T_surf;
    a.last_index_surf = last_index_surf;
    a.m1_surf = m1_surf;
    a.m2_surf = m2_surf;
    a.median_index = median_index;
    a.blend_mask = blend_mask;
    a.records = (const Surfel3D*)records;

    BwdLayout L;
    const bool explicit_vd = view_model == 2 || (use_view_grads && prefilter);
    const bool generic = color_model >= 2 || view_model == 2;
    const bool lite = !generic && !grad_softnesses && !explicit_vd && !grad_normals &&
                      !abs_means2d && !prefilter && !surf;
    int slots = generic ? 64 : 32;
    if (lite) {
        slots = 24;
        L.off_cg = (color_model >= 1 && grad_color_grads) ? kLiteCg : -1;
        L.off_cq = -1;
        L.off_op = kLiteOp;
        L.off_soft = -1;
        L.off_tm = kLiteTm;
        L.off_vd = -1;
        L.off_n = -1;
        L.off_ks = -1;
        L.off_ls = -1;
        L.off_abs = -1;
        L.off_ctr = -1;
        L.ncomp = kLiteComp;
    } else if (!generic) {
        L.off_cg = (color_model >= 1 && grad_color_grads) ? kFixCg : -1;
        L.off_cq = -1;
        L.off_op = kFixOp;
        L.off_soft = grad_softnesses ? kFixSoft : -1;
        L.off_tm = kFixTm;
        L.off_vd = explicit_vd ? kFixVd : -1;
        L.off_n = grad_normals ? kFixN : -1;
        L.off_ks = -1;
        L.off_ls = -1;
        L.off_abs = abs_means2d ? kFixAbs : -1;
        L.off_ctr = prefilter ? kFixCtr : -1;
        L.ncomp = kFixComp;
    } else {
        int off = 3;
        L.off_cg = (color_model >= 1 && grad_color_grads) ? off : -1;
        off += L.off_cg >= 0 ? 6 : 0;
        L.off_cq = (color_model >= 2 && grad_color_quads) ? off : -1;
        off += L.off_cq >= 0 ? 9 : 0;
        L.off_op = off++;
        L.off_soft = grad_softnesses ? off : -1;
        off += grad_softnesses ? 3 : 0;
        L.off_tm = off;
        off += 9;
        L.off_vd = explicit_vd ? off : -1;
        off += explicit_vd ? 3 : 0;
        L.off_n = grad_normals ? off : -1;
        off += grad_normals ? 3 : 0;
        L.off_ks = (view_model == 2 && grad_specular_ks) ? off : -1;
        off += L.off_ks >= 0 ? 3 : 0;
        L.off_ls = (view_model == 2 && grad_specular_log_s) ? off : -1;
        off += L.off_ls >= 0 ? 1 : 0;
        L.off_abs = abs_means2d ? off : -1;
        off += abs_means2d ? 1 : 0;
        L.off_ctr = prefilter ? off : -1;
        off += prefilter ? 2 : 0;
        L.ncomp = off;
    }
    L.derive_vg = use_view_grads && grad_view_grads;
    L.derive_vd = use_view_grads && !prefilter;
    HX_REQUIRE(L.ncomp <= 64, "internal: too many gradient components");
    HX_REQUIRE(!use_view_grads || view_grads, "view_grads required with use_view_grads");
    HX_REQUIRE(color_model < 1 || color_grads, "color_grads required for color_model >= 1");
    HX_REQUIRE(color_model < 2 || color_quads, "color_quads required for quadratic models");
    HX_REQUIRE(view_model != 2 || (specular_ks && specular_log_s), "lobe needs specular params");
    if (surf) return prefilter ? launch_bwd3d_n<true, true>(a, L, slots, stream)
                               : launch_bwd3d_n<true, false>(a, L, slots, stream);
    return prefilter ? launch_bwd3d_n<false, true>(a, L, slots, stream)
                     : launch_bwd3d_n<false, false>(a, L, slots, stream);
}

extern "C" int hx_hexels3d_geometry_backward(
    int P, int num_rendered, const float* means3d, const float* scales, float scale_modifier,
    const float* rotations, const float* projmatrix, const float* campos, int image_width,
    int image_height, const int32_t* radii, const float* transMats, const float* grad_transMats,
    const float* grad_view_dirs, const float* grad_normals, const float* grad_points_xy_center,
    float* grad_means3d, float* grad_means2d, int means2d_stride, float* grad_scales,
    float* grad_rotations, int accumulate, cudaStream_t stream) {
    HX_REQUIRE(P >= 0, "hexels3d_geometry_backward: bad P");
    if (P == 0 || num_rendered == 0) return HX_OK;
    HX_REQUIRE(means3d && scales && rotations && projmatrix && campos && radii &&
                   grad_transMats && grad_view_dirs && grad_means3d && grad_scales &&
                   grad_rotations,
               "hexels3d_geometry_backward: null pointer");
    // rotations are read and written as float4, scales as float2
    HX_REQUIRE(((uintptr_t)rotations | (uintptr_t)grad_rotations) % 16 == 0 &&
                   ((uintptr_t)scales | (uintptr_t)grad_scales) % 8 == 0,
               "hexels3d_geometry_backward: rotations (and their gradients) must start on a "
               "16-byte boundary, scales (and theirs) on an 8-byte boundary");
    const int blocks = ceil_div(P, 256);
    if (grad_means2d) {
        HX_REQUIRE(transMats && (means2d_stride == 3 || means2d_stride == 4),
                   "means2d stride must be 3 or 4");
        means2d3d_bwd_kernel<<<blocks, 256, 0, stream>>>(P, image_width, image_height,
                                                         means2d_stride, radii, transMats,
                                                         grad_transMats, grad_means2d,
                                                         accumulate != 0);
        HX_LAUNCH_CHECK("means2d3d_bwd_kernel");
    }
    geometry3d_bwd_kernel<<<blocks, 256, 0, stream>>>(
        P, means3d, (const float2*)scales, scale_modifier, (const float4*)rotations, projmatrix,
        campos, image_width, image_height, radii, grad_transMats, grad_view_dirs, grad_normals,
        grad_means3d, (float2*)grad_scales, (float4*)grad_rotations, accumulate != 0);
    HX_LAUNCH_CHECK("geometry3d_bwd_kernel");
    if (grad_points_xy_center) {
        center3d_bwd_kernel<<<blocks, 256, 0, stream>>>(P, means3d, projmatrix, image_width,
                                                        image_height,
                                                        (const float2*)grad_points_xy_center,
                                                        grad_means3d);
        HX_LAUNCH_CHECK("center3d_bwd_kernel");
    }
    return HX_OK;
}
