// S5: 2D image-hexel compositing — top-10 normalised weighted sum of
// hexagon-SDF sigmoid weights, forward and backward, for the four geometry x
// colour variants of the reference (scale+rotation or 2x2 affine; flat colour
// or linear colour gradient), each with scalar, per-primitive or per-edge
// softness, optional peak sharpness and emission.
//
// Per-pixel arithmetic follows gsplat/cuda/csrc/hexels_forward.cu:16-859 and
// hexels_backward.cu:11-1387 of the reference in the same order.  Changes of
// schedule, not of results:
//   * per-primitive terms that the reference recomputes for every pixel
//     (sincos of the rotation, scale + 1e-8, anti-aliasing factors, the
//     softness triplet) are computed once per primitive while staging the
//     batch into shared memory;
//   * one templated kernel serves all variants;
//   * the backward sums each parameter's partials over the lanes of a warp
//     that hold the same hexagon (a binary tree of shuffles) and adds one
//     global atomic per (warp, hexagon, component) instead of one per
//     (pixel, hexagon, component).
#include "hx_topk.cuh"

namespace hx {

namespace {

constexpr float kHexA = 0.5f * 1.7320508f;  // sqrt(3) / 2
constexpr float kHexB = 0.5f;
constexpr float kEntropyEps = 1e-7f;
constexpr double kEpsHex = 1e-4;  // EPS (config.h:9)

__device__ __forceinline__ float sigmoid_neg_dist(float dist, float softness) {
    const float x = dist * softness;
    return 1.f / (1.f + __expf(x));
}

__device__ __forceinline__ float sign_subgrad(float x) {
    return (x > 0.f) ? 1.f : ((x < 0.f) ? -1.f : 0.f);
}

// Pointy-top hexagon SDF: max(|v|, |a u + b v|, |a u - b v|) - 1, with the
// index of the active edge (ties prefer edge 2 over 1, and 1/2 over 0).
__device__ __forceinline__ float hex_sdf(float u, float v, int& edge) {
    const float d0 = fabsf(v);
    // hexels_forward.cu:31-32: a u fused, b v = v / 2 exact (the rounding the
    // reference's build gives these lines)
    const float t1 = __fmaf_rn(kHexA, u, kHexB * v);
    const float t2 = __fmaf_rn(kHexA, u, -(kHexB * v));
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

// Per-primitive terms staged in shared memory.
struct HexPrim {
    float x, y;      // centre (pixels)
    float g0, g1;    // cos, sin (scale/rot) | a00, a01 (affine)
    float g2, g3;    // sx + 1e-8, sy + 1e-8 | a10, a11
    float su, sv;    // anti-aliasing scale factors (1 when off)
    float s0, s1, s2;  // softness per edge
    float sharp;
    int id;
    int pad_;
};

__device__ __forceinline__ float3 load_softness(const float* softnesses, int stride,
                                                float dflt, int g) {
    if (softnesses == nullptr || stride <= 0) return make_float3(dflt, dflt, dflt);
    if (stride == 3) {
        const float* s = softnesses + g * 3;
        return make_float3(s[0], s[1], s[2]);
    }
    const float s = softnesses[g];
    return make_float3(s, s, s);
}

template <bool AFFINE>
__device__ __forceinline__ HexPrim make_prim(int g, const float2* xys, const float2* scales,
                                             const float* rotation, const float4* affines,
                                             float aa, const float* softnesses, int stride,
                                             float soft_dflt, const float* sharpness) {
    HexPrim p;
    const float2 xy = xys[g];
    p.x = xy.x;
    p.y = xy.y;
    p.su = 1.f;
    p.sv = 1.f;
    if (AFFINE) {
        const float4 a = affines[g];
        p.g0 = a.x;
        p.g1 = a.y;
        p.g2 = a.z;
        p.g3 = a.w;
        if (aa > 0.f) {
            const float inv_len_u2 = a.x * a.x + a.z * a.z;
            const float inv_len_v2 = a.y * a.y + a.w * a.w;
            p.su = rsqrtf(1.f + aa * inv_len_u2);
            p.sv = rsqrtf(1.f + aa * inv_len_v2);
        }
    } else {
        float s, c;
        sincosf(rotation[g], &s, &c);
        const float2 sc = scales[g];
        p.g0 = c;
        p.g1 = s;
        p.g2 = sc.x + 1e-8f;
        p.g3 = sc.y + 1e-8f;
        if (aa > 0.f) {
            const float inv_sx2 = 1.f / (p.g2 * p.g2);
            const float inv_sy2 = 1.f / (p.g3 * p.g3);
            p.su = rsqrtf(1.f + aa * inv_sx2);
            p.sv = rsqrtf(1.f + aa * inv_sy2);
        }
    }
    const float3 s3 = load_softness(softnesses, stride, soft_dflt, g);
    p.s0 = s3.x;
    p.s1 = s3.y;
    p.s2 = s3.z;
    p.sharp = sharpness ? sharpness[g] : 0.f;
    p.id = g;
    return p;
}

// Local hexagon coordinates of pixel offset delta = centre - pixel.
struct HexLocal {
    float u_rot, v_rot;    // rotated (scale/rot) — unused for affine
    float u_base, v_base;  // before anti-aliasing scale
    float u, v;            // final
};

template <bool AFFINE>
__device__ __forceinline__ HexLocal hex_local(const HexPrim& p, float dx, float dy) {
    HexLocal l;
    if (AFFINE) {
        l.u_rot = 0.f;
        l.v_rot = 0.f;
        l.u_base = dx * p.g0 + dy * p.g2;
        l.v_base = dx * p.g1 + dy * p.g3;
    } else {
        // The reference's expressions (hexels_forward.cu:62-63) with the
        // fused multiply-adds its fast-math build forms, written out so that
        // this build rounds the same way: weights tie-break the top-10 by
        // exact comparison, so one ulp here can reorder a pixel's slots.
        l.u_rot = __fmaf_rn(dy, p.g1, __fmul_rn(dx, p.g0));
        l.v_rot = __fmaf_rn(dy, p.g0, -__fmul_rn(dx, p.g1));
        l.u_base = l.u_rot / p.g2;
        l.v_base = l.v_rot / p.g3;
    }
    l.u = l.u_base * p.su;
    l.v = l.v_base * p.sv;
    return l;
}

__device__ __forceinline__ float edge_softness(const HexPrim& p, int edge) {
    return (edge == 0) ? p.s0 : ((edge == 1) ? p.s1 : p.s2);
}

template <bool AFFINE>
__device__ __forceinline__ float hex_alpha(const HexPrim& p, float dx, float dy, float& peak) {
    const HexLocal l = hex_local<AFFINE>(p, dx, dy);
    int edge;
    const float dist = hex_sdf(l.u, l.v, edge);
    float alpha = sigmoid_neg_dist(dist, edge_softness(p, edge));
    peak = 0.f;
    if (p.sharp > 0.f) {
        const float r2 = l.u * l.u + l.v * l.v;
        const float pk = __expf(-p.sharp * r2);
        peak = pk;
        alpha *= pk;
    }
    return alpha;
}

}  // namespace

struct HexFwdArgs {
    int tiles_x;
    int num_points;
    int num_intersects;
    unsigned img_w, img_h;
    int channels;
    const int* ids_sorted;
    const int2* tile_bins;
    const float2* xys;
    const float2* scales;
    const float* rotation;
    const float4* affines;
    const float* colors;
    const float* color_grads;
    float color_grad_scale;
    float aa;
    const float* softnesses;
    int softness_stride;
    float softness_default;
    const float* sharpness;
    const float* emission;
    float* out_img;
    int* pixel_topk;
    float* weights_sum;
    float* entropy;
};

// One thread per pixel over 16x16 tiles; the tile's candidates are staged
// batch by batch in shared memory and every pixel keeps the reference's
// top-10 (hexels_forward.cu:169-337): the first ten candidates fill slots
// 0..9 in order, after which a candidate whose weight exceeds the current
// minimum replaces the minimum's slot (lowest slot among equal minima).  Once
// the ten slots are full they stay full, so the reference's empty-slot test
// in the minimum scan never fires and is left out.  Slot ids and peaks live
// in shared memory ([slot][thread], conflict-free) so that a replacement is
// two stores; the weights stay in registers for the minimum scan.
template <bool AFFINE, bool CGRAD>
__global__ void __launch_bounds__(256) hexel_fwd_kernel(const HexFwdArgs a) {
    __shared__ HexPrim s_prim[kBlockSize];
    __shared__ int s_ids[kTopK][kBlockSize];
    __shared__ float s_peaks[kTopK][kBlockSize];
    const int tile_id = blockIdx.y * a.tiles_x + blockIdx.x;
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
    const int2 lp = tile_pixel16(tr);
    const unsigned i = blockIdx.y * kBlockY + lp.y;
    const unsigned j = blockIdx.x * kBlockX + lp.x;
    const float px = (float)j;
    const float py = (float)i;
    const int pix_id = i * a.img_w + j;
    const bool inside = (i < a.img_h && j < a.img_w);
    const int C = a.channels;

    int2 range = a.tile_bins[tile_id];
    range.y = min(range.y, a.num_intersects);
    range.x = max(0, min(range.x, range.y));
    if (range.x == range.y) {
        if (inside) {
            for (int c = 0; c < C; ++c) a.out_img[pix_id * C + c] = 0.f;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) a.pixel_topk[pix_id * kTopK + k] = -1;
            if (a.weights_sum) a.weights_sum[pix_id] = (float)kEpsHex;
            if (a.entropy) a.entropy[pix_id] = 0.f;
        }
        return;
    }

    float vals[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        vals[k] = 0.f;
        s_ids[k][tr] = -1;
        s_peaks[k][tr] = 0.f;
    }
    int min_id = 0;
    float min_val = -1.f;

    for (int batch_start = range.x; batch_start < range.y; batch_start += kBlockSize) {
        __syncthreads();
        const int idx = batch_start + tr;
        if (idx < range.y) {
            const int g = min(max(a.ids_sorted[idx], 0), a.num_points - 1);
            s_prim[tr] = make_prim<AFFINE>(g, a.xys, a.scales, a.rotation,
                                           a.affines, a.aa, a.softnesses, a.softness_stride,
                                           a.softness_default, a.sharpness);
        }
        __syncthreads();
        const int batch_size = min(kBlockSize, range.y - batch_start);
        if (inside) {
            for (int t = 0; t < batch_size; ++t) {
                const HexPrim& p = s_prim[t];
                float peak;
                const float alpha = hex_alpha<AFFINE>(p, p.x - px, p.y - py, peak);
                if (alpha > min_val) {
                    s_ids[min_id][tr] = p.id;
                    s_peaks[min_id][tr] = peak;
#pragma unroll
                    for (int k = 0; k < kTopK; ++k)
                        if (k == min_id) vals[k] = alpha;
                    if (min_val < 0.f && min_id + 1 < kTopK) {
                        ++min_id;
                    } else {
                        ArgMin<0, kTopK>::run(vals, min_id, min_val);
                    }
                }
            }
        }
    }
    if (!inside) return;

    int ids[kTopK];
    float peaks[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        ids[k] = s_ids[k][tr];
        peaks[k] = s_peaks[k][tr];
    }

    float sum_val = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k)
        if (ids[k] >= 0) sum_val += vals[k];
    const float denom = (float)((double)sum_val + kEpsHex);

    for (int c = 0; c < C; ++c) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int g = ids[k];
            if (g < 0) continue;
            const float vis = vals[k] / denom;
            if (CGRAD) {
                const float2 xy = a.xys[g];
                const float2 delta = {xy.x - px, xy.y - py};
                const float base = a.colors[g * C + c];
                const float gx = a.color_grads[(g * 2 + 0) * C + c];
                const float gy = a.color_grads[(g * 2 + 1) * C + c];
                const float color = base + a.color_grad_scale * (delta.x * gx + delta.y * gy);
                acc += color * vis;
            } else {
                acc += a.colors[g * C + c] * vis;
            }
        }
        if (a.emission) {
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const int g = ids[k];
                if (g < 0) continue;
                acc += a.emission[g * C + c] * peaks[k];
            }
        }
        a.out_img[pix_id * C + c] = acc;
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) a.pixel_topk[pix_id * kTopK + k] = ids[k];
    if (a.weights_sum) a.weights_sum[pix_id] = denom;
    if (a.entropy) {
        float ent = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            if (ids[k] < 0) continue;
            const float p = vals[k] / denom;
            ent += -p * logf(p + kEntropyEps);
        }
        a.entropy[pix_id] = ent;
    }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
struct HexBwdArgs {
    unsigned img_w, img_h;
    int channels;
    int num_points;
    const float2* xys;
    const float2* scales;
    const float* rotation;
    const float4* affines;
    const float* colors;
    const float* color_grads;
    float color_grad_scale;
    const float* emission;
    const float* v_output;
    const float* v_weights_sum;
    const float* v_entropy;
    const int* pixel_topk;
    float aa;
    const float* softnesses;
    int softness_stride;
    float softness_default;
    const float* sharpness;
    float* v_xy;
    float* v_scale;   // (N,2) scale/rot
    float* v_rot;     // (N,)  scale/rot
    float* v_affines; // (N,4) affine
    float* v_colors;
    float* v_color_grads;
    float* v_emission;
    float* v_sharpness;
    float* v_softnesses;
};

// One thread per pixel over 16x16 tiles (8x4 pixels per warp).  Pass 1 recomputes the stored ids'
// weights and the normalisation gradient of every slot; pass 2 computes each
// slot's partials for every parameter, sums them over the lanes of the warp
// that hold the same id (KeyTree) and adds each group's sum with one global
// atomic.  Every lane of a warp runs both passes (pixels outside the image or
// with no stored id contribute zeros) so that the warp-wide sums stay
// converged.
template <bool AFFINE, bool CGRAD>
__global__ void __launch_bounds__(256) hexel_bwd_kernel(const HexBwdArgs a) {
    __shared__ int s_id[kTopK][kBlockSize];
    __shared__ float s_alpha[kTopK][kBlockSize];
    __shared__ float s_vn[kTopK][kBlockSize];
    const int C = a.channels;
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
    const unsigned lane = tr & 31;
    const int2 lp = tile_pixel16(tr);
    const unsigned i = blockIdx.y * kBlockY + lp.y;
    const unsigned j = blockIdx.x * kBlockX + lp.x;
    const float px = (float)j;
    const float py = (float)i;
    const bool inside = (i < a.img_h && j < a.img_w);
    const int pix_id = min((int)(i * a.img_w + j), (int)(a.img_w * a.img_h - 1));
    const int* topk = a.pixel_topk + pix_id * kTopK;
    // Mirrors the reference's early exits: outside pixels and pixels whose
    // first slot is empty contribute nothing.
    const bool active = inside && topk[0] >= 0;
    const float* v_out = a.v_output + C * pix_id;

    // pass 1: weights of the stored ids, their sum, and the gradient of each
    // slot's normalised weight before normalisation (sum_c colour * v_out)
    float denom = (float)kEpsHex;
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k) {
        int g = active ? topk[k] : -1;
        if (g >= a.num_points) g = -1;
        float alpha = 0.f, v_norm_d = 0.f;
        if (g >= 0) {
            const HexPrim p = make_prim<AFFINE>(g, a.xys, a.scales, a.rotation, a.affines, a.aa,
                                                a.softnesses, a.softness_stride,
                                                a.softness_default, a.sharpness);
            float peak;
            alpha = hex_alpha<AFFINE>(p, p.x - px, p.y - py, peak);
            denom += alpha;
            const float dx = p.x - px, dy = p.y - py;
            for (int c = 0; c < C; ++c) {
                const float vo = v_out[c];
                if (CGRAD) {
                    const float base = a.colors[C * g + c];
                    const float gx = a.color_grads[(g * 2 + 0) * C + c];
                    const float gy = a.color_grads[(g * 2 + 1) * C + c];
                    const float color = base + a.color_grad_scale * (dx * gx + dy * gy);
                    v_norm_d += color * vo;
                } else {
                    v_norm_d += a.colors[C * g + c] * vo;
                }
            }
        }
        s_id[k][tr] = g;
        s_alpha[k][tr] = alpha;
        s_vn[k][tr] = v_norm_d;
    }
    float v_d_sum = 0.f;
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k)
        if (s_id[k][tr] >= 0) v_d_sum += -s_alpha[k][tr] / (denom * denom) * s_vn[k][tr];

    const float v_ws = (active && a.v_weights_sum) ? a.v_weights_sum[pix_id] : 0.f;
    const float v_ent = (active && a.v_entropy) ? a.v_entropy[pix_id] : 0.f;
    float ent_avg = 0.f;
    if (v_ent != 0.f) {
#pragma unroll 1
        for (int k = 0; k < kTopK; ++k) {
            if (s_id[k][tr] < 0) continue;
            const float p = s_alpha[k][tr] / denom;
            ent_avg += p * -(logf(p + kEntropyEps) + 1.f);
        }
    }

    // pass 2: per-parameter partials of every slot, summed per id over the warp
    const bool with_sharp = a.sharpness != nullptr && a.v_sharpness != nullptr;
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k) {
        const int g = s_id[k][tr];
        const bool valid = g >= 0;
        const KeyTree t = key_tree(lane, g);
        const bool lead = t.first && valid;
        const int gs = valid ? g : 0;  // a safe index for lanes without an id
        float geo[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float v_sharp = 0.f, v_soft = 0.f, norm_d = 0.f, dx = 0.f, dy = 0.f, peak = 0.f;
        int edge = 0;
        if (valid) {
            const HexPrim p = make_prim<AFFINE>(g, a.xys, a.scales, a.rotation, a.affines, a.aa,
                                                a.softnesses, a.softness_stride,
                                                a.softness_default, a.sharpness);
            const float2 delta = {p.x - px, p.y - py};
            dx = delta.x;
            dy = delta.y;
            const float alpha = s_alpha[k][tr];
            norm_d = alpha / denom;
            // gradient of this slot's raw weight: normalisation, then the
            // weight-sum and entropy statistics
            float v_d = s_vn[k][tr] / denom;
            v_d += v_d_sum;
            if (v_ws != 0.f) v_d += v_ws;
            if (v_ent != 0.f) {
                const float dhdp = -(logf(norm_d + kEntropyEps) + 1.f);
                v_d += v_ent * ((dhdp - ent_avg) / denom);
            }
            const HexLocal l = hex_local<AFFINE>(p, delta.x, delta.y);
            const float dist = hex_sdf(l.u, l.v, edge);
            // SDF partials w.r.t. (u, v); |.| has subgradient sign(0) = 0
            // (hexels_backward.cu:15-18, 100-128).
            float du, dv;
            if (edge == 0) {
                du = 0.f;
                dv = sign_subgrad(l.v);
            } else if (edge == 1) {
                const float s = sign_subgrad(kHexA * l.u + kHexB * l.v);
                du = kHexA * s;
                dv = kHexB * s;
            } else {
                const float s = sign_subgrad(kHexA * l.u - kHexB * l.v);
                du = kHexA * s;
                dv = -kHexB * s;
            }
            const float soft = edge_softness(p, edge);
            const float sig = sigmoid_neg_dist(dist, soft);
            float v_sig = v_d;
            float v_u_peak = 0.f, v_v_peak = 0.f;
            if (p.sharp > 0.f) {
                const float r2 = l.u * l.u + l.v * l.v;
                peak = __expf(-p.sharp * r2);
                v_sig = v_d * peak;
                float v_peak_emit = 0.f;
                if (a.v_emission && peak > 0.f)
                    for (int c = 0; c < C; ++c) v_peak_emit += a.emission[C * g + c] * v_out[c];
                const float v_peak = v_d * sig + v_peak_emit;
                const float v_r2 = v_peak * peak * (-p.sharp);
                v_u_peak = v_r2 * 2.f * l.u;
                v_v_peak = v_r2 * 2.f * l.v;
                v_sharp = v_peak * peak * (-r2);
            }
            v_soft = v_sig * (-dist) * sig * (1.f - sig);
            const float v_dist = v_sig * (-soft) * sig * (1.f - sig);
            float v_u = v_dist * du;
            float v_v = v_dist * dv;
            v_u += v_u_peak;
            v_v += v_v_peak;
            const float v_u_base = v_u * p.su;
            const float v_v_base = v_v * p.sv;
            const float v_s_u = v_u * l.u_base;
            const float v_s_v = v_v * l.v_base;
            if (AFFINE) {
                geo[0] = v_u_base * p.g0 + v_v_base * p.g1;
                geo[1] = v_u_base * p.g2 + v_v_base * p.g3;
                float v_a00 = delta.x * v_u_base;
                float v_a01 = delta.x * v_v_base;
                float v_a10 = delta.y * v_u_base;
                float v_a11 = delta.y * v_v_base;
                if (a.aa > 0.f) {
                    const float su3 = p.su * p.su * p.su;
                    const float sv3 = p.sv * p.sv * p.sv;
                    v_a00 += v_s_u * (-a.aa * p.g0 * su3);
                    v_a10 += v_s_u * (-a.aa * p.g2 * su3);
                    v_a01 += v_s_v * (-a.aa * p.g1 * sv3);
                    v_a11 += v_s_v * (-a.aa * p.g3 * sv3);
                }
                geo[2] = v_a00;
                geo[3] = v_a01;
                geo[4] = v_a10;
                geo[5] = v_a11;
            } else {
                const float inv_sx = 1.f / p.g2;
                const float inv_sy = 1.f / p.g3;
                const float v_u_rot = v_u_base * inv_sx;
                const float v_v_rot = v_v_base * inv_sy;
                float v_sx = v_u_base * (-l.u_rot) * inv_sx * inv_sx;
                float v_sy = v_v_base * (-l.v_rot) * inv_sy * inv_sy;
                if (a.aa > 0.f) {
                    const float ds_u = a.aa * (p.su * p.su * p.su) * (inv_sx * inv_sx * inv_sx);
                    const float ds_v = a.aa * (p.sv * p.sv * p.sv) * (inv_sy * inv_sy * inv_sy);
                    v_sx += v_s_u * ds_u;
                    v_sy += v_s_v * ds_v;
                }
                const float cos_t = p.g0, sin_t = p.g1;
                geo[0] = v_u_rot * cos_t + v_v_rot * (-sin_t);
                geo[1] = v_u_rot * sin_t + v_v_rot * cos_t;
                geo[2] = v_sx;
                geo[3] = v_sy;
                geo[4] = v_u_rot * l.v_rot + v_v_rot * (-l.u_rot);
            }
        }
        // colours, colour gradients and their share of the centre gradient
        for (int c = 0; c < C; ++c) {
            const float vo = v_out[c];
            const float w = valid ? norm_d * vo : 0.f;
            group_add(t, lead, a.v_colors + C * gs + c, w);
            if (CGRAD) {
                group_add(t, lead, a.v_color_grads + (gs * 2 + 0) * C + c,
                          w * a.color_grad_scale * dx);
                group_add(t, lead, a.v_color_grads + (gs * 2 + 1) * C + c,
                          w * a.color_grad_scale * dy);
                if (valid) {
                    geo[0] += w * a.color_grad_scale * a.color_grads[(g * 2 + 0) * C + c];
                    geo[1] += w * a.color_grad_scale * a.color_grads[(g * 2 + 1) * C + c];
                }
            }
        }
        if (a.v_emission) {
            for (int c = 0; c < C; ++c)
                group_add(t, lead, a.v_emission + C * gs + c,
                          (valid && peak > 0.f) ? peak * v_out[c] : 0.f);
        }
        group_add(t, lead, a.v_xy + 2 * gs + 0, geo[0]);
        group_add(t, lead, a.v_xy + 2 * gs + 1, geo[1]);
        if (AFFINE) {
#pragma unroll
            for (int q = 0; q < 4; ++q) group_add(t, lead, a.v_affines + 4 * gs + q, geo[2 + q]);
        } else {
            group_add(t, lead, a.v_scale + 2 * gs + 0, geo[2]);
            group_add(t, lead, a.v_scale + 2 * gs + 1, geo[3]);
            group_add(t, lead, a.v_rot + gs, geo[4]);
        }
        if (with_sharp) group_add(t, lead, a.v_sharpness + gs, v_sharp);
        if (a.v_softnesses) {
            if (a.softness_stride == 3) {
#pragma unroll
                for (int q = 0; q < 3; ++q)
                    group_add(t, lead, a.v_softnesses + 3 * gs + q, edge == q ? v_soft : 0.f);
            } else {
                group_add(t, lead, a.v_softnesses + gs, v_soft);
            }
        }
    }
}

}  // namespace hx

using namespace hx;

namespace {

template <bool AFFINE, bool CGRAD>
int launch_fwd(const HexFwdArgs& a, int tiles_y, cudaStream_t stream) {
    dim3 grid(a.tiles_x, tiles_y), block(kBlockX, kBlockY);
    hexel_fwd_kernel<AFFINE, CGRAD><<<grid, block, 0, stream>>>(a);
    HX_LAUNCH_CHECK("hexel_fwd_kernel");
    return HX_OK;
}

template <bool AFFINE, bool CGRAD>
int launch_bwd(const HexBwdArgs& a, cudaStream_t stream) {
    dim3 grid(ceil_div((int)a.img_w, kBlockX), ceil_div((int)a.img_h, kBlockY));
    dim3 block(kBlockX, kBlockY);
    hexel_bwd_kernel<AFFINE, CGRAD><<<grid, block, 0, stream>>>(a);
    HX_LAUNCH_CHECK("hexel_bwd_kernel");
    return HX_OK;
}

}  // namespace

extern "C" int hx_hexels2d_forward(
    int tiles_x, int tiles_y, unsigned img_width, unsigned img_height, int channels,
    int num_points, int num_intersects, const int32_t* gaussian_ids_sorted,
    const int32_t* tile_bins, const float* xys, const float* scales, const float* rotation, const float* affines,
    const float* colors, const float* color_grads, float color_grad_scale, float aa_kernel_size,
    const float* softnesses, int softness_stride, float softness_default, const float* sharpness,
    const float* emission, float* out_img, int32_t* pixel_topk, float* weights_sum,
    float* entropy, cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "hexels2d_forward: channels must be >= 1");
    HX_REQUIRE(softness_stride == 0 || softness_stride == 1 || softness_stride == 3,
               "hexels2d_forward: softness_stride must be 0, 1 or 3");
    if (tiles_x == 0 || tiles_y == 0 || img_width == 0 || img_height == 0) return HX_OK;
    const bool affine = affines != nullptr;
    HX_REQUIRE(tile_bins && out_img && pixel_topk, "hexels2d_forward: null pointer");
    HX_REQUIRE(num_intersects == 0 || (gaussian_ids_sorted && num_points > 0 && xys && colors &&
                                       (affine || (scales && rotation))),
               "hexels2d_forward: null pointer");
    HX_REQUIRE((unsigned)ceil_div((int)img_width, kBlockX) <= (unsigned)tiles_x &&
                   (unsigned)ceil_div((int)img_height, kBlockY) <= (unsigned)tiles_y,
               "tile bounds do not cover the image");
    HexFwdArgs a;
    a.tiles_x = tiles_x;
    a.num_points = num_points;
    a.num_intersects = num_intersects;
    a.img_w = img_width;
    a.img_h = img_height;
    a.channels = channels;
    a.ids_sorted = gaussian_ids_sorted;
    a.tile_bins = (const int2*)tile_bins;
    a.xys = (const float2*)xys;
    a.scales = (const float2*)scales;
    a.rotation = rotation;
    a.affines = (const float4*)affines;
    a.colors = colors;
    a.color_grads = color_grads;
    a.color_grad_scale = color_grad_scale;
    a.aa = aa_kernel_size;
    a.softnesses = softnesses;
    a.softness_stride = softnesses ? softness_stride : 0;
    a.softness_default = softness_default;
    a.sharpness = sharpness;
    a.emission = emission;
    a.out_img = out_img;
    a.pixel_topk = pixel_topk;
    a.weights_sum = weights_sum;
    a.entropy = entropy;
    const bool cg = color_grads != nullptr;
    if (affine) return cg ? launch_fwd<true, true>(a, tiles_y, stream)
                          : launch_fwd<true, false>(a, tiles_y, stream);
    return cg ? launch_fwd<false, true>(a, tiles_y, stream)
              : launch_fwd<false, false>(a, tiles_y, stream);
}

extern "C" int hx_hexels2d_backward(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* scales, const float* rotation, const float* affines, const float* colors,
    const float* color_grads, float color_grad_scale, const float* emission,
    const float* v_output, const float* v_weights_sum, const float* v_entropy,
    const int32_t* pixel_topk, float aa_kernel_size, const float* softnesses, int softness_stride,
    float softness_default, const float* sharpness, float* v_xy, float* v_scale, float* v_rot,
    float* v_affines, float* v_colors, float* v_color_grads, float* v_emission,
    float* v_sharpness, float* v_softnesses, cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "hexels2d_backward: channels must be >= 1");
    HX_REQUIRE(softness_stride == 0 || softness_stride == 1 || softness_stride == 3,
               "hexels2d_backward: softness_stride must be 0, 1 or 3");
    if (img_width == 0 || img_height == 0 || num_points == 0) return HX_OK;
    const bool affine = affines != nullptr;
    const bool cg = color_grads != nullptr;
    HX_REQUIRE(xys && colors && v_output && pixel_topk && v_xy && v_colors &&
                   (affine ? v_affines != nullptr : (scales && rotation && v_scale && v_rot)) &&
                   (!cg || v_color_grads),
               "hexels2d_backward: null pointer");
    HexBwdArgs a;
    a.img_w = img_width;
    a.img_h = img_height;
    a.channels = channels;
    a.num_points = num_points;
    a.xys = (const float2*)xys;
    a.scales = (const float2*)scales;
    a.rotation = rotation;
    a.affines = (const float4*)affines;
    a.colors = colors;
    a.color_grads = color_grads;
    a.color_grad_scale = color_grad_scale;
    a.emission = emission;
    a.v_output = v_output;
    a.v_weights_sum = v_weights_sum;
    a.v_entropy = v_entropy;
    a.pixel_topk = pixel_topk;
    a.aa = aa_kernel_size;
    a.softnesses = softnesses;
    a.softness_stride = softnesses ? softness_stride : 0;
    a.softness_default = softness_default;
    a.sharpness = sharpness;
    a.v_xy = v_xy;
    a.v_scale = v_scale;
    a.v_rot = v_rot;
    a.v_affines = v_affines;
    a.v_colors = v_colors;
    a.v_color_grads = v_color_grads;
    a.v_emission = (emission && v_emission) ? v_emission : nullptr;
    a.v_sharpness = v_sharpness;
    a.v_softnesses = (softnesses && a.softness_stride > 0) ? v_softnesses : nullptr;
    if (affine) return cg ? launch_bwd<true, true>(a, stream) : launch_bwd<true, false>(a, stream);
    return cg ? launch_bwd<false, true>(a, stream) : launch_bwd<false, false>(a, stream);
}
