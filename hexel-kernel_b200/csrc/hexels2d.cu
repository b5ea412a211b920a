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
//   * the backward accumulates per-primitive partials in a shared-memory hash
//     table and flushes one global atomic per (primitive, component) per tile
//     instead of up to ~20 global atomics per (pixel, primitive).
#include "hx_common.cuh"

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
    const float t1 = kHexA * u + kHexB * v;
    const float t2 = kHexA * u - kHexB * v;
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
        l.u_rot = dx * p.g0 + dy * p.g1;
        l.v_rot = -dx * p.g1 + dy * p.g0;
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

template <bool AFFINE, bool CGRAD>
__global__ void __launch_bounds__(256) hexel_fwd_kernel(const HexFwdArgs a) {
    __shared__ HexPrim s_prim[kBlockSize];
    const int tile_id = blockIdx.y * a.tiles_x + blockIdx.x;
    const unsigned i = blockIdx.y * kBlockY + threadIdx.y;
    const unsigned j = blockIdx.x * kBlockX + threadIdx.x;
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
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

    int ids[kTopK];
    float vals[kTopK];
    float peaks[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        ids[k] = -1;
        vals[k] = 0.f;
        peaks[k] = 0.f;
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
#pragma unroll
                    for (int k = 0; k < kTopK; ++k) {
                        if (k == min_id) {
                            ids[k] = p.id;
                            vals[k] = alpha;
                            peaks[k] = peak;
                        }
                    }
                    if (min_val < 0.f && min_id + 1 < kTopK) {
                        ++min_id;
                    } else {
                        min_val = 1e30f;
                        bool found_empty = false;
#pragma unroll
                        for (int k = 0; k < kTopK; ++k) {
                            if (!found_empty) {
                                if (ids[k] < 0) {
                                    min_id = k;
                                    min_val = -1.0f;
                                    found_empty = true;
                                } else if (vals[k] < min_val) {
                                    min_id = k;
                                    min_val = vals[k];
                                }
                            }
                        }
                    }
                }
            }
        }
    }
    if (!inside) return;

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
    // shared-memory table layout (component offsets within a slot; -1 = absent)
    int ncomp, off_col, off_cg, off_em, off_sh, off_soft, table_cap;
};

namespace {

struct Table {
    int* keys;
    float* acc;
    int cap;
    int ncomp;
};

__device__ __forceinline__ int table_find(const Table& t, int g) {
    if (t.cap == 0) return -1;
    const unsigned mask = (unsigned)t.cap - 1u;
    const unsigned h = ((unsigned)g * 2654435761u) & mask;
    volatile int* keys = t.keys;
#pragma unroll 1
    for (int probe = 0; probe < 32; ++probe) {
        const unsigned s = (h + probe) & mask;
        const int k = keys[s];
        if (k == g) return (int)s;
        if (k == -1) {
            const int prev = atomicCAS(t.keys + s, -1, g);
            if (prev == -1 || prev == g) return (int)s;
        }
    }
    return -1;
}

// Adds `v` to component `comp` of slot `slot`, or to global `*gptr` when the
// primitive has no slot.
__device__ __forceinline__ void acc_add(const Table& t, int slot, int comp, float* gptr, float v) {
    if (slot >= 0)
        atomicAdd(t.acc + slot * t.ncomp + comp, v);
    else
        atomicAdd(gptr, v);
}

}  // namespace

template <bool AFFINE, bool CGRAD>
__global__ void __launch_bounds__(256) hexel_bwd_kernel(const HexBwdArgs a) {
    extern __shared__ __align__(16) unsigned char s_raw[];
    Table tab;
    tab.cap = a.table_cap;
    tab.ncomp = a.ncomp;
    tab.keys = reinterpret_cast<int*>(s_raw);
    tab.acc = reinterpret_cast<float*>(s_raw + sizeof(int) * a.table_cap);
    const int tid = threadIdx.y * kBlockX + threadIdx.x;
    for (int s = tid; s < tab.cap; s += kBlockSize) tab.keys[s] = -1;
    for (int s = tid; s < tab.cap * tab.ncomp; s += kBlockSize) tab.acc[s] = 0.f;
    __syncthreads();

    const int C = a.channels;
    const unsigned i = blockIdx.y * kBlockY + threadIdx.y;
    const unsigned j = blockIdx.x * kBlockX + threadIdx.x;
    const float px = (float)j;
    const float py = (float)i;
    const bool inside = (i < a.img_h && j < a.img_w);
    const int pix_id = min((int)(i * a.img_w + j), (int)(a.img_w * a.img_h - 1));
    const int* topk = a.pixel_topk + pix_id * kTopK;
    // Mirrors the reference's early exits: outside pixels and pixels whose
    // first slot is empty contribute nothing.
    const bool active = inside && topk[0] >= 0;

    if (active) {
        const float* v_out = a.v_output + C * pix_id;
        int ids[kTopK];
        int slots[kTopK];
        float d_local[kTopK], u_coord[kTopK], v_coord[kTopK], prim_peak[kTopK];
        float v_peak_emit[kTopK], v_d_local[kTopK];
        float denom = (float)kEpsHex;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            int g = topk[k];
            if (g >= a.num_points) g = -1;
            ids[k] = g;
            slots[k] = -1;
            d_local[k] = u_coord[k] = v_coord[k] = prim_peak[k] = v_peak_emit[k] = 0.f;
            v_d_local[k] = 0.f;
            if (g < 0) continue;
            const HexPrim p = make_prim<AFFINE>(g, a.xys, a.scales, a.rotation, a.affines, a.aa,
                                                a.softnesses, a.softness_stride,
                                                a.softness_default, a.sharpness);
            const HexLocal l = hex_local<AFFINE>(p, p.x - px, p.y - py);
            int edge;
            const float dist = hex_sdf(l.u, l.v, edge);
            const float sig = sigmoid_neg_dist(dist, edge_softness(p, edge));
            float alpha = sig;
            if (p.sharp > 0.f) {
                const float r2 = l.u * l.u + l.v * l.v;
                const float pk = __expf(-p.sharp * r2);
                prim_peak[k] = pk;
                alpha *= pk;
            }
            denom += alpha;
            d_local[k] = alpha;
            u_coord[k] = l.u;
            v_coord[k] = l.v;
        }

        float v_d_sum = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int g = ids[k];
            if (g < 0) continue;
            const int slot = table_find(tab, g);
            slots[k] = slot;
            const float alpha = d_local[k];
            const float norm_d = alpha / denom;
            float v_norm_d = 0.f;
            float dx = 0.f, dy = 0.f;
            if (CGRAD) {
                const float2 xy = a.xys[g];
                dx = xy.x - px;
                dy = xy.y - py;
            }
            for (int c = 0; c < C; ++c) {
                const float vo = v_out[c];
                if (CGRAD) {
                    const float base = a.colors[C * g + c];
                    const float gx = a.color_grads[(g * 2 + 0) * C + c];
                    const float gy = a.color_grads[(g * 2 + 1) * C + c];
                    const float color = base + a.color_grad_scale * (dx * gx + dy * gy);
                    acc_add(tab, slot, a.off_col + c, a.v_colors + C * g + c, norm_d * vo);
                    acc_add(tab, slot, a.off_cg + c, a.v_color_grads + (g * 2 + 0) * C + c,
                            norm_d * vo * a.color_grad_scale * dx);
                    acc_add(tab, slot, a.off_cg + C + c, a.v_color_grads + (g * 2 + 1) * C + c,
                            norm_d * vo * a.color_grad_scale * dy);
                    v_norm_d += color * vo;
                } else {
                    acc_add(tab, slot, a.off_col + c, a.v_colors + C * g + c, norm_d * vo);
                    v_norm_d += a.colors[C * g + c] * vo;
                }
            }
            if (a.emission && a.v_emission) {
                const float peak = prim_peak[k];
                if (peak > 0.f) {
                    float vpe = 0.f;
                    for (int c = 0; c < C; ++c) {
                        acc_add(tab, slot, a.off_em + c, a.v_emission + C * g + c,
                                peak * v_out[c]);
                        vpe += a.emission[C * g + c] * v_out[c];
                    }
                    v_peak_emit[k] = vpe;
                }
            }
            if (CGRAD) {
                float vdx = 0.f, vdy = 0.f;
                for (int c = 0; c < C; ++c) {
                    const float gx = a.color_grads[(g * 2 + 0) * C + c];
                    const float gy = a.color_grads[(g * 2 + 1) * C + c];
                    vdx += norm_d * v_out[c] * a.color_grad_scale * gx;
                    vdy += norm_d * v_out[c] * a.color_grad_scale * gy;
                }
                acc_add(tab, slot, 0, a.v_xy + 2 * g + 0, vdx);
                acc_add(tab, slot, 1, a.v_xy + 2 * g + 1, vdy);
            }
            v_d_local[k] = v_norm_d / denom;
            v_d_sum += -alpha / (denom * denom) * v_norm_d;
        }
#pragma unroll
        for (int k = 0; k < kTopK; ++k) v_d_local[k] += v_d_sum;

        const float v_ws = a.v_weights_sum ? a.v_weights_sum[pix_id] : 0.f;
        const float v_ent = a.v_entropy ? a.v_entropy[pix_id] : 0.f;
        if (v_ws != 0.f) {
#pragma unroll
            for (int k = 0; k < kTopK; ++k)
                if (ids[k] >= 0) v_d_local[k] += v_ws;
        }
        if (v_ent != 0.f) {
            float dHdp[kTopK];
            float avg = 0.f;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                dHdp[k] = 0.f;
                if (ids[k] < 0) continue;
                const float p = d_local[k] / denom;
                const float dhdp = -(logf(p + kEntropyEps) + 1.f);
                dHdp[k] = dhdp;
                avg += p * dhdp;
            }
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                if (ids[k] < 0) continue;
                const float dhdw = (dHdp[k] - avg) / denom;
                v_d_local[k] += v_ent * dhdw;
            }
        }

#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int g = ids[k];
            if (g < 0) continue;
            const int slot = slots[k];
            const HexPrim p = make_prim<AFFINE>(g, a.xys, a.scales, a.rotation, a.affines, a.aa,
                                                a.softnesses, a.softness_stride,
                                                a.softness_default, a.sharpness);
            const float2 delta = {p.x - px, p.y - py};
            const HexLocal l = hex_local<AFFINE>(p, delta.x, delta.y);
            int edge;
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
            const float v_d = v_d_local[k];
            float v_sig = v_d;
            float v_u_peak = 0.f, v_v_peak = 0.f;
            if (p.sharp > 0.f) {
                const float r2 = u_coord[k] * u_coord[k] + v_coord[k] * v_coord[k];
                const float peak = prim_peak[k];
                v_sig = v_d * peak;
                const float v_peak = v_d * sig + v_peak_emit[k];
                const float v_r2 = v_peak * peak * (-p.sharp);
                v_u_peak = v_r2 * 2.f * u_coord[k];
                v_v_peak = v_r2 * 2.f * v_coord[k];
                if (a.v_sharpness) acc_add(tab, slot, a.off_sh, a.v_sharpness + g,
                                           v_peak * peak * (-r2));
            }
            if (a.v_softnesses) {
                const float v_soft = v_sig * (-dist) * sig * (1.f - sig);
                if (a.softness_stride == 3)
                    acc_add(tab, slot, a.off_soft + edge, a.v_softnesses + g * 3 + edge, v_soft);
                else if (a.softness_stride == 1)
                    acc_add(tab, slot, a.off_soft, a.v_softnesses + g, v_soft);
            }
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
                const float v_dx = v_u_base * p.g0 + v_v_base * p.g1;
                const float v_dy = v_u_base * p.g2 + v_v_base * p.g3;
                acc_add(tab, slot, 0, a.v_xy + 2 * g + 0, v_dx);
                acc_add(tab, slot, 1, a.v_xy + 2 * g + 1, v_dy);
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
                acc_add(tab, slot, 2, a.v_affines + 4 * g + 0, v_a00);
                acc_add(tab, slot, 3, a.v_affines + 4 * g + 1, v_a01);
                acc_add(tab, slot, 4, a.v_affines + 4 * g + 2, v_a10);
                acc_add(tab, slot, 5, a.v_affines + 4 * g + 3, v_a11);
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
                const float v_dx = v_u_rot * cos_t + v_v_rot * (-sin_t);
                const float v_dy = v_u_rot * sin_t + v_v_rot * cos_t;
                const float v_rot_angle = v_u_rot * l.v_rot + v_v_rot * (-l.u_rot);
                acc_add(tab, slot, 0, a.v_xy + 2 * g + 0, v_dx);
                acc_add(tab, slot, 1, a.v_xy + 2 * g + 1, v_dy);
                acc_add(tab, slot, 2, a.v_scale + 2 * g + 0, v_sx);
                acc_add(tab, slot, 3, a.v_scale + 2 * g + 1, v_sy);
                acc_add(tab, slot, 4, a.v_rot + g, v_rot_angle);
            }
        }
    }

    __syncthreads();
    // Flush: one global atomic per (primitive, non-zero component).
    for (int s = tid; s < tab.cap; s += kBlockSize) {
        const int g = tab.keys[s];
        if (g < 0) continue;
        const float* acc = tab.acc + s * tab.ncomp;
        auto put = [&](float* dst, float v) {
            if (v != 0.f) atomicAdd(dst, v);
        };
        put(a.v_xy + 2 * g + 0, acc[0]);
        put(a.v_xy + 2 * g + 1, acc[1]);
        if (AFFINE) {
            for (int q = 0; q < 4; ++q) put(a.v_affines + 4 * g + q, acc[2 + q]);
        } else {
            put(a.v_scale + 2 * g + 0, acc[2]);
            put(a.v_scale + 2 * g + 1, acc[3]);
            put(a.v_rot + g, acc[4]);
        }
        for (int c = 0; c < C; ++c) put(a.v_colors + C * g + c, acc[a.off_col + c]);
        if (a.off_cg >= 0)
            for (int q = 0; q < 2 * C; ++q) put(a.v_color_grads + 2 * C * g + q, acc[a.off_cg + q]);
        if (a.off_em >= 0)
            for (int c = 0; c < C; ++c) put(a.v_emission + C * g + c, acc[a.off_em + c]);
        if (a.off_sh >= 0) put(a.v_sharpness + g, acc[a.off_sh]);
        if (a.off_soft >= 0) {
            if (a.softness_stride == 3)
                for (int q = 0; q < 3; ++q) put(a.v_softnesses + 3 * g + q, acc[a.off_soft + q]);
            else
                put(a.v_softnesses + g, acc[a.off_soft]);
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

constexpr int kMaxTableComp = 40;

template <bool AFFINE, bool CGRAD>
int launch_bwd(HexBwdArgs a, cudaStream_t stream) {
    const size_t smem = sizeof(int) * a.table_cap + sizeof(float) * (size_t)a.table_cap * a.ncomp;
    static bool attr_set[64] = {};
    int dev = 0;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        HX_CUDA_TRY(cudaFuncSetAttribute(hexel_bwd_kernel<AFFINE, CGRAD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(sizeof(int) * 512 +
                                               sizeof(float) * 512 * kMaxTableComp)));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    dim3 grid(ceil_div((int)a.img_w, kBlockX), ceil_div((int)a.img_h, kBlockY));
    dim3 block(kBlockX, kBlockY);
    hexel_bwd_kernel<AFFINE, CGRAD><<<grid, block, smem, stream>>>(a);
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
    // slot layout: geometry (5 or 6), colours, [colour gradients], [emission],
    // [sharpness], [softness]
    int off = affine ? 6 : 5;
    a.off_col = off;
    off += channels;
    a.off_cg = cg ? off : -1;
    off += cg ? 2 * channels : 0;
    a.off_em = a.v_emission ? off : -1;
    off += a.v_emission ? channels : 0;
    a.off_sh = (sharpness && v_sharpness) ? off : -1;
    off += (sharpness && v_sharpness) ? 1 : 0;
    a.off_soft = a.v_softnesses ? off : -1;
    off += a.v_softnesses ? a.softness_stride : 0;
    a.ncomp = off;
    a.table_cap = off <= kMaxTableComp ? 512 : 0;  // 0: accumulate straight to global
    if (a.table_cap == 0) a.ncomp = 1;
    if (!(sharpness && v_sharpness)) a.v_sharpness = v_sharpness;  // unused without sharpness
    if (affine) return cg ? launch_bwd<true, true>(a, stream) : launch_bwd<true, false>(a, stream);
    return cg ? launch_bwd<false, true>(a, stream) : launch_bwd<false, false>(a, stream);
}
