// S3 / S4: Image-GS compositing — top-K normalised weighted sum, plain sum and
// the tile-less brute-force variant, forward and backward.
//
// Per-pixel arithmetic follows gsplat/cuda/csrc/forward.cu:76-410 and
// backward.cu:23-438 of the reference in the same operation order, compiled
// with the same fast-math flags, so images and top-K ids match bit for bit.
// What differs is the schedule:
//   * forward: candidates are staged per batch as packed float4/float2 in
//     shared memory; slot ids sit in shared memory and the top-K minimum is
//     cached and recomputed (as a tree) only after an insertion (same rule:
//     first empty slot, else first minimum, replace iff strictly greater);
//   * top-K backward: instead of ~80 global atomics per pixel, the lanes of
//     a warp that hold the same Gaussian sum their partials with a shuffle
//     tree and one lane adds each component with a global atomic;
//   * plain-sum backward: warp shuffle reduction, then shared-memory
//     accumulation across the CTA's warps, then one global atomic per
//     candidate component per tile.
#include "hx_topk.cuh"

namespace hx {

constexpr double kEpsTopK = 1e-4;     // EPS (config.h:9)
constexpr double kEpsNoTiles = 1e-7;  // EPS_no_tiles (config.h:10)

// A tile's [start, end) range clipped to the intersection list, and a
// primitive id clamped into [0, num_points): malformed bins or ids then read
// valid memory instead of faulting (their output is unspecified, as in the
// reference).
__device__ __forceinline__ int2 clamp_range(int2 r, int num_intersects) {
    r.y = min(r.y, num_intersects);
    r.x = max(0, min(r.x, r.y));
    return r;
}

__device__ __forceinline__ int clamp_id(int g, int num_points) {
    return min(max(g, 0), num_points - 1);
}

// Gaussian falloff exponent at pixel offset delta = xy - pixel.
__device__ __forceinline__ float gauss_sigma(const float3 conic, const float2 delta) {
    return 0.5f * (conic.x * delta.x * delta.x + conic.z * delta.y * delta.y) +
           conic.y * delta.x * delta.y;
}

__device__ __forceinline__ bool sigma_invalid(float sigma) {
    return sigma < 0.f || isnan(sigma) || isinf(sigma);
}

// Top-K slot selection: the first empty slot (value -1), else the first
// minimum of the stored values (forward.cu:263-275).
template <int K>
__device__ __forceinline__ void topk_find_min(const int (&ids)[K], const float (&vals)[K],
                                              int& min_id, float& min_val) {
    min_id = -1;
    min_val = 1e30f;
    bool found_empty = false;
#pragma unroll
    for (int k = 0; k < K; ++k) {
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

template <int K>
__device__ __forceinline__ void topk_insert(int (&ids)[K], float (&vals)[K], int& min_id,
                                            float& min_val, int g, float alpha) {
    if (alpha > min_val) {
#pragma unroll
        for (int k = 0; k < K; ++k) {
            if (k == min_id) {
                ids[k] = g;
                vals[k] = alpha;
            }
        }
        topk_find_min<K>(ids, vals, min_id, min_val);
    }
}

// ---------------------------------------------------------------------------
// Top-K forward (forward.cu:172-320), one 16x16 tile per CTA, 8x4 pixels per
// warp.  The reference's slot rule (first empty slot, else first minimum,
// replace iff strictly greater) fills slots 0..K-1 in order and, once they are
// full, never empties one, so the empty-slot search reduces to "next slot"
// while filling and the minimum scan to a tree over the K weights.  Slot ids
// live in shared memory ([slot][thread], conflict-free), so a replacement is
// one store; the weights stay in registers.
//
// Candidates are visited in list order, 32 at a time per warp: each lane
// bounds one candidate's weight over the warp's 8x4 pixel block from below
// in sigma (half the conic's smallest eigenvalue times the squared distance
// from the centre to the block, less rounding margins) and the warp skips
// every candidate whose bound cannot beat the smallest current top-K minimum
// of its lanes.  Minima only grow, so a skipped candidate would have been
// rejected by every lane; the result is the reference's, bit for bit.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) topk_fwd_kernel(
    int tiles_x, unsigned img_w, unsigned img_h, int channels, int num_points, int num_intersects,
    const int* __restrict__ gaussian_ids_sorted, const int2* __restrict__ tile_bins,
    const float2* __restrict__ xys, const float3* __restrict__ conics,
    const float* __restrict__ colors, float* __restrict__ out_img, int* __restrict__ pixel_topk,
    float* __restrict__ out_weights_sum, float* __restrict__ out_entropy) {
    __shared__ float4 s_a[kBlockSize];  // xy.x, xy.y, conic.x, conic.y
    __shared__ float4 s_b[kBlockSize];  // conic.z, id bits, eigenvalue lower bound, -
    __shared__ int s_ids[kTopK][kBlockSize];

    const int tile_id = blockIdx.y * tiles_x + blockIdx.x;
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
    const unsigned lane = tr & 31;
    const int2 lp = tile_pixel16(tr);
    const unsigned i = blockIdx.y * kBlockY + lp.y;
    const unsigned j = blockIdx.x * kBlockX + lp.x;
    const float px = (float)j;
    const float py = (float)i;
    const int pix_id = i * img_w + j;
    const bool inside = (i < img_h && j < img_w);
    // the warp's pixel block [rx0, rx0 + 7] x [ry0, ry0 + 3]
    const float rx0 = (float)(blockIdx.x * kBlockX + ((tr >> 5) & 1) * 8);
    const float ry0 = (float)(blockIdx.y * kBlockY + (tr >> 6) * 4);

    const int2 range = clamp_range(tile_bins[tile_id], num_intersects);
    float vals[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        vals[k] = 0.f;
        s_ids[k][tr] = -1;
    }
    int min_id = 0;
    float min_val = -1.f;

    for (int batch_start = range.x; batch_start < range.y; batch_start += kBlockSize) {
        __syncthreads();
        const int idx = batch_start + tr;
        if (idx < range.y) {
            const int g = clamp_id(gaussian_ids_sorted[idx], num_points);
            const float2 xy = xys[g];
            const float3 c = conics[g];
            // smallest eigenvalue of [[c.x, c.y], [c.y, c.z]], lowered by a
            // margin that covers its own rounding and that of sigma
            const float hd = 0.5f * (c.x - c.z);
            const float lam = 0.5f * (c.x + c.z) - sqrtf(hd * hd + c.y * c.y);
            const float lam_lo = lam - 1e-5f * (fabsf(c.x) + fabsf(c.z) + 2.f * fabsf(c.y));
            s_a[tr] = make_float4(xy.x, xy.y, c.x, c.y);
            s_b[tr] = make_float4(c.z, __int_as_float(g), lam_lo, 0.f);
        }
        __syncthreads();
        const int batch_size = min(kBlockSize, range.y - batch_start);
        for (int c0 = 0; c0 < batch_size; c0 += 32) {
            // smallest top-K minimum over the warp's pixels (-1 while any is
            // still filling; the int order of the bits is the float order
            // for the non-negative values, and any negative stays negative)
            const int wmin_bits = __reduce_min_sync(
                kFullMask, inside ? __float_as_int(min_val) : 0x7f800000);
            const float wmin = __int_as_float(wmin_bits);
            const float s_max = wmin > 0.f ? -__logf(wmin) * 1.0001f + 1e-3f : -1.f;
            const int tc = c0 + (int)lane;
            bool pass = tc < batch_size;
            if (pass && s_max >= 0.f) {
                const float4 a = s_a[tc];
                const float lam_lo = s_b[tc].z;
                const float ddx = fmaxf(fmaxf(rx0 - a.x, a.x - (rx0 + 7.f)), 0.f);
                const float ddy = fmaxf(fmaxf(ry0 - a.y, a.y - (ry0 + 3.f)), 0.f);
                const float sigma_lb = 0.5f * lam_lo * (ddx * ddx + ddy * ddy);
                pass = !(sigma_lb > s_max);
            }
            unsigned todo = __ballot_sync(kFullMask, pass);
            while (todo) {
                const int t = c0 + __ffs(todo) - 1;
                todo &= todo - 1;
                if (!inside) continue;
                const float4 a = s_a[t];
                const float4 b = s_b[t];
                const float2 delta = {a.x - px, a.y - py};
                const float sigma = gauss_sigma(make_float3(a.z, a.w, b.x), delta);
                if (sigma_invalid(sigma)) continue;
                const float alpha = __expf(-sigma);
                if (alpha > min_val) {
                    s_ids[min_id][tr] = __float_as_int(b.y);
#pragma unroll
                    for (int k = 0; k < kTopK; ++k)
                        if (k == min_id) vals[k] = alpha;
                    if (min_val < 0.f && min_id + 1 < kTopK)
                        ++min_id;
                    else
                        ArgMin<0, kTopK>::run(vals, min_id, min_val);
                }
            }
        }
    }
    if (!inside) return;

    int ids[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) ids[k] = s_ids[k][tr];

    if (!inside) return;

    float sum_val = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k)
        if (ids[k] >= 0) sum_val += vals[k];
    const float denom = (float)((double)sum_val + kEpsTopK);

    for (int c = 0; c < channels; ++c) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int g = ids[k];
            if (g < 0) continue;
            const float vis = vals[k] / denom;
            acc += colors[g * channels + c] * vis;
        }
        out_img[pix_id * channels + c] = acc;
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) pixel_topk[pix_id * kTopK + k] = ids[k];
    if (out_weights_sum) out_weights_sum[pix_id] = denom;
    if (out_entropy) {
        float entropy = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            if (ids[k] < 0) continue;
            const float p = vals[k] / denom;
            entropy += -p * logf(p + 1e-7f);
        }
        out_entropy[pix_id] = entropy;
    }
}

// ---------------------------------------------------------------------------
// Plain-sum forward (forward.cu:76-170).
// ---------------------------------------------------------------------------
template <int MAXC>
__global__ void __launch_bounds__(256) sum_fwd_kernel(
    int tiles_x, unsigned img_w, unsigned img_h, int channels, int num_points, int num_intersects,
    const int* __restrict__ gaussian_ids_sorted, const int2* __restrict__ tile_bins,
    const float2* __restrict__ xys, const float3* __restrict__ conics,
    const float* __restrict__ colors, float* __restrict__ out_img) {
    __shared__ float4 s_a[kBlockSize];
    __shared__ float2 s_b[kBlockSize];
    const int tile_id = blockIdx.y * tiles_x + blockIdx.x;
    const unsigned i = blockIdx.y * kBlockY + threadIdx.y;
    const unsigned j = blockIdx.x * kBlockX + threadIdx.x;
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
    const float px = (float)j;
    const float py = (float)i;
    const int pix_id = i * img_w + j;
    const bool inside = (i < img_h && j < img_w);
    const int2 range = clamp_range(tile_bins[tile_id], num_intersects);
    float pix_out[MAXC];
#pragma unroll
    for (int c = 0; c < MAXC; ++c) pix_out[c] = 0.f;

    for (int batch_start = range.x; batch_start < range.y; batch_start += kBlockSize) {
        __syncthreads();
        const int idx = batch_start + tr;
        if (idx < range.y) {
            const int g = clamp_id(gaussian_ids_sorted[idx], num_points);
            const float2 xy = xys[g];
            const float3 c = conics[g];
            s_a[tr] = make_float4(xy.x, xy.y, c.x, c.y);
            s_b[tr] = make_float2(c.z, __int_as_float(g));
        }
        __syncthreads();
        const int batch_size = min(kBlockSize, range.y - batch_start);
        if (inside) {
            for (int t = 0; t < batch_size; ++t) {
                const float4 a = s_a[t];
                const float2 b = s_b[t];
                const float2 delta = {a.x - px, a.y - py};
                const float sigma = gauss_sigma(make_float3(a.z, a.w, b.x), delta);
                if (sigma_invalid(sigma)) continue;
                const float vis = __expf(-sigma);
                const int g = __float_as_int(b.y);
#pragma unroll
                for (int c = 0; c < MAXC; ++c)
                    if (c < channels) pix_out[c] += colors[g * channels + c] * vis;
            }
        }
    }
    if (inside) {
#pragma unroll
        for (int c = 0; c < MAXC; ++c)
            if (c < channels) out_img[pix_id * channels + c] = pix_out[c];
    }
}

// ---------------------------------------------------------------------------
// Plain-sum backward (backward.cu:23-157).  `valid` is sticky per pixel as in
// the reference: once a candidate has an invalid exponent, that pixel stops
// contributing for the rest of the tile.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int MAXC>
__global__ void __launch_bounds__(256) sum_bwd_kernel(
    int tiles_x, unsigned img_w, unsigned img_h, int channels, int num_points, int num_intersects,
    const int* __restrict__ gaussian_ids_sorted, const int2* __restrict__ tile_bins,
    const float2* __restrict__ xys, const float3* __restrict__ conics,
    const float* __restrict__ colors, const float* __restrict__ v_output,
    float* __restrict__ v_xy, float* __restrict__ v_conic, float* __restrict__ v_colors) {
    constexpr int NCOMP = 5 + MAXC;
    __shared__ float4 s_a[kBlockSize];
    __shared__ float2 s_b[kBlockSize];
    __shared__ float s_rgb[kBlockSize][MAXC];
    __shared__ float s_acc[kBlockSize][NCOMP];

    const int tile_id = blockIdx.y * tiles_x + blockIdx.x;
    const unsigned i = blockIdx.y * kBlockY + threadIdx.y;
    const unsigned j = blockIdx.x * kBlockX + threadIdx.x;
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
    const int lane = tr & 31;
    const float px = (float)j;
    const float py = (float)i;
    const int pix_id = min(i * img_w + j, img_w * img_h - 1);
    const bool inside = (i < img_h && j < img_w);
    const int2 range = clamp_range(tile_bins[tile_id], num_intersects);

    float v_out[MAXC];
#pragma unroll
    for (int c = 0; c < MAXC; ++c) v_out[c] = (c < channels) ? v_output[channels * pix_id + c] : 0.f;

    bool valid = inside;
    for (int batch_start = range.x; batch_start < range.y; batch_start += kBlockSize) {
        __syncthreads();
        const int idx = batch_start + tr;
        if (idx < range.y) {
            const int g = clamp_id(gaussian_ids_sorted[idx], num_points);
            const float2 xy = xys[g];
            const float3 c = conics[g];
            s_a[tr] = make_float4(xy.x, xy.y, c.x, c.y);
            s_b[tr] = make_float2(c.z, __int_as_float(g));
#pragma unroll
            for (int c2 = 0; c2 < MAXC; ++c2)
                s_rgb[tr][c2] = (c2 < channels) ? colors[channels * g + c2] : 0.f;
        }
#pragma unroll
        for (int q = 0; q < NCOMP; ++q) s_acc[tr][q] = 0.f;
        __syncthreads();
        const int batch_size = min(kBlockSize, range.y - batch_start);
        for (int t = 0; t < batch_size; ++t) {
            const float4 a = s_a[t];
            const float2 b = s_b[t];
            const float3 conic = make_float3(a.z, a.w, b.x);
            const float2 delta = {a.x - px, a.y - py};
            const float sigma = gauss_sigma(conic, delta);
            const float d = __expf(-sigma);
            if (sigma_invalid(sigma)) valid = false;
            float v_rgb_local[MAXC];
            float vc0 = 0.f, vc1 = 0.f, vc2 = 0.f, vx = 0.f, vy = 0.f;
#pragma unroll
            for (int c = 0; c < MAXC; ++c) v_rgb_local[c] = 0.f;
            if (valid) {
#pragma unroll
                for (int c = 0; c < MAXC; ++c)
                    if (c < channels) v_rgb_local[c] = d * v_out[c];
                float v_sigma = 0.f;
#pragma unroll
                for (int c = 0; c < MAXC; ++c)
                    if (c < channels) v_sigma += s_rgb[t][c] * v_out[c];
                v_sigma *= -d;
                vc0 = 0.5f * v_sigma * delta.x * delta.x;
                vc1 = v_sigma * delta.x * delta.y;
                vc2 = 0.5f * v_sigma * delta.y * delta.y;
                vx = v_sigma * (conic.x * delta.x + conic.y * delta.y);
                vy = v_sigma * (conic.y * delta.x + conic.z * delta.y);
            }
#pragma unroll
            for (int c = 0; c < MAXC; ++c)
                if (c < channels) v_rgb_local[c] = warp_sum(v_rgb_local[c]);
            vc0 = warp_sum(vc0);
            vc1 = warp_sum(vc1);
            vc2 = warp_sum(vc2);
            vx = warp_sum(vx);
            vy = warp_sum(vy);
            if (lane == 0) {
                atomicAdd(&s_acc[t][0], vx);
                atomicAdd(&s_acc[t][1], vy);
                atomicAdd(&s_acc[t][2], vc0);
                atomicAdd(&s_acc[t][3], vc1);
                atomicAdd(&s_acc[t][4], vc2);
#pragma unroll
                for (int c = 0; c < MAXC; ++c)
                    if (c < channels) atomicAdd(&s_acc[t][5 + c], v_rgb_local[c]);
            }
        }
        __syncthreads();
        if (tr < batch_size) {
            const int g = __float_as_int(s_b[tr].y);
            atomicAdd(v_xy + 2 * g + 0, s_acc[tr][0]);
            atomicAdd(v_xy + 2 * g + 1, s_acc[tr][1]);
            atomicAdd(v_conic + 3 * g + 0, s_acc[tr][2]);
            atomicAdd(v_conic + 3 * g + 1, s_acc[tr][3]);
            atomicAdd(v_conic + 3 * g + 2, s_acc[tr][4]);
#pragma unroll
            for (int c = 0; c < MAXC; ++c)
                if (c < channels) atomicAdd(v_colors + channels * g + c, s_acc[tr][5 + c]);
        }
    }
}

// ---------------------------------------------------------------------------
// Top-K backward (backward.cu:159-316 tiled, 318-438 tile-less).  One thread
// per pixel, 256-thread CTAs over 16x16 pixel blocks with 8x4 pixels per
// warp; `eps` is the normaliser offset of the forward.  Pass 1 recomputes
// the stored ids' weights into shared columns; pass 2 computes every slot's
// partials, sums them over the lanes of the warp that hold the same Gaussian
// (KeyTree) and adds each group's sum with one global atomic.  Every lane
// runs both passes (pixels outside the image contribute zeros) so that the
// warp-wide sums stay converged.  The grid covers pixel rows [row0, row1)
// (the whole image, or one stripe of tile rows).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) topk_bwd_kernel(
    unsigned img_w, unsigned img_h, unsigned row0, unsigned row1, int channels, int num_points,
    float eps,
    const float2* __restrict__ xys, const float3* __restrict__ conics,
    const float* __restrict__ rgbs, const float* __restrict__ v_output,
    const float* __restrict__ v_weights_sum, const float* __restrict__ v_entropy,
    const int* __restrict__ pixel_topk, float* __restrict__ v_xy, float* __restrict__ v_conic,
    float* __restrict__ v_rgb) {
    __shared__ int s_id[kTopK][kBlockSize];
    __shared__ float s_d[kTopK][kBlockSize];
    __shared__ float s_vn[kTopK][kBlockSize];
    const int tr = threadIdx.y * kBlockX + threadIdx.x;
    const unsigned lane = tr & 31;
    const int2 lp = tile_pixel16(tr);
    const unsigned i = row0 + blockIdx.y * kBlockY + lp.y;
    const unsigned j = blockIdx.x * kBlockX + lp.x;
    const float px = (float)j;
    const float py = (float)i;
    const bool inside = (i < row1 && i < img_h && j < img_w);
    const int pix_id = min((int)(i * img_w + j), (int)(img_w * img_h - 1));
    const float* v_out = v_output + channels * pix_id;

    // pass 1: weights of the stored ids, their sum, and sum_c colour * v_out
    float denom = eps;
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k) {
        int g = inside ? pixel_topk[pix_id * kTopK + k] : -1;
        if (g >= num_points) g = -1;
        float d = 0.f, v_norm_d = 0.f;
        if (g >= 0) {
            const float2 xy = xys[g];
            const float2 delta = {xy.x - px, xy.y - py};
            d = __expf(-gauss_sigma(conics[g], delta));
            denom += d;
            for (int c = 0; c < channels; ++c) v_norm_d += rgbs[channels * g + c] * v_out[c];
        }
        s_id[k][tr] = g;
        s_d[k][tr] = d;
        s_vn[k][tr] = v_norm_d;
    }
    float v_d_sum = 0.f;
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k)
        if (s_id[k][tr] >= 0) v_d_sum += -s_d[k][tr] / (denom * denom) * s_vn[k][tr];
    const float v_ws = (inside && v_weights_sum) ? v_weights_sum[pix_id] : 0.f;
    const float v_ent = (inside && v_entropy) ? v_entropy[pix_id] : 0.f;
    float ent_avg = 0.f;
    if (v_ent != 0.f) {
#pragma unroll 1
        for (int k = 0; k < kTopK; ++k) {
            if (s_id[k][tr] < 0) continue;
            const float p = s_d[k][tr] / denom;
            ent_avg += p * -(logf(p + 1e-7f) + 1.f);
        }
    }

    // pass 2: per-slot partials, summed per Gaussian over the warp
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k) {
        const int g = s_id[k][tr];
        const bool valid = g >= 0;
        const KeyTree t = key_tree(lane, g);
        const bool lead = t.first && valid;
        const int gs = valid ? g : 0;  // a safe index for lanes without an id
        float vx = 0.f, vy = 0.f, vc0 = 0.f, vc1 = 0.f, vc2 = 0.f, norm_d = 0.f;
        if (valid) {
            const float d = s_d[k][tr];
            norm_d = d / denom;
            float v_d = s_vn[k][tr] / denom;
            v_d += v_d_sum;
            if (v_ws != 0.f) v_d += v_ws;
            if (v_ent != 0.f) {
                const float dhdp = -(logf(norm_d + 1e-7f) + 1.f);
                v_d += v_ent * ((dhdp - ent_avg) / denom);
            }
            const float v_sigma = v_d * -d;
            const float3 conic = conics[g];
            const float2 xy = xys[g];
            const float2 delta = {xy.x - px, xy.y - py};
            vc0 = 0.5f * v_sigma * delta.x * delta.x;
            vc1 = v_sigma * delta.x * delta.y;
            vc2 = 0.5f * v_sigma * delta.y * delta.y;
            vx = v_sigma * (conic.x * delta.x + conic.y * delta.y);
            vy = v_sigma * (conic.y * delta.x + conic.z * delta.y);
        }
        for (int c = 0; c < channels; ++c)
            group_add(t, lead, v_rgb + channels * gs + c, valid ? norm_d * v_out[c] : 0.f);
        group_add(t, lead, v_xy + 2 * gs + 0, vx);
        group_add(t, lead, v_xy + 2 * gs + 1, vy);
        group_add(t, lead, v_conic + 3 * gs + 0, vc0);
        group_add(t, lead, v_conic + 3 * gs + 1, vc1);
        group_add(t, lead, v_conic + 3 * gs + 2, vc2);
    }
}

// ---------------------------------------------------------------------------
// Tile-less top-K forward (forward.cu:322-410): every pixel scans all N
// Gaussians; Gaussians are staged through shared memory 1024 at a time.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) no_tiles_fwd_kernel(
    unsigned img_w, unsigned img_h, int channels, int num_points, const float2* __restrict__ xys,
    const float3* __restrict__ conics, const float* __restrict__ colors,
    float* __restrict__ out_img, int* __restrict__ pixel_topk) {
    __shared__ float4 s_a[1024];
    __shared__ float s_b[1024];
    const unsigned i = blockIdx.y * 32 + threadIdx.y;
    const unsigned j = blockIdx.x * 32 + threadIdx.x;
    const int tr = threadIdx.y * 32 + threadIdx.x;
    const float px = (float)j;
    const float py = (float)i;
    const int pix_id = i * img_w + j;
    const bool inside = (i < img_h && j < img_w);
    int ids[kTopK];
    float vals[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        ids[k] = -1;
        vals[k] = 0.f;
    }
    int min_id = 0;
    float min_val = -1.f;
    for (int base = 0; base < num_points; base += 1024) {
        __syncthreads();
        if (base + tr < num_points) {
            const float2 xy = xys[base + tr];
            const float3 c = conics[base + tr];
            s_a[tr] = make_float4(xy.x, xy.y, c.x, c.y);
            s_b[tr] = c.z;
        }
        __syncthreads();
        const int cnt = min(1024, num_points - base);
        if (inside) {
            for (int t = 0; t < cnt; ++t) {
                const float4 a = s_a[t];
                const float2 delta = {a.x - px, a.y - py};
                const float sigma = gauss_sigma(make_float3(a.z, a.w, s_b[t]), delta);
                if (sigma_invalid(sigma)) continue;
                const float alpha = __expf(-sigma);
                topk_insert<kTopK>(ids, vals, min_id, min_val, base + t, alpha);
            }
        }
    }
    if (!inside) return;
    for (int c = 0; c < channels; ++c) {
        float sum_val = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k)
            if (ids[k] >= 0) sum_val += vals[k];
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int g = ids[k];
            if (g < 0) continue;
            // float / double promotes: the reference divides in double here.
            const float vis = (float)((double)vals[k] / ((double)sum_val + kEpsNoTiles));
            acc += colors[g * channels + c] * vis;
        }
        out_img[pix_id * channels + c] = acc;
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) pixel_topk[pix_id * kTopK + k] = ids[k];
}

int launch_topk_bwd(unsigned img_w, unsigned img_h, unsigned row0, unsigned row1, int channels,
                    int num_points, float eps, const float* xys, const float* conics,
                    const float* colors, const float* v_output, const float* v_ws,
                    const float* v_ent, const int* pixel_topk, float* v_xy, float* v_conic,
                    float* v_colors, cudaStream_t stream) {
    if (row1 <= row0) return HX_OK;
    dim3 grid(ceil_div((int)img_w, kBlockX), ceil_div((int)(row1 - row0), kBlockY));
    dim3 block(kBlockX, kBlockY);
    topk_bwd_kernel<<<grid, block, 0, stream>>>(
        img_w, img_h, row0, row1, channels, num_points, eps, (const float2*)xys,
        (const float3*)conics, colors, v_output, v_ws, v_ent, pixel_topk, v_xy, v_conic,
        v_colors);
    HX_LAUNCH_CHECK("topk_bwd_kernel");
    return HX_OK;
}

}  // namespace hx

using namespace hx;

extern "C" int hx_nd_rasterize_forward(int tiles_x, int tiles_y, unsigned img_width,
                                       unsigned img_height, int channels, int num_points,
                                       int num_intersects,
                                       const int32_t* gaussian_ids_sorted,
                                       const int32_t* tile_bins, const float* xys,
                                       const float* conics, const float* colors, float* out_img,
                                       cudaStream_t stream) {
    HX_REQUIRE(channels >= 1 && channels <= kMaxChannels,
               "nd_rasterize_forward supports 1..%d channels (got %d)", kMaxChannels, channels);
    HX_REQUIRE(tiles_x >= 0 && tiles_y >= 0, "bad tile bounds");
    if (tiles_x == 0 || tiles_y == 0 || img_width == 0 || img_height == 0) return HX_OK;
    HX_REQUIRE(tile_bins && out_img, "nd_rasterize_forward: null pointer");
    HX_REQUIRE(num_intersects == 0 || (gaussian_ids_sorted && num_points > 0 && xys && conics &&
                                       colors),
               "nd_rasterize_forward: null pointer");
    dim3 grid(tiles_x, tiles_y), block(kBlockX, kBlockY);
    if (channels <= 3)
        sum_fwd_kernel<3><<<grid, block, 0, stream>>>(
            tiles_x, img_width, img_height, channels, num_points, num_intersects,
            gaussian_ids_sorted, (const int2*)tile_bins,
            (const float2*)xys, (const float3*)conics, colors, out_img);
    else
        sum_fwd_kernel<kMaxChannels><<<grid, block, 0, stream>>>(
            tiles_x, img_width, img_height, channels, num_points, num_intersects,
            gaussian_ids_sorted, (const int2*)tile_bins,
            (const float2*)xys, (const float3*)conics, colors, out_img);
    HX_LAUNCH_CHECK("sum_fwd_kernel");
    return HX_OK;
}

extern "C" int hx_nd_rasterize_backward(int tiles_x, int tiles_y, unsigned img_width,
                                        unsigned img_height, int channels, int num_points,
                                        int num_intersects,
                                        const int32_t* gaussian_ids_sorted,
                                        const int32_t* tile_bins, const float* xys,
                                        const float* conics, const float* colors,
                                        const float* v_output, float* v_xy, float* v_conic,
                                        float* v_colors, cudaStream_t stream) {
    HX_REQUIRE(channels >= 1 && channels <= kMaxChannels,
               "nd_rasterize_backward supports 1..%d channels (got %d)", kMaxChannels, channels);
    if (tiles_x == 0 || tiles_y == 0 || img_width == 0 || img_height == 0) return HX_OK;
    if (num_intersects == 0 || num_points == 0) return HX_OK;
    HX_REQUIRE(gaussian_ids_sorted && tile_bins && xys && conics && colors && v_output && v_xy &&
                   v_conic && v_colors,
               "nd_rasterize_backward: null pointer");
    dim3 grid(tiles_x, tiles_y), block(kBlockX, kBlockY);
    if (channels <= 3)
        sum_bwd_kernel<3><<<grid, block, 0, stream>>>(
            tiles_x, img_width, img_height, channels, num_points, num_intersects,
            gaussian_ids_sorted, (const int2*)tile_bins,
            (const float2*)xys, (const float3*)conics, colors, v_output, v_xy, v_conic, v_colors);
    else
        sum_bwd_kernel<kMaxChannels><<<grid, block, 0, stream>>>(
            tiles_x, img_width, img_height, channels, num_points, num_intersects,
            gaussian_ids_sorted, (const int2*)tile_bins,
            (const float2*)xys, (const float3*)conics, colors, v_output, v_xy, v_conic, v_colors);
    HX_LAUNCH_CHECK("sum_bwd_kernel");
    return HX_OK;
}

extern "C" int hx_nd_rasterize_forward_topk_norm(
    int tiles_x, int tiles_y, unsigned img_width, unsigned img_height, int channels,
    int num_points, int num_intersects,
    const int32_t* gaussian_ids_sorted, const int32_t* tile_bins, const float* xys,
    const float* conics, const float* colors, float* out_img, int32_t* pixel_topk,
    float* weights_sum, float* entropy, cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "nd_rasterize_forward_topk_norm: channels must be >= 1");
    if (tiles_x == 0 || tiles_y == 0 || img_width == 0 || img_height == 0) return HX_OK;
    HX_REQUIRE(tile_bins && out_img && pixel_topk, "nd_rasterize_forward_topk_norm: null pointer");
    HX_REQUIRE(num_intersects == 0 || (gaussian_ids_sorted && num_points > 0 && xys && conics &&
                                       colors),
               "nd_rasterize_forward_topk_norm: null pointer");
    HX_REQUIRE((unsigned)ceil_div((int)img_width, kBlockX) <= (unsigned)tiles_x &&
                   (unsigned)ceil_div((int)img_height, kBlockY) <= (unsigned)tiles_y,
               "tile bounds do not cover the image");
    dim3 grid(tiles_x, tiles_y), block(kBlockX, kBlockY);
    topk_fwd_kernel<<<grid, block, 0, stream>>>(
        tiles_x, img_width, img_height, channels, num_points, num_intersects,
        gaussian_ids_sorted, (const int2*)tile_bins,
        (const float2*)xys, (const float3*)conics, colors, out_img, pixel_topk, weights_sum,
        entropy);
    HX_LAUNCH_CHECK("topk_fwd_kernel");
    return HX_OK;
}

extern "C" int hx_nd_rasterize_backward_topk_norm(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* conics, const float* colors, const float* v_output, const float* v_weights_sum,
    const float* v_entropy, const int32_t* pixel_topk, float* v_xy, float* v_conic,
    float* v_colors, cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "nd_rasterize_backward_topk_norm: channels must be >= 1");
    if (img_width == 0 || img_height == 0 || num_points == 0) return HX_OK;
    HX_REQUIRE(xys && conics && colors && v_output && pixel_topk && v_xy && v_conic && v_colors,
               "nd_rasterize_backward_topk_norm: null pointer");
    return launch_topk_bwd(img_width, img_height, 0u, img_height, channels, num_points,
                           (float)kEpsTopK, xys, conics, colors, v_output, v_weights_sum,
                           v_entropy, pixel_topk, v_xy, v_conic, v_colors, stream);
}

extern "C" int hx_nd_rasterize_backward_topk_norm_rows(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* conics, const float* colors, const float* v_output, const float* v_weights_sum,
    const float* v_entropy, const int32_t* pixel_topk, int row_begin, int row_end, float* v_xy,
    float* v_conic, float* v_colors, cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "nd_rasterize_backward_topk_norm_rows: channels must be >= 1");
    HX_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= (int)img_height,
               "nd_rasterize_backward_topk_norm_rows: rows must satisfy 0 <= begin <= end <= H");
    if (img_width == 0 || row_begin == row_end || num_points == 0) return HX_OK;
    HX_REQUIRE(xys && conics && colors && v_output && pixel_topk && v_xy && v_conic && v_colors,
               "nd_rasterize_backward_topk_norm_rows: null pointer");
    return launch_topk_bwd(img_width, img_height, (unsigned)row_begin, (unsigned)row_end, channels,
                           num_points, (float)kEpsTopK, xys, conics, colors, v_output,
                           v_weights_sum, v_entropy, pixel_topk, v_xy, v_conic, v_colors, stream);
}

extern "C" int hx_nd_rasterize_forward_no_tiles(unsigned img_width, unsigned img_height,
                                                int channels, int num_points, const float* xys,
                                                const float* conics, const float* colors,
                                                float* out_img, int32_t* pixel_topk,
                                                cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "nd_rasterize_forward_no_tiles: channels must be >= 1");
    HX_REQUIRE(num_points >= 0, "nd_rasterize_forward_no_tiles: bad num_points");
    if (img_width == 0 || img_height == 0) return HX_OK;
    HX_REQUIRE(out_img && pixel_topk && (num_points == 0 || (xys && conics && colors)),
               "nd_rasterize_forward_no_tiles: null pointer");
    dim3 grid(ceil_div((int)img_width, 32), ceil_div((int)img_height, 32)), block(32, 32);
    no_tiles_fwd_kernel<<<grid, block, 0, stream>>>(img_width, img_height, channels, num_points,
                                                    (const float2*)xys, (const float3*)conics,
                                                    colors, out_img, pixel_topk);
    HX_LAUNCH_CHECK("no_tiles_fwd_kernel");
    return HX_OK;
}

extern "C" int hx_nd_rasterize_backward_no_tiles(unsigned img_width, unsigned img_height,
                                                 int channels, int num_points, const float* xys,
                                                 const float* conics, const float* colors,
                                                 const float* v_output, const int32_t* pixel_topk,
                                                 float* v_xy, float* v_conic, float* v_colors,
                                                 cudaStream_t stream) {
    HX_REQUIRE(channels >= 1, "nd_rasterize_backward_no_tiles: channels must be >= 1");
    if (img_width == 0 || img_height == 0 || num_points == 0) return HX_OK;
    HX_REQUIRE(xys && conics && colors && v_output && pixel_topk && v_xy && v_conic && v_colors,
               "nd_rasterize_backward_no_tiles: null pointer");
    return launch_topk_bwd(img_width, img_height, 0u, img_height, channels, num_points,
                           (float)kEpsNoTiles, xys, conics, colors, v_output, nullptr, nullptr,
                           pixel_topk, v_xy, v_conic, v_colors, stream);
}
