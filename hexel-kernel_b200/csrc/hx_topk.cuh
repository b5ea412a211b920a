// Building blocks of the top-10 compositing kernels (Image-GS and 2D hexels):
// the pixel layout of a 16x16 tile, the minimum scan of the top-10 slots and
// the per-warp sums that stand in for per-pixel gradient atomics.
#pragma once

#include "hx_common.cuh"

namespace hx {

// Pixel (x, y) within its 16x16 tile for thread `tr` of a 256-thread CTA: each
// warp covers an 8x4 block, so that the lanes of a warp see similar candidate
// rankings in the forward and share more ids in the backward.
__device__ __forceinline__ int2 tile_pixel16(int tr) {
    const int warp = tr >> 5, lane = tr & 31;
    return make_int2(((warp & 1) << 3) | (lane & 7), ((warp >> 1) << 2) | (lane >> 3));
}

// Index of the smallest of vals[LO, LO + N), the lowest index among equal
// values, as a pairwise tree (a higher index wins only when strictly
// smaller, which keeps the first-minimum choice of a left-to-right scan).
template <int LO, int N>
struct ArgMin {
    static __device__ __forceinline__ void run(const float (&vals)[kTopK], int& idx, float& v) {
        if constexpr (N == 1) {
            idx = LO;
            v = vals[LO];
        } else {
            int i0, i1;
            float v0, v1;
            ArgMin<LO, N / 2>::run(vals, i0, v0);
            ArgMin<LO + N / 2, N - N / 2>::run(vals, i1, v1);
            const bool right = v1 < v0;
            idx = right ? i1 : i0;
            v = right ? v1 : v0;
        }
    }
};

constexpr unsigned kFullMask = 0xffffffffu;

// Binary summation tree over the lanes of a warp that hold the same key, in
// lane order: at level l every remaining lane adds the value of the next
// remaining lane above it, then the lanes of odd rank at that level drop out.
// After the last level the lowest lane of each key group holds the group's
// sum.  The tree depends on the keys only, so it is built once per stored id
// and reused for every gradient component.
struct KeyTree {
    int src[5];     // lane read at each level (own lane when nothing is added)
    unsigned add;   // bit l: this lane adds at level l
    int levels;     // warp-uniform
    bool first;     // lowest lane of its key group
};

// All 32 lanes of the warp must call this (and key_sum / group_add) together.
__device__ __forceinline__ KeyTree key_tree(unsigned lane, int key) {
    KeyTree t;
    const unsigned peers = __match_any_sync(kFullMask, key);
    const unsigned below = (1u << lane) - 1u;
    unsigned rank = __popc(peers & below);
    unsigned above = peers & ~below & ~(1u << lane);
    t.first = rank == 0u;
    t.add = 0u;
    t.levels = 0;
#pragma unroll
    for (int l = 0; l < 5; ++l) {
        t.src[l] = (int)lane;
        if (!__any_sync(kFullMask, above != 0u)) break;
        const int next = __ffs(above);
        if (next) {
            t.src[l] = next - 1;
            t.add |= 1u << l;
        }
        above &= ~__ballot_sync(kFullMask, rank & 1u);
        rank >>= 1;
        t.levels = l + 1;
    }
    return t;
}

__device__ __forceinline__ float key_sum(const KeyTree& t, float x) {
#pragma unroll
    for (int l = 0; l < 5; ++l) {
        if (l >= t.levels) break;
        const float y = __shfl_sync(kFullMask, x, t.src[l]);
        if ((t.add >> l) & 1u) x += y;
    }
    return x;
}

// Sums `v` over the key group; its lowest lane adds a non-zero sum to `*dst`
// when `lead` is set.  Every lane of the warp calls this with the same tree.
__device__ __forceinline__ void group_add(const KeyTree& t, bool lead, float* dst, float v) {
    const float s = key_sum(t, v);
    if (lead && s != 0.f) atomicAdd(dst, s);
}

}  // namespace hx
