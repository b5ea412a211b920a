// S2: 2D tile binning — intersection emission, stable sort by tile, tile
// ranges.
//
// Reference: gsplat/utils.py:96-162 and gsplat/cuda/csrc/forward.cu:11-71.
// The reference emits (tile << 32 | 0, gaussian id) pairs one Gaussian per
// thread, sorts all 64 key bits with torch.sort and then scans the sorted
// keys for tile boundaries.  Here a warp emits 32 Gaussians' rectangles
// cooperatively (coalesced stores), the fused path keeps 32-bit tile keys and
// sorts only ceil(log2(num_tiles)) bits, and tile ranges are read off the
// sorted keys.  Because the low 32 key bits are always zero, a stable sort by
// tile yields exactly the reference's sorted lists: within a tile, Gaussians
// in ascending id order.
#include "hx_common.cuh"
#include "hx_sort.cuh"
#include "hx_tiles.cuh"

namespace hx {

__device__ __forceinline__ TileRect gaussian_rect(const float2* xys, const int* radii, int idx,
                                                  int tiles_x, int tiles_y, int row_begin,
                                                  int row_end, bool& valid) {
    TileRect r = {0, 0, 0, 0};
    valid = false;
    const int rad = radii[idx];
    if (rad <= 0) return r;
    r = tile_rect(xys[idx], (float)rad, tiles_x, tiles_y);
    if ((int)r.y0 < row_begin) r.y0 = row_begin;
    if ((int)r.y1 > row_end) r.y1 = row_end;
    valid = r.x1 > r.x0 && r.y1 > r.y0;
    return r;
}

// One warp emits the rectangles of 32 consecutive Gaussians: lane j computes
// Gaussian j's rectangle and output offset, then all 32 lanes write each
// rectangle's tiles in row-major order.
template <typename KeyT, int kShift>
__global__ void __launch_bounds__(256) emit_keys_kernel(
    int n, int num_intersects, const float2* __restrict__ xys, const int* __restrict__ radii,
    const int* __restrict__ cum_tiles_hit, int tiles_x, int tiles_y, int row_begin, int row_end,
    KeyT* __restrict__ keys, int* __restrict__ vals) {
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int idx = gwarp * 32 + lane;
    bool valid = false;
    TileRect r = {0, 0, 0, 0};
    int off = 0;
    if (idx < n) {
        r = gaussian_rect(xys, radii, idx, tiles_x, tiles_y, row_begin, row_end, valid);
        off = idx == 0 ? 0 : cum_tiles_hit[idx - 1];
    }
    unsigned todo = __ballot_sync(0xffffffffu, valid);
    while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1;
        const unsigned x0 = __shfl_sync(0xffffffffu, r.x0, j);
        const unsigned y0 = __shfl_sync(0xffffffffu, r.y0, j);
        const unsigned x1 = __shfl_sync(0xffffffffu, r.x1, j);
        const unsigned y1 = __shfl_sync(0xffffffffu, r.y1, j);
        const int base = __shfl_sync(0xffffffffu, off, j);
        const int gid = gwarp * 32 + j;
        const int w = (int)(x1 - x0);
        const int area = w * (int)(y1 - y0);
        for (int e = lane; e < area; e += 32) {
            const int pos = base + e;
            if (pos < 0 || pos >= num_intersects) continue;
            const int ty = (int)y0 + e / w;
            const int tx = (int)x0 + e % w;
            const KeyT tile = (KeyT)(ty * tiles_x + tx);
            keys[pos] = tile << kShift;
            vals[pos] = gid;
        }
    }
}

__global__ void __launch_bounds__(256) count_tiles_kernel(int n, const float2* __restrict__ xys,
                                                          const int* __restrict__ radii,
                                                          int tiles_x, int tiles_y, int row_begin,
                                                          int row_end, int* __restrict__ counts) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    bool valid;
    TileRect r = gaussian_rect(xys, radii, idx, tiles_x, tiles_y, row_begin, row_end, valid);
    counts[idx] = valid ? (int)((r.x1 - r.x0) * (r.y1 - r.y0)) : 0;
}

// Tile ranges from keys sorted by tile: tile_bins[t] = [first, last + 1).
// tile_bins must be zeroed beforehand (empty tiles stay (0, 0)).
template <typename KeyT, int kShift>
__global__ void __launch_bounds__(256) tile_ranges_kernel(int num_intersects, int num_tiles,
                                                          const KeyT* __restrict__ sorted_keys,
                                                          int2* __restrict__ tile_bins,
                                                          long long* __restrict__ keys64_out) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= num_intersects) return;
    const int cur = (int)(sorted_keys[idx] >> kShift);
    if (keys64_out) keys64_out[idx] = (long long)cur << 32;
    if (cur < 0 || cur >= num_tiles) return;
    if (idx == 0) tile_bins[cur].x = 0;
    if (idx == num_intersects - 1) tile_bins[cur].y = num_intersects;
    if (idx == 0) return;
    const int prev = (int)(sorted_keys[idx - 1] >> kShift);
    if (prev != cur) {
        if (prev >= 0 && prev < num_tiles) tile_bins[prev].y = idx;
        tile_bins[cur].x = idx;
    }
}

}  // namespace hx

using namespace hx;

extern "C" int hx_map_gaussian_to_intersects(int num_points, int num_intersects, const float* xys,
                                             const int32_t* radii, const int32_t* cum_tiles_hit,
                                             int tiles_x, int tiles_y, int64_t* isect_ids,
                                             int32_t* gaussian_ids, cudaStream_t stream) {
    HX_REQUIRE(num_points >= 0 && num_intersects >= 0, "map_gaussian_to_intersects: bad sizes");
    if (num_points == 0 || num_intersects == 0) return HX_OK;
    HX_REQUIRE(xys && radii && cum_tiles_hit && isect_ids && gaussian_ids,
               "map_gaussian_to_intersects: null pointer");
    HX_REQUIRE(tiles_x > 0 && tiles_y > 0, "tile bounds must be positive");
    emit_keys_kernel<unsigned long long, 32><<<ceil_div(num_points, 256), 256, 0, stream>>>(
        num_points, num_intersects, (const float2*)xys, radii, cum_tiles_hit, tiles_x, tiles_y, 0,
        tiles_y, (unsigned long long*)isect_ids, gaussian_ids);
    HX_LAUNCH_CHECK("emit_keys_kernel<u64>");
    return HX_OK;
}

extern "C" int hx_get_tile_bin_edges(int num_intersects, int num_tiles,
                                     const int64_t* isect_ids_sorted, int32_t* tile_bins,
                                     cudaStream_t stream) {
    HX_REQUIRE(num_intersects >= 0 && num_tiles >= 0, "get_tile_bin_edges: bad sizes");
    if (num_tiles == 0) return HX_OK;
    HX_REQUIRE(tile_bins, "get_tile_bin_edges: null tile_bins");
    HX_CUDA_TRY(cudaMemsetAsync(tile_bins, 0, sizeof(int32_t) * 2 * (size_t)num_tiles, stream));
    if (num_intersects == 0) return HX_OK;
    HX_REQUIRE(isect_ids_sorted, "get_tile_bin_edges: null keys");
    tile_ranges_kernel<unsigned long long, 32><<<ceil_div(num_intersects, 256), 256, 0, stream>>>(
        num_intersects, num_tiles, (const unsigned long long*)isect_ids_sorted, (int2*)tile_bins,
        nullptr);
    HX_LAUNCH_CHECK("tile_ranges_kernel<u64>");
    return HX_OK;
}

extern "C" int hx_count_tiles_2d(int num_points, const float* xys, const int32_t* radii,
                                 int tiles_x, int tiles_y, int tile_row_begin, int tile_row_end,
                                 int32_t* counts, cudaStream_t stream) {
    HX_REQUIRE(num_points >= 0, "count_tiles_2d: bad size");
    if (num_points == 0) return HX_OK;
    HX_REQUIRE(xys && radii && counts, "count_tiles_2d: null pointer");
    HX_REQUIRE(0 <= tile_row_begin && tile_row_begin <= tile_row_end && tile_row_end <= tiles_y,
               "count_tiles_2d: stripe rows [%d, %d) outside [0, %d)", tile_row_begin,
               tile_row_end, tiles_y);
    count_tiles_kernel<<<ceil_div(num_points, 256), 256, 0, stream>>>(
        num_points, (const float2*)xys, radii, tiles_x, tiles_y, tile_row_begin, tile_row_end,
        counts);
    HX_LAUNCH_CHECK("count_tiles_kernel");
    return HX_OK;
}

extern "C" size_t hx_bin_gaussians_2d_workspace_bytes(int num_intersects, int num_tiles) {
    (void)num_tiles;
    const size_t n = num_intersects > 0 ? (size_t)num_intersects : 1;
    return 2 * align256(sizeof(uint32_t) * n) + align256(sizeof(int32_t) * n) +
           sort_workspace_bytes<uint32_t>((int)n);
}

extern "C" int hx_bin_gaussians_2d(int num_points, int num_intersects, const float* xys,
                                   const int32_t* radii, const int32_t* cum_tiles_hit, int tiles_x,
                                   int tiles_y, int tile_row_begin, int tile_row_end,
                                   int32_t* gaussian_ids_sorted, int32_t* tile_bins,
                                   int64_t* isect_ids_sorted, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
    HX_REQUIRE(num_points >= 0 && num_intersects >= 0, "bin_gaussians_2d: bad sizes");
    HX_REQUIRE(tiles_x > 0 && tiles_y > 0, "tile bounds must be positive");
    HX_REQUIRE(0 <= tile_row_begin && tile_row_begin <= tile_row_end && tile_row_end <= tiles_y,
               "bin_gaussians_2d: stripe rows [%d, %d) outside [0, %d)", tile_row_begin,
               tile_row_end, tiles_y);
    const int num_tiles = tiles_x * tiles_y;
    HX_REQUIRE(tile_bins, "bin_gaussians_2d: null tile_bins");
    HX_CUDA_TRY(cudaMemsetAsync(tile_bins, 0, sizeof(int32_t) * 2 * (size_t)num_tiles, stream));
    if (num_intersects == 0 || num_points == 0) return HX_OK;
    HX_REQUIRE(xys && radii && cum_tiles_hit && gaussian_ids_sorted,
               "bin_gaussians_2d: null pointer");
    const size_t need = hx_bin_gaussians_2d_workspace_bytes(num_intersects, num_tiles);
    if (!workspace || workspace_bytes < need)
        return set_error(HX_ERR_WORKSPACE, "bin_gaussians_2d: workspace of %zu bytes needed", need);
    char* p = (char*)workspace;
    uint32_t* keys = (uint32_t*)p;
    p += align256(sizeof(uint32_t) * (size_t)num_intersects);
    uint32_t* keys_sorted = (uint32_t*)p;
    p += align256(sizeof(uint32_t) * (size_t)num_intersects);
    int* vals = (int*)p;
    p += align256(sizeof(int32_t) * (size_t)num_intersects);
    void* sort_ws = p;
    const size_t sort_bytes = sort_workspace_bytes<uint32_t>(num_intersects);

    emit_keys_kernel<uint32_t, 0><<<ceil_div(num_points, 256), 256, 0, stream>>>(
        num_points, num_intersects, (const float2*)xys, radii, cum_tiles_hit, tiles_x, tiles_y,
        tile_row_begin, tile_row_end, keys, vals);
    HX_LAUNCH_CHECK("emit_keys_kernel<u32>");
    int rc = sort_pairs<uint32_t>(keys, vals, keys_sorted, gaussian_ids_sorted, num_intersects, 0,
                                  tile_bits(num_tiles), sort_ws, sort_bytes, stream);
    if (rc != HX_OK) return rc;
    tile_ranges_kernel<uint32_t, 0><<<ceil_div(num_intersects, 256), 256, 0, stream>>>(
        num_intersects, num_tiles, keys_sorted, (int2*)tile_bins, (long long*)isect_ids_sorted);
    HX_LAUNCH_CHECK("tile_ranges_kernel<u32>");
    return HX_OK;
}
