// Stable LSD radix sort of (key, int32 value) pairs, 8-bit digits.
//
// Each pass is reduce-then-scan and waits on nothing across CTAs:
//   1. upsweep  — per-CTA digit histogram of a tile of 256 x ITEMS keys
//      (ITEMS = 16 for large inputs, 4 below 2M keys so that a pass over a
//      million keys still spreads over ~1000 CTAs),
//   2. scan     — per-digit exclusive scan over CTAs (digit-major layout),
//   3. downsweep — stable in-tile ranking (warp match + per-warp running
//      counters), reorder through shared memory, coalesced scatter.
// Stability: within a tile, warp w owns keys [32 ITEMS w, 32 ITEMS (w + 1))
// and processes them 32 at a time in index order, so equal digits keep their input order;
// tiles are ordered by the scan.  This replaces the stable CUB / PyTorch radix
// sorts the reference calls (gsplat/utils.py:159, hexels3d_forward.cu:3013).
#include <atomic>
#include "hx_common.cuh"
#include "hx_sort.cuh"

namespace hx {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kRadix = 256;
constexpr int kSmallSortN = 1 << 21;  // below: 4 keys per thread, else 16

inline int sort_items(int n) { return n < kSmallSortN ? 4 : 16; }

template <typename K>
__device__ __forceinline__ unsigned digit_of(K key, int shift, unsigned mask) {
    return (unsigned)(key >> shift) & mask;
}

template <typename K, int ITEMS>
__global__ void __launch_bounds__(kSortThreads) sort_upsweep_kernel(const K* __restrict__ keys,
                                                                    int n, int shift,
                                                                    unsigned mask,
                                                                    int* __restrict__ hist,
                                                                    int num_tiles) {
    __shared__ int s_hist[kSortWarps][kRadix];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads)
        (&s_hist[0][0])[i] = 0;
    __syncthreads();
    constexpr int kTile = kSortThreads * ITEMS;
    const int base = blockIdx.x * kTile + warp * (kTile / kSortWarps);
#pragma unroll 4
    for (int i = 0; i < ITEMS; ++i) {
        const int idx = base + i * 32 + lane;
        if (idx < n) atomicAdd(&s_hist[warp][digit_of(keys[idx], shift, mask)], 1);
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kRadix; d += kSortThreads) {
        int c = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) c += s_hist[w][d];
        hist[(size_t)d * num_tiles + blockIdx.x] = c;
    }
}

// One CTA per digit: exclusive scan of that digit's per-tile counts in place;
// the digit's total goes to digit_totals[d].
__global__ void __launch_bounds__(256) sort_scan_kernel(int* __restrict__ hist, int num_tiles,
                                                        int* __restrict__ digit_totals) {
    __shared__ int s_warp[8];
    __shared__ int s_carry;
    const int d = blockIdx.x;
    int* row = hist + (size_t)d * num_tiles;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    for (int base = 0; base < num_tiles; base += 256) {
        const int j = base + threadIdx.x;
        const int v = j < num_tiles ? row[j] : 0;
        int inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        if (lane == 31) s_warp[warp] = inc;
        __syncthreads();
        int wpre = 0, tot = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            int s = s_warp[w];
            if (w < warp) wpre += s;
            tot += s;
        }
        const int carry = s_carry;
        if (j < num_tiles) row[j] = carry + wpre + inc - v;
        __syncthreads();
        if (threadIdx.x == 0) s_carry = carry + tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) digit_totals[d] = s_carry;
}

template <typename K, int ITEMS>
__global__ void __launch_bounds__(kSortThreads) sort_downsweep_kernel(
    const K* __restrict__ keys_in, const int* __restrict__ vals_in, K* __restrict__ keys_out,
    int* __restrict__ vals_out, int n, int shift, unsigned mask, const int* __restrict__ hist,
    const int* __restrict__ digit_totals, int num_tiles) {
    constexpr int kTile = kSortThreads * ITEMS;
    extern __shared__ __align__(16) unsigned char s_raw[];
    K* s_keys = reinterpret_cast<K*>(s_raw);
    int* s_vals = reinterpret_cast<int*>(s_raw + sizeof(K) * kTile);
    int* s_cnt = s_vals + kTile;                  // [kSortWarps][kRadix]
    int* s_local_start = s_cnt + kSortWarps * kRadix;  // [kRadix]
    int* s_global = s_local_start + kRadix;       // [kRadix]
    __shared__ int s_warp_sums[kSortWarps];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned lanemask_lt = (1u << lane) - 1u;
    const int tile_base = blockIdx.x * kTile;
    const int tile_n = min(kTile, n - tile_base);

    for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) s_cnt[i] = 0;

    // Global base of each digit: exclusive scan over digits of digit_totals
    // plus this tile's offset within the digit.
    {
        const int d = threadIdx.x;  // kSortThreads == kRadix
        const int tot = digit_totals[d];
        int inc = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        if (lane == 31) s_warp_sums[warp] = inc;
        __syncthreads();
        int wpre = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w)
            if (w < warp) wpre += s_warp_sums[w];
        s_global[d] = wpre + inc - tot + hist[(size_t)d * num_tiles + blockIdx.x];
    }

    K key[ITEMS];
    int val[ITEMS];
    int rank[ITEMS];
    unsigned dig[ITEMS];
    const int wbase = tile_base + warp * (kTile / kSortWarps);
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int idx = wbase + i * 32 + lane;
        const bool ok = idx < n;
        key[i] = ok ? keys_in[idx] : K(0);
        val[i] = ok ? vals_in[idx] : 0;
        dig[i] = ok ? digit_of(key[i], shift, mask) : 0xFFFFu;
    }
    __syncthreads();

    // Per-warp stable ranking: rank = running count of the digit in this warp
    // before this 32-key step + number of lower lanes with the same digit.
    int* my_cnt = s_cnt + warp * kRadix;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const bool ok = dig[i] != 0xFFFFu;
        const unsigned active = __ballot_sync(0xffffffffu, ok);
        unsigned peers = __match_any_sync(0xffffffffu, dig[i]);
        peers &= active;
        int before = 0;
        if (ok) before = my_cnt[dig[i]];
        __syncwarp();
        if (ok) {
            rank[i] = before + __popc(peers & lanemask_lt);
            const int leader = __ffs(peers) - 1;
            if (lane == leader) my_cnt[dig[i]] = before + __popc(peers);
        } else {
            rank[i] = 0;
        }
        __syncwarp();
    }
    __syncthreads();

    // Per digit: exclusive prefix over warps, tile total, then the tile-local
    // start of each digit.
    {
        const int d = threadIdx.x;
        int run = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) {
            const int c = s_cnt[w * kRadix + d];
            s_cnt[w * kRadix + d] = run;
            run += c;
        }
        int inc = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        __syncthreads();
        if (lane == 31) s_warp_sums[warp] = inc;
        __syncthreads();
        int wpre = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w)
            if (w < warp) wpre += s_warp_sums[w];
        s_local_start[d] = wpre + inc - run;
    }
    __syncthreads();

#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        if (dig[i] != 0xFFFFu) {
            const int pos = s_local_start[dig[i]] + s_cnt[warp * kRadix + dig[i]] + rank[i];
            s_keys[pos] = key[i];
            s_vals[pos] = val[i];
        }
    }
    __syncthreads();

    for (int j = threadIdx.x; j < tile_n; j += kSortThreads) {
        const K k = s_keys[j];
        const unsigned d = digit_of(k, shift, mask);
        const int g = s_global[d] + (j - s_local_start[d]);
        keys_out[g] = k;
        vals_out[g] = s_vals[j];
    }
}

template <typename K>
size_t sort_workspace_bytes(int n) {
    // histogram sized for the smaller tiles, which need the most rows
    const int tiles = ceil_div(n > 0 ? n : 1, kSortThreads * 4);
    return align256(sizeof(K) * (size_t)n) + align256(sizeof(int) * (size_t)n) +
           align256(sizeof(int) * (size_t)kRadix * tiles) + align256(sizeof(int) * kRadix);
}

template <typename K, int ITEMS>
int sort_passes(const K* keys_in, const int* vals_in, K* keys_out, int* vals_out, int n,
                int begin_bit, int end_bit, K* alt_keys, int* alt_vals, int* hist, int* totals,
                cudaStream_t stream) {
    constexpr int kTile = kSortThreads * ITEMS;
    const int tiles = ceil_div(n, kTile);
    const size_t smem = sizeof(K) * kTile + sizeof(int) * kTile +
                        sizeof(int) * (kSortWarps * kRadix + 2 * kRadix);
    // the dynamic shared-memory limit is raised once per device (host threads
    // may sort concurrently: the flags are atomic)
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        HX_CUDA_TRY(cudaFuncSetAttribute(sort_downsweep_kernel<K, ITEMS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    const int bits = end_bit - begin_bit;
    const int passes = (bits + 7) / 8;
    int shift = begin_bit;
    const K* src_k = keys_in;
    const int* src_v = vals_in;
    for (int p_i = 0; p_i < passes; ++p_i) {
        // Spread the bits evenly over the passes.
        const int remaining = end_bit - shift;
        const int pass_bits = (remaining + (passes - p_i) - 1) / (passes - p_i);
        const unsigned mask = (1u << pass_bits) - 1u;
        // The last pass writes the caller's output buffers.
        const bool to_out = ((passes - 1 - p_i) % 2) == 0;
        K* dst_k = to_out ? keys_out : alt_keys;
        int* dst_v = to_out ? vals_out : alt_vals;
        sort_upsweep_kernel<K, ITEMS><<<tiles, kSortThreads, 0, stream>>>(src_k, n, shift, mask,
                                                                         hist, tiles);
        HX_LAUNCH_CHECK("sort_upsweep_kernel");
        sort_scan_kernel<<<kRadix, 256, 0, stream>>>(hist, tiles, totals);
        HX_LAUNCH_CHECK("sort_scan_kernel");
        sort_downsweep_kernel<K, ITEMS><<<tiles, kSortThreads, smem, stream>>>(
            src_k, src_v, dst_k, dst_v, n, shift, mask, hist, totals, tiles);
        HX_LAUNCH_CHECK("sort_downsweep_kernel");
        src_k = dst_k;
        src_v = dst_v;
        shift += pass_bits;
    }
    return HX_OK;
}

template <typename K>
int sort_pairs(const K* keys_in, const int* vals_in, K* keys_out, int* vals_out, int n,
               int begin_bit, int end_bit, void* ws, size_t ws_bytes, cudaStream_t stream) {
    HX_REQUIRE(n >= 0, "sort: n must be non-negative (got %d)", n);
    HX_REQUIRE(begin_bit >= 0 && end_bit <= (int)(8 * sizeof(K)) && begin_bit <= end_bit,
               "sort: invalid bit range [%d, %d)", begin_bit, end_bit);
    if (n == 0) return HX_OK;
    HX_REQUIRE(keys_in && vals_in && keys_out && vals_out, "sort: null pointer");
    if (!ws || ws_bytes < sort_workspace_bytes<K>(n))
        return set_error(HX_ERR_WORKSPACE, "sort: workspace of %zu bytes needed",
                         sort_workspace_bytes<K>(n));
    const int bits = end_bit - begin_bit;
    if (bits == 0) {
        HX_CUDA_TRY(cudaMemcpyAsync(keys_out, keys_in, sizeof(K) * (size_t)n,
                                    cudaMemcpyDeviceToDevice, stream));
        HX_CUDA_TRY(cudaMemcpyAsync(vals_out, vals_in, sizeof(int) * (size_t)n,
                                    cudaMemcpyDeviceToDevice, stream));
        return HX_OK;
    }
    const int max_tiles = ceil_div(n, kSortThreads * 4);
    char* p = (char*)ws;
    K* alt_keys = (K*)p;
    p += align256(sizeof(K) * (size_t)n);
    int* alt_vals = (int*)p;
    p += align256(sizeof(int) * (size_t)n);
    int* hist = (int*)p;
    p += align256(sizeof(int) * (size_t)kRadix * max_tiles);
    int* totals = (int*)p;
    if (sort_items(n) == 4)
        return sort_passes<K, 4>(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit,
                                 alt_keys, alt_vals, hist, totals, stream);
    return sort_passes<K, 16>(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit,
                              alt_keys, alt_vals, hist, totals, stream);
}

template int sort_pairs<uint32_t>(const uint32_t*, const int*, uint32_t*, int*, int, int, int,
                                  void*, size_t, cudaStream_t);
template int sort_pairs<unsigned long long>(const unsigned long long*, const int*,
                                            unsigned long long*, int*, int, int, int, void*,
                                            size_t, cudaStream_t);
template size_t sort_workspace_bytes<uint32_t>(int);
template size_t sort_workspace_bytes<unsigned long long>(int);

}  // namespace hx

using namespace hx;

extern "C" size_t hx_sort_pairs_workspace_bytes(int n, int key_bytes) {
    return key_bytes == 8 ? sort_workspace_bytes<unsigned long long>(n)
                          : sort_workspace_bytes<uint32_t>(n);
}

extern "C" int hx_sort_pairs_u64(const uint64_t* keys_in, const int32_t* vals_in,
                                 uint64_t* keys_out, int32_t* vals_out, int n, int begin_bit,
                                 int end_bit, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream) {
    return sort_pairs<unsigned long long>((const unsigned long long*)keys_in, vals_in,
                                          (unsigned long long*)keys_out, vals_out, n, begin_bit,
                                          end_bit, workspace, workspace_bytes, stream);
}

extern "C" int hx_sort_pairs_u32(const uint32_t* keys_in, const int32_t* vals_in,
                                 uint32_t* keys_out, int32_t* vals_out, int n, int begin_bit,
                                 int end_bit, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream) {
    return sort_pairs<uint32_t>(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit,
                                workspace, workspace_bytes, stream);
}
