// Inclusive int32 prefix sum (reduce-then-scan, three short kernels, no
// inter-block waiting).  Used for the per-primitive tile counts, which are at
// most a few million entries, so the second level fits one CTA.
#include "hx_common.cuh"

namespace hx {

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;  // 4096 elements per CTA
constexpr int kScanMaxPartials = 1024 * 16;

__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread (blockDim.x <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    int inc = warp_inclusive_scan(v);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? s_warp[lane] : 0;
        int winc = warp_inclusive_scan(w);
        s_warp[lane] = winc - w;
        if (lane == 31) s_warp[32] = winc;
    }
    __syncthreads();
    total = s_warp[32];
    int r = inc - v + s_warp[warp];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kScanThreads) scan_tiles_kernel(const int* __restrict__ in,
                                                                  int* __restrict__ out, int n,
                                                                  int* __restrict__ partials) {
    __shared__ int s_data[kScanTile];
    __shared__ int s_warp[33];
    const int base = blockIdx.x * kScanTile;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        int j = i * kScanThreads + threadIdx.x;
        s_data[j] = (base + j < n) ? in[base + j] : 0;
    }
    __syncthreads();
    int local[kScanItems];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        sum += s_data[threadIdx.x * kScanItems + i];
        local[i] = sum;
    }
    int total;
    int off = block_exclusive_scan(sum, s_warp, total);
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) s_data[threadIdx.x * kScanItems + i] = local[i] + off;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        int j = i * kScanThreads + threadIdx.x;
        if (base + j < n) out[base + j] = s_data[j];
    }
    if (threadIdx.x == 0) partials[blockIdx.x] = total;
}

// Exclusive scan of the per-CTA totals (one CTA of 1024 threads) and the
// 64-bit grand total.
__global__ void __launch_bounds__(1024) scan_partials_kernel(int* __restrict__ partials,
                                                            int count,
                                                            long long* __restrict__ total_out) {
    __shared__ int s_warp[33];
    __shared__ long long s_total;
    const int per = (count + blockDim.x - 1) / blockDim.x;
    const int begin = threadIdx.x * per;
    int vals[16];
    int sum = 0;
    long long sum64 = 0;
    for (int i = 0; i < per && i < 16; ++i) {
        int j = begin + i;
        int v = j < count ? partials[j] : 0;
        vals[i] = v;
        sum += v;
        sum64 += v;
    }
    if (threadIdx.x == 0) s_total = 0;
    __syncthreads();
    atomicAdd((unsigned long long*)&s_total, (unsigned long long)sum64);
    int total;
    int off = block_exclusive_scan(sum, s_warp, total);
    for (int i = 0; i < per && i < 16; ++i) {
        int j = begin + i;
        if (j < count) partials[j] = off;
        off += vals[i];
    }
    __syncthreads();
    if (threadIdx.x == 0 && total_out) *total_out = s_total;
}

__global__ void __launch_bounds__(256) scan_add_kernel(int* __restrict__ out, int n,
                                                       const int* __restrict__ partials) {
    const int b = blockIdx.x;
    const int add = partials[b];
    if (add == 0) return;
    const int base = b * kScanTile;
    for (int j = threadIdx.x; j < kScanTile; j += blockDim.x) {
        if (base + j < n) out[base + j] += add;
    }
}

}  // namespace hx

using namespace hx;

extern "C" size_t hx_scan_workspace_bytes(int n) {
    if (n <= 0) return 256;
    return align256((size_t)ceil_div(n, kScanTile) * sizeof(int));
}

extern "C" int hx_inclusive_scan_i32(const int32_t* in, int32_t* out, int n, int64_t* total_out,
                                     void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream) {
    HX_REQUIRE(n >= 0, "scan: n must be non-negative (got %d)", n);
    if (n == 0) {
        if (total_out) HX_CUDA_TRY(cudaMemsetAsync(total_out, 0, sizeof(int64_t), stream));
        return HX_OK;
    }
    HX_REQUIRE(in && out, "scan: null pointer");
    const int tiles = ceil_div(n, kScanTile);
    HX_REQUIRE(tiles <= kScanMaxPartials, "scan: n=%d exceeds the supported maximum %d", n,
               kScanMaxPartials * kScanTile);
    if (!workspace || workspace_bytes < hx_scan_workspace_bytes(n))
        return set_error(HX_ERR_WORKSPACE, "scan: workspace of %zu bytes needed",
                         hx_scan_workspace_bytes(n));
    int* partials = (int*)workspace;
    scan_tiles_kernel<<<tiles, kScanThreads, 0, stream>>>(in, out, n, partials);
    HX_LAUNCH_CHECK("scan_tiles_kernel");
    scan_partials_kernel<<<1, 1024, 0, stream>>>(partials, tiles, (long long*)total_out);
    HX_LAUNCH_CHECK("scan_partials_kernel");
    if (tiles > 1) {
        scan_add_kernel<<<tiles, 256, 0, stream>>>(out, n, partials);
        HX_LAUNCH_CHECK("scan_add_kernel");
    }
    return HX_OK;
}

// ---------------------------------------------------------------------------
// No-allocation variant: the per-CTA partial sums live in a fixed file-scope
// device array (kScanMaxPartials ints = 64 KiB, enough for n up to
// kScanMaxPartials * kScanTile = 67,108,864 elements) instead of a caller
// workspace.  Every call on a device shares that array; each call writes
// every partial it reads before reading it, so nothing needs clearing, but
// two calls that overlap on one device (concurrent streams or host threads)
// race on the array and must be serialised by the caller.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

static __device__ __align__(256) int g_noalloc_partials[kScanMaxPartials];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
int* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Address of this device's copy of the array, looked up once per device (on
// the first call with that device current) and cached.
int noalloc_partials(int** out) {
    int dev = -1;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    HX_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "scan_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
        if (e != cudaSuccess || p == nullptr)
            return set_error(HX_ERR_CUDA, "scan_noalloc: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<int*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return HX_OK;
}

}  // namespace

extern "C" int hx_inclusive_scan_i32_noalloc(const int32_t* in, int32_t* out, int n,
                                             int64_t* total_out, cudaStream_t stream) {
    HX_REQUIRE(n >= 0, "scan_noalloc: n must be non-negative (got %d)", n);
    HX_REQUIRE(n <= kScanMaxPartials * kScanTile,
               "scan_noalloc: n=%d exceeds the fixed scratch maximum of %d elements", n,
               kScanMaxPartials * kScanTile);
    int* partials = nullptr;
    const int rc = noalloc_partials(&partials);
    if (rc != HX_OK) return rc;
    if (n == 0) {
        if (total_out) HX_CUDA_TRY(cudaMemsetAsync(total_out, 0, sizeof(int64_t), stream));
        return HX_OK;
    }
    HX_REQUIRE(in && out, "scan_noalloc: null pointer");
    const int tiles = ceil_div(n, kScanTile);
    scan_tiles_kernel<<<tiles, kScanThreads, 0, stream>>>(in, out, n, partials);
    HX_LAUNCH_CHECK("scan_tiles_kernel");
    scan_partials_kernel<<<1, 1024, 0, stream>>>(partials, tiles, (long long*)total_out);
    HX_LAUNCH_CHECK("scan_partials_kernel");
    if (tiles > 1) {
        scan_add_kernel<<<tiles, 256, 0, stream>>>(out, n, partials);
        HX_LAUNCH_CHECK("scan_add_kernel");
    }
    return HX_OK;
}
