// Mean-squared-error loss and its gradient in one pass over the prediction
// and the target: every CTA walks a grid-stride range in float4 steps, writes
// the gradient, reduces its squared differences (warp shuffles, then one
// shared slot per warp) and adds its sum to the loss with one atomic.
#include "hx_common.cuh"

namespace hx {

constexpr int kLossThreads = 256;

// Scalar form for inputs that are not 16-byte aligned.
__global__ void __launch_bounds__(kLossThreads) l2_loss_grad_scalar_kernel(
    const float* __restrict__ pred, const float* __restrict__ target, int64_t n, float inv_n,
    float* __restrict__ grad, float* __restrict__ loss) {
    __shared__ float s_warp[kLossThreads / 32];
    const float g2 = 2.f * inv_n;
    float acc = 0.f;
    const int64_t stride = (int64_t)gridDim.x * kLossThreads;
    for (int64_t i = (int64_t)blockIdx.x * kLossThreads + threadIdx.x; i < n; i += stride) {
        const float d = pred[i] - target[i];
        grad[i] = d * g2;
        acc += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) s_warp[warp] = acc;
    __syncthreads();
    if (warp == 0) {
        acc = lane < kLossThreads / 32 ? s_warp[lane] : 0.f;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0 && acc != 0.f) atomicAdd(loss, acc * inv_n);
    }
}

__global__ void __launch_bounds__(kLossThreads) l2_loss_grad_kernel(
    const float4* __restrict__ pred, const float4* __restrict__ target, int64_t n4,
    const float* __restrict__ pred_tail, const float* __restrict__ target_tail, int tail,
    float inv_n, float4* __restrict__ grad, float* __restrict__ grad_tail,
    float* __restrict__ loss) {
    __shared__ float s_warp[kLossThreads / 32];
    const float g2 = 2.f * inv_n;
    float acc = 0.f;
    const int64_t stride = (int64_t)gridDim.x * kLossThreads;
    for (int64_t i = (int64_t)blockIdx.x * kLossThreads + threadIdx.x; i < n4; i += stride) {
        const float4 p = pred[i];
        const float4 t = target[i];
        const float4 d = make_float4(p.x - t.x, p.y - t.y, p.z - t.z, p.w - t.w);
        grad[i] = make_float4(d.x * g2, d.y * g2, d.z * g2, d.w * g2);
        acc += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
    }
    if (blockIdx.x == 0 && (int)threadIdx.x < tail) {
        const float d = pred_tail[threadIdx.x] - target_tail[threadIdx.x];
        grad_tail[threadIdx.x] = d * g2;
        acc += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) s_warp[warp] = acc;
    __syncthreads();
    if (warp == 0) {
        acc = lane < kLossThreads / 32 ? s_warp[lane] : 0.f;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0 && acc != 0.f) atomicAdd(loss, acc * inv_n);
    }
}

}  // namespace hx

using namespace hx;

extern "C" int hx_l2_loss_grad(const float* pred, const float* target, int64_t n, float inv_n,
                               float* grad, float* loss, cudaStream_t stream) {
    HX_REQUIRE(n >= 0, "l2_loss_grad: n must be non-negative");
    if (n == 0) return HX_OK;
    HX_REQUIRE(pred && target && grad && loss, "l2_loss_grad: null pointer");
    int dev = 0, sms = 0;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    HX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (((uintptr_t)pred | (uintptr_t)target | (uintptr_t)grad) % 16 != 0) {
        const int64_t want = (n + kLossThreads - 1) / kLossThreads;
        const int blocks = (int)(want < 4LL * sms ? want : 4LL * sms);
        l2_loss_grad_scalar_kernel<<<blocks, kLossThreads, 0, stream>>>(pred, target, n, inv_n,
                                                                        grad, loss);
        HX_LAUNCH_CHECK("l2_loss_grad_scalar_kernel");
        return HX_OK;
    }
    const int64_t n4 = n / 4;
    const int tail = (int)(n - 4 * n4);
    // a few waves of 256-thread CTAs: enough loads in flight for HBM, one
    // atomic per CTA
    const int64_t want = (n4 + kLossThreads - 1) / kLossThreads;
    const int blocks = (int)(want < 4LL * sms ? (want > 0 ? want : 1) : 4LL * sms);
    l2_loss_grad_kernel<<<blocks, kLossThreads, 0, stream>>>(
        (const float4*)pred, (const float4*)target, n4, pred + 4 * n4, target + 4 * n4, tail,
        inv_n, (float4*)grad, grad + 4 * n4, loss);
    HX_LAUNCH_CHECK("l2_loss_grad_kernel");
    return HX_OK;
}
