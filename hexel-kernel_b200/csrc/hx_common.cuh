// Shared definitions for the B200 hexel rasteriser kernels and their C-ABI.
//
// Every exported entry point is `extern "C"`, takes plain device pointers,
// sizes and a cudaStream_t, and returns an hx_status code.  A human-readable
// message for the last failure on the calling host thread is available from
// hx_last_error().  Nothing here allocates device memory: outputs and
// scratch ("workspace") are owned by the caller.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/hexel_b200.h"

namespace hx {

// Tile geometry and top-K width of the Image-GS / 2D-hexel kernels
// (reference gsplat/cuda/csrc/config.h:1-10).
constexpr int kBlockX = 16;
constexpr int kBlockY = 16;
constexpr int kBlockSize = kBlockX * kBlockY;
constexpr int kTopK = 10;
constexpr int kMaxChannels = 12;

// Records a formatted error for hx_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

// Checks the launch status of the last kernel on this thread.
int check_launch(const char* what);

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Rounds a byte count up to 256 so workspace sub-buffers stay aligned.
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace hx

#define HX_REQUIRE(cond, ...)                                              \
    do {                                                                   \
        if (!(cond)) return ::hx::set_error(HX_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

#define HX_CUDA_TRY(expr)                                                  \
    do {                                                                   \
        cudaError_t _e = (expr);                                           \
        if (_e != cudaSuccess)                                             \
            return ::hx::set_error(HX_ERR_CUDA, "%s failed: %s", #expr,   \
                                   cudaGetErrorString(_e));                \
    } while (0)

#define HX_LAUNCH_CHECK(what)                                              \
    do {                                                                   \
        int _rc = ::hx::check_launch(what);                                \
        if (_rc != HX_OK) return _rc;                                      \
    } while (0)
