// Error reporting and version query of the C-ABI.
#include <stdarg.h>
#include <stdio.h>

#include "hx_common.cuh"

#include <atomic>

namespace {
thread_local char g_last_error[1024] = "";
// Kernels launched by this library since load (all devices, all threads).
std::atomic<unsigned long long> g_launches{0};
}

namespace hx {

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return set_error(HX_ERR_CUDA, "%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    }
    return HX_OK;
}

}  // namespace hx

extern "C" {

int hx_abi_version(void) { return HX_ABI_VERSION; }

const char* hx_last_error(void) { return g_last_error; }

void hx_clear_error(void) { g_last_error[0] = '\0'; }

unsigned long long hx_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
