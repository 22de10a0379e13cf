// common.cu — error reporting, launch accounting and library identity.
#include "common.cuh"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

namespace warp {

static thread_local char g_err[512] = "";
static std::atomic<uint64_t> g_launches{0};

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return e == cudaErrorMemoryAllocation ? WARP_E_NOMEM : WARP_E_CUDA;
}

void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
    static const bool on = [] {
        const char *s = getenv("WARP_PDL");
        return !(s && s[0] == '0');
    }();
    return on;
}

}  // namespace warp

extern "C" const char *warp_version(void) { return "warp_b200 0.1 sm_100a"; }

extern "C" const char *warp_last_error(void) { return warp::g_err; }

extern "C" uint64_t warp_launch_count(void) {
    return warp::g_launches.load(std::memory_order_relaxed);
}

extern "C" int warp_device_ok(int dev) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || dev < 0 || dev >= n) {
        cudaGetLastError();
        return 0;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    return major == 10 && minor == 0;
}
