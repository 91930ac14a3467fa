// capi.cu -- status reporting and the per-device status word of the C ABI.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "ane_internal.h"

namespace ane {

static thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(ANE_CUDA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ANE_CUDA_OK;
}

// Cached per device; concurrent first calls from several host threads each
// store the same value (atomics, so there is no data race).
int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

int resident_grid(const void* kernel, int threads, size_t smem, int64_t want) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
        per_sm <= 0)
        per_sm = 1;
    const int64_t cap = (int64_t)per_sm * sm_count();
    if (want < 1) want = 1;
    return (int)(want < cap ? want : cap);
}

}  // namespace ane

extern "C" {

int ane_cuda_abi_version(void) { return 1; }

const char* ane_cuda_status_string(int status) {
    switch (status) {
        case ANE_CUDA_OK: return "ok";
        case ANE_CUDA_ERR_INVALID_ARG: return "invalid argument";
        case ANE_CUDA_ERR_UNSUPPORTED: return "unsupported";
        case ANE_CUDA_ERR_CUDA: return "CUDA error";
        default: return "unknown status";
    }
}

const char* ane_cuda_last_error(void) { return ane::g_last_error; }

}  // extern "C"
