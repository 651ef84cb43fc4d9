// Library identification, status strings and the thread-local error slot.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "skv_common.cuh"

namespace skv {

static thread_local char g_last_error[512] = "";
static std::atomic<long long> g_launches{0};

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return SKV_OK;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

}  // namespace skv

extern "C" {

const char* skv_version(void) { return "shadowkv_b200 0.1.0 (sm_100a)"; }

const char* skv_status_string(int status) {
    switch (status) {
        case SKV_OK: return "ok";
        case SKV_ERR_INVALID_ARGUMENT: return "invalid argument";
        case SKV_ERR_SHAPE: return "shape mismatch";
        case SKV_ERR_GROUP_SIZE: return "int4 group_size mismatch";
        case SKV_ERR_SCRATCH: return "scratch buffer too small";
        case SKV_ERR_TOO_LARGE: return "size beyond limit";
        case SKV_ERR_CUDA: return "CUDA error";
        case SKV_ERR_UNSUPPORTED: return "unsupported configuration";
        default: return "unknown status";
    }
}

const char* skv_last_error(void) { return skv::g_last_error; }

int64_t skv_launch_count(void) { return skv::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
