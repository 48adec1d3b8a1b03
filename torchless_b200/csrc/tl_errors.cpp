// tl_errors.cpp -- per-thread error message behind tl_last_error().
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "torchless_b200.h"

namespace tl {

namespace {
thread_local char g_msg[1024] = "";
}

tl_status set_error(tl_status s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return s;
}

void clear_error() { g_msg[0] = '\0'; }

int sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace tl

extern "C" {

const char* tl_last_error(void) { return tl::g_msg; }

const char* tl_status_name(tl_status s) {
    switch (s) {
        case TL_OK: return "TL_OK";
        case TL_ERR_INVALID_ARGUMENT: return "TL_ERR_INVALID_ARGUMENT";
        case TL_ERR_UNSUPPORTED: return "TL_ERR_UNSUPPORTED";
        case TL_ERR_IO: return "TL_ERR_IO";
        case TL_ERR_FORMAT: return "TL_ERR_FORMAT";
        case TL_ERR_CUDA: return "TL_ERR_CUDA";
        case TL_ERR_OUT_OF_MEMORY: return "TL_ERR_OUT_OF_MEMORY";
        case TL_ERR_CAPACITY: return "TL_ERR_CAPACITY";
        case TL_ERR_TIMEOUT: return "TL_ERR_TIMEOUT";
    }
    return "TL_ERR_UNKNOWN";
}

}  // extern "C"
