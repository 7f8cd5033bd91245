// Library-wide C ABI plumbing: status strings, the per-thread CUDA error
// record and the cached per-device SM count used to size grids.
#include "common.cuh"

#include <mutex>

namespace t4b {

namespace {
thread_local int g_last_cuda_error = 0;
std::mutex g_sm_mutex;
int g_sm_counts[64] = {0};
}  // namespace

int record_cuda_error(cudaError_t err) {
    g_last_cuda_error = (int)err;
    return T4B_ERR_CUDA;
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    {
        std::lock_guard<std::mutex> lock(g_sm_mutex);
        if (g_sm_counts[dev]) return g_sm_counts[dev];
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    std::lock_guard<std::mutex> lock(g_sm_mutex);
    g_sm_counts[dev] = n;
    return n;
}

}  // namespace t4b

extern "C" {

const char* t4b_status_string(int status) {
    switch (status) {
        case T4B_OK: return "ok";
        case T4B_ERR_INVALID_VALUE: return "invalid value (size, group size or mode out of range)";
        case T4B_ERR_NULL_POINTER: return "a required pointer is NULL";
        case T4B_ERR_MISALIGNED: return "a pointer is not aligned as the operation requires";
        case T4B_ERR_UNSUPPORTED: return "shape or option not supported by this build";
        case T4B_ERR_CUDA: return "CUDA runtime error (see t4b_last_cuda_error)";
        default: return "unknown status";
    }
}

int t4b_last_cuda_error(void) { return t4b::g_last_cuda_error; }

int t4b_version(void) { return (1 << 16) | 0; }

}  // extern "C"
