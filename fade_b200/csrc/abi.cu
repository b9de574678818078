// Library-wide C ABI helpers: status strings, version, last CUDA error.
#include <atomic>

#include "common.cuh"

namespace fade {
static std::atomic<int> g_last_cuda_error{0};
void set_last_cuda_error(int e) { g_last_cuda_error.store(e); }
}  // namespace fade

extern "C" const char* fade_status_string(int status) {
    switch (status) {
        case FADE_OK: return "ok";
        case FADE_ERR_INVALID_ARG: return "invalid argument";
        case FADE_ERR_ODD_DIM: return "last dim must be divisible by the packing factor";
        case FADE_ERR_GROUP: return "S must be divisible by group_size";
        case FADE_ERR_UNSUPPORTED: return "shape or dtype combination not supported by the sm_100a kernels";
        case FADE_ERR_ALIGN: return "pointer or stride violates the 16-byte alignment rule";
        case FADE_ERR_WORKSPACE: return "workspace missing or too small";
        case FADE_ERR_CUDA: return "CUDA runtime error";
        case FADE_ERR_TIMEOUT: return "a bounded device wait timed out";
        default: return "unknown status";
    }
}

extern "C" int fade_version(void) { return 100; }

extern "C" int fade_last_cuda_error(void) { return fade::g_last_cuda_error.load(); }

extern "C" int fade_set_device(int device) {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur == device) return FADE_OK;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        fade::set_last_cuda_error((int)e);
        return FADE_ERR_CUDA;
    }
    return FADE_OK;
}

extern "C" int fade_sm_count(void) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return n;
}
