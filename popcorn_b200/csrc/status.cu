// Status strings and the per-thread CUDA error record
// (popcorn src/common.cuh:16-27, src/unary.cu:89-110).
#include "common.cuh"

namespace pcb {

namespace {
// One record per host thread, as in popcorn: a cgo caller has to query it from
// the OS thread that made the failing call.
thread_local cudaError_t t_last_cuda_error = cudaSuccess;

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

popcornStatus_t record_cuda(cudaError_t err) {
    if (err != cudaSuccess) {
        t_last_cuda_error = err;
        return POPCORN_ERROR_CUDA;
    }
    return POPCORN_SUCCESS;
}

int device_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        return kB200Sms;
    }
    int n = __atomic_load_n(&g_sm_count[dev], __ATOMIC_RELAXED);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            n = kB200Sms;
        }
        __atomic_store_n(&g_sm_count[dev], n, __ATOMIC_RELAXED);
    }
    return n;
}

}  // namespace pcb

extern "C" const char* popcornGetErrorString(popcornStatus_t status) {
    switch (status) {
        case POPCORN_SUCCESS:
            return "success";
        case POPCORN_ERROR_INVALID_VALUE:
            return "invalid value";
        case POPCORN_ERROR_CUDA:
            return "CUDA error";
        default:
            return "unknown error";
    }
}

extern "C" cudaError_t popcornGetLastCudaError(void) { return pcb::t_last_cuda_error; }

extern "C" const char* popcornGetLastCudaErrorString(void) {
    return cudaGetErrorString(pcb::t_last_cuda_error);
}
