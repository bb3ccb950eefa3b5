// Status strings and the per-thread CUDA error record
// (popcorn src/common.cuh:16-27, src/unary.cu:89-110).
//
// The record is popcorn's own: the C++17 inline thread_local variable
// __popcorn_last_cuda_error of popcorn's src/common.cuh, declared here with
// the same name and type. An inline variable is one object per program, so
// when this library is linked together with popcorn's other operators
// (unary.o, binary.o, ...) both write the same per-thread record, and
// popcornGetLastCudaError reports the last failure of either library. The
// three functions below are weak definitions for the same reason: popcorn's
// unary.o defines them too, and its (identical) strong definitions win
// without a duplicate-symbol error.
#include "common.cuh"

// One record per host thread, as in popcorn: a cgo caller has to query it from
// the OS thread that made the failing call.
inline thread_local cudaError_t __popcorn_last_cuda_error = cudaSuccess;

namespace pcb {

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

popcornStatus_t record_cuda(cudaError_t err) {
    if (err != cudaSuccess) {
        ::__popcorn_last_cuda_error = err;
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

extern "C" __attribute__((weak)) const char* popcornGetErrorString(popcornStatus_t status) {
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

extern "C" __attribute__((weak)) cudaError_t popcornGetLastCudaError(void) { return ::__popcorn_last_cuda_error; }

extern "C" __attribute__((weak)) const char* popcornGetLastCudaErrorString(void) {
    return cudaGetErrorString(::__popcorn_last_cuda_error);
}
