// popcorn ABI entry points of the dequant-matmul and the path selection.
//
// Argument handling is popcorn's (src/quantize.cu:96-102, :311-317): null
// buffers -> POPCORN_ERROR_INVALID_VALUE, checked before sizes; any size <= 0
// -> POPCORN_SUCCESS without work; launch errors -> POPCORN_ERROR_CUDA.
#include "common.cuh"

namespace pcb {
namespace {

// More than four activation rows and more than this many multiply-adds take
// the tensor path: measured on a B200 it beats every CUDA-core variant there
// (M = 5..8: N = 2048, K = 4096 8.1 us against 10.3 us; N = K = 4096 9.1
// against 15.0 us). Smaller calls are launch-bound on any path and stay on
// the f32 path, whose results match popcorn's to f32 rounding -- popcorn's
// own test fixtures (M = 16, N = K = 1024: 2^24) keep its 1e-5 absolute
// tolerance.
constexpr int64_t kTensorMinMacs = int64_t(1) << 25;
// Up to this many activation rows the CUDA cores keep up with HBM.
constexpr int64_t kSimtMaxRows = 4;

bool mul_overflows(int64_t a, int64_t b) {
    return a != 0 && b > INT64_MAX / a;
}

popcornMatmulPath_t select_path(const float* x, const int8_t* q, int64_t M, int64_t N, int64_t K) {
    if (M > kSimtMaxRows && !mul_overflows(M, N) && !mul_overflows(M * N, K) &&
        M * N * K > kTensorMinMacs && tc_supported(x, q, M, N, K)) {
        return POPCORN_MATMUL_PATH_TENSOR_F16;
    }
    return POPCORN_MATMUL_PATH_SIMT_F32;
}

popcornStatus_t run(float* out, const float* x, const int8_t* q, const float* scale,
                    int64_t M, int64_t N, int64_t K, popcornMatmulPath_t path, cudaStream_t stream) {
    if (path == POPCORN_MATMUL_PATH_AUTO) path = select_path(x, q, M, N, K);
    switch (path) {
        case POPCORN_MATMUL_PATH_SIMT_F32:
            return simt_dequant_matmul(out, x, q, scale, M, N, K, stream);
        case POPCORN_MATMUL_PATH_TENSOR_F16:
            if (!tc_supported(x, q, M, N, K)) return POPCORN_ERROR_INVALID_VALUE;
            return tc_dequant_matmul(out, x, q, scale, M, N, K, stream);
        default:
            return POPCORN_ERROR_INVALID_VALUE;
    }
}

}  // namespace
}  // namespace pcb

extern "C" popcornStatus_t popcornDequantizeMatmul_i8f32(float* out, const float* x, const int8_t* qweight,
                                                         const float* scale, int64_t M, int64_t N, int64_t K,
                                                         cudaStream_t stream) {
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    return pcb::run(out, x, qweight, scale, M, N, K, POPCORN_MATMUL_PATH_AUTO, stream);
}

extern "C" popcornStatus_t popcornDequantizeMatmulBatched_i8f32(float* out, const float* x, const int8_t* qweight,
                                                                const float* scale, int64_t B, int64_t M, int64_t N,
                                                                int64_t K, cudaStream_t stream) {
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (B <= 0 || M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (pcb::mul_overflows(B, M)) return POPCORN_ERROR_INVALID_VALUE;
    // x is contiguous [B, M, K] and out contiguous [B, M, N]: one matmul over
    // B*M rows reads the shared weights once instead of once per batch.
    return pcb::run(out, x, qweight, scale, B * M, N, K, POPCORN_MATMUL_PATH_AUTO, stream);
}

extern "C" popcornStatus_t popcornDequantizeMatmulPath_i8f32(float* out, const float* x, const int8_t* qweight,
                                                             const float* scale, int64_t M, int64_t N, int64_t K,
                                                             popcornMatmulPath_t path, cudaStream_t stream) {
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    return pcb::run(out, x, qweight, scale, M, N, K, path, stream);
}

extern "C" popcornMatmulPath_t popcornDequantizeMatmulSelectPath(const float* x, const int8_t* qweight,
                                                                 int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_MATMUL_PATH_SIMT_F32;
    return pcb::select_path(x, qweight, M, N, K);
}

extern "C" int popcornDequantizeMatmulLaunchCount(const float* x, const int8_t* qweight, int64_t M, int64_t N,
                                                  int64_t K, popcornMatmulPath_t path) {
    if (x == nullptr || qweight == nullptr || M <= 0 || N <= 0 || K <= 0) return 0;
    if (path == POPCORN_MATMUL_PATH_AUTO) path = pcb::select_path(x, qweight, M, N, K);
    if (path == POPCORN_MATMUL_PATH_TENSOR_F16) {
        return pcb::tc_supported(x, qweight, M, N, K) ? pcb::tc_launch_count(M, N, K) : 0;
    }
    return pcb::simt_launch_count(x, qweight, M, N, K);
}

extern "C" int popcornB200DeviceErrors(unsigned int* flags) {
    if (flags == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    unsigned int a = 0, b = 0, c = 0, d = 0;
    cudaError_t e = pcb::tc_take_errors(&a);
    if (e == cudaSuccess) e = pcb::gemv_take_errors(&b);
    if (e == cudaSuccess) e = pcb::i4_take_errors(&c);
    if (e == cudaSuccess) e = pcb::grouped_take_errors(&d);
    *flags = a | ((b | c | d) << 16);
    return pcb::record_cuda(e);
}
