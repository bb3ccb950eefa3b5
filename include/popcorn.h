/*
 * popcorn.h -- C ABI of the int8 weight-only dequant-matmul path, built for
 * NVIDIA B200 (sm_100a).
 *
 * Every declaration below has the same name, parameter list, parameter
 * meaning, status codes and enumerator values as popcorn's public header
 * (popcorn include/popcorn.h), so a cgo or C caller that was built against
 * popcorn links against this library without source changes. Only the
 * quantized-linear subset of popcorn's ABI is provided here; the other popcorn
 * operators (elementwise, norms, backward, optimizer) are not part of this
 * library.
 *
 * Conventions shared by every entry point:
 *   - all buffers are device pointers owned by the caller;
 *   - a null buffer pointer returns POPCORN_ERROR_INVALID_VALUE before any
 *     size is looked at;
 *   - any size <= 0 is a no-op that returns POPCORN_SUCCESS;
 *   - work is enqueued asynchronously on `stream` (NULL = legacy default
 *     stream); only launch-time CUDA errors are reported, and the CUDA error
 *     code behind a POPCORN_ERROR_CUDA is kept per host thread.
 */
#ifndef POPCORN_H
#define POPCORN_H

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (popcorn include/popcorn.h:11-16). */
typedef enum {
    POPCORN_SUCCESS = 0,
    POPCORN_ERROR_INVALID_VALUE = 1,
    POPCORN_ERROR_CUDA = 2,
} popcornStatus_t;

/* Short description of a status code (popcorn include/popcorn.h:19,
 * src/unary.cu:91-102). */
const char* popcornGetErrorString(popcornStatus_t status);

/* The CUDA error behind the most recent POPCORN_ERROR_CUDA returned on the
 * calling host thread; cudaSuccess if there was none (popcorn
 * include/popcorn.h:21-23, src/common.cuh:16-27). */
cudaError_t popcornGetLastCudaError(void);

/* cudaGetErrorString() of popcornGetLastCudaError() (popcorn
 * include/popcorn.h:25-27, src/unary.cu:104-110). */
const char* popcornGetLastCudaErrorString(void);

/*
 * out[m, n] = sum_k x[m, k] * (qweight[n, k] * scale[n])
 *
 * Replaces popcorn's popcornDequantizeMatmul_i8f32 (include/popcorn.h:464-473,
 * src/quantize.cu:86-112). x is row-major [M, K] f32, qweight is row-major
 * [N, K] int8 (one row per output channel), scale is [N] f32 and out is
 * row-major [M, N] f32. Accumulation is f32. Small problems and M <= 4 run on
 * an f32 CUDA-core path; large problems run on the tcgen05 tensor-core path:
 * up to 128 activation rows as 16-bit fixed point per row (two int8 digits,
 * int8 tensor cores, exact int32 sums), more rows rounded to f16 after a
 * per-row power-of-two rescaling (normwise relative error well below 2e-3).
 */
popcornStatus_t popcornDequantizeMatmul_i8f32(
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * Batched form with weights shared across the batch:
 * out[b, m, n] = sum_k x[b, m, k] * (qweight[n, k] * scale[n]).
 *
 * Replaces popcorn's popcornDequantizeMatmulBatched_i8f32
 * (include/popcorn.h:491-501, src/quantize.cu:300-327). x is contiguous
 * [B, M, K] and out contiguous [B, M, N], so the call is the single matmul
 * above with B*M rows; the weights are streamed once, not once per batch.
 */
popcornStatus_t popcornDequantizeMatmulBatched_i8f32(
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t B,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * Symmetric per-output-channel int8 quantization of a row-major [N, K] f32
 * matrix:
 *   scale[n]  = max_k |input[n, k]| / 127   (1.0 when that maximum is 0)
 *   out[n, k] = rint(input[n, k] / scale[n]) clamped to [-128, 127]
 *
 * Replaces popcorn's popcornQuantize_f32i8 (include/popcorn.h:527-534,
 * src/quantize.cu:452-565). Codes and scales are bit-identical to popcorn's
 * GPU kernels (IEEE division, round-half-to-even, NaN skipped by the row
 * maximum). Unlike popcorn's version it allocates no temporary device memory
 * and does not synchronize the device, so it is stream-ordered.
 */
popcornStatus_t popcornQuantize_f32i8(
    int8_t* out,
    float* scale,
    const float* input,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * Per-group int8 dequant-matmul:
 *   out[m, n] = sum_k x[m, k] * (qweight[n, k] * scale[n, k / group_size])
 * with scale row-major [N, K / group_size]. group_size must be positive and
 * divide K (else POPCORN_ERROR_INVALID_VALUE, checked after the null
 * pointers and the size <= 0 no-op, as popcorn does).
 *
 * Replaces popcorn's popcornDequantizeMatmulGrouped_i8f32
 * (include/popcorn.h:475-487, src/quantize.cu:114-218). f32 arithmetic:
 * small problems and group sizes that are not a multiple of 16 follow
 * popcorn's own operation order (bit-identical to its kernel); otherwise the
 * group scale multiplies each 16-column partial sum, within f32 rounding of
 * popcorn's result.
 */
popcornStatus_t popcornDequantizeMatmulGrouped_i8f32(
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    int64_t group_size,
    cudaStream_t stream
);

/*
 * Per-group symmetric int8 quantization: every group of group_size
 * consecutive values of a row gets its own scale
 *   scale[n, g] = max |input[n, g*gs .. (g+1)*gs)| / 127   (1.0 when 0)
 *   out[n, k]   = rint(input[n, k] / scale[n, k / gs]) clamped to [-128, 127]
 *
 * Replaces popcorn's popcornQuantizeGrouped_f32i8 (include/popcorn.h:536-546,
 * src/quantize.cu:567-697): codes and scales bit-identical to its kernels,
 * no temporary allocation, no device synchronization.
 */
popcornStatus_t popcornQuantizeGrouped_f32i8(
    int8_t* out,
    float* scale,
    const float* input,
    int64_t N,
    int64_t K,
    int64_t group_size,
    cudaStream_t stream
);

/*
 * Int4 per-group asymmetric dequant-matmul:
 *   out[m, n] = sum_k x[m, k] * ((c(n, k) - zero[n, g]) * scale[n, g]),
 *   g = k / group_size,
 * where qweight is row-major [N, K/2] bytes holding two 4-bit codes each, the
 * even k in the low nibble: c(n, k) = qweight[n, k/2] & 0xF for even k and
 * qweight[n, k/2] >> 4 for odd k. scale and zero are row-major
 * [N, K / group_size]. group_size must be positive and divide K, and K must
 * be even (else POPCORN_ERROR_INVALID_VALUE, checked in that order after the
 * null pointers and the size <= 0 no-op, as popcorn does).
 *
 * Replaces popcorn's popcornDequantizeMatmulGrouped_i4f32
 * (include/popcorn.h:503-517, src/quantize.cu:329-446). f32 arithmetic:
 * small problems, group sizes that are not a multiple of 16 and unaligned
 * operands follow popcorn's own operation order (bit-identical to its
 * kernel); otherwise each 16-column slice applies its group's zero point and
 * scale once, within f32 rounding of popcorn's result.
 */
popcornStatus_t popcornDequantizeMatmulGrouped_i4f32(
    float* out,
    const float* x,
    const uint8_t* qweight,
    const float* scale,
    const float* zero,
    int64_t M,
    int64_t N,
    int64_t K,
    int64_t group_size,
    cudaStream_t stream
);

/*
 * Int4 per-group asymmetric quantization of a row-major [N, K] f32 matrix:
 *   scale[n, g] = (max - min) / 15 over the group (1.0 when that is 0)
 *   zero[n, g]  = -min / scale[n, g]
 *   code        = rint(input / scale + zero) clamped to [0, 15]
 * with min and max skipping NaN; codes are packed two per byte into out
 * [N, K/2], the even k in the low nibble. Argument checks as for the int4
 * matmul above.
 *
 * Replaces popcorn's popcornQuantizeGrouped_f32i4 (include/popcorn.h:548-562,
 * src/quantize.cu:699-888): packed codes, scales and zero points
 * bit-identical to its kernels, no temporary allocation, no device
 * synchronization.
 */
popcornStatus_t popcornQuantizeGrouped_f32i4(
    uint8_t* out,
    float* scale,
    float* zero,
    const float* input,
    int64_t N,
    int64_t K,
    int64_t group_size,
    cudaStream_t stream
);

#ifdef __cplusplus
}
#endif

#endif /* POPCORN_H */
