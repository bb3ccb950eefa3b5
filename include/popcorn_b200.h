/*
 * popcorn_b200.h -- entry points that this B200 build adds beside the popcorn
 * ABI in popcorn.h. None of them changes or replaces a popcorn entry point.
 * Conventions (device pointers, null -> POPCORN_ERROR_INVALID_VALUE, sizes
 * <= 0 -> no-op, asynchronous on `stream`) are those of popcorn.h.
 */
#ifndef POPCORN_B200_H
#define POPCORN_B200_H

#include "popcorn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Kernel paths of the dequant-matmul. */
typedef enum {
    /* What popcornDequantizeMatmul_i8f32 picks for the shape and pointers. */
    POPCORN_MATMUL_PATH_AUTO = 0,
    /* f32 CUDA-core path: int8 codes are widened exactly to f32 and every
     * product is accumulated in f32 (max relative error ~1e-6 normwise).
     * Runs any shape and any alignment. */
    POPCORN_MATMUL_PATH_SIMT_F32 = 1,
    /* tcgen05 tensor-core path. Up to 128 activation rows (K <= 65536): each
     * row becomes 16-bit fixed point (rint(x * 32512 / max|x|)) held as two
     * int8 digits, the int8 codes multiply them on the int8 tensor cores with
     * exact int32 sums (~4e-5 normwise). More rows: codes become f16 (exact),
     * each activation row is rescaled by a power of two and rounded to f16,
     * products accumulate in f32 in tensor memory (~2e-4 normwise). Needs
     * K % 16 == 0 and a 16-byte aligned qweight. Takes stream-ordered scratch
     * (about M*K*2 bytes, plus up to 10 MB of split-K partials) from a
     * library-private memory pool. */
    POPCORN_MATMUL_PATH_TENSOR_F16 = 2,
} popcornMatmulPath_t;

/*
 * Dequantize (expand) per-channel int8 weights to f32:
 *   out[n, k] = (float)qweight[n, k] * scale[n]
 * popcorn has no kernel for this; the arithmetic is the per-element weight
 * expansion inside popcorn's fused matmul (src/quantize.cu:71) and in its
 * round-trip test (test/test_quantize.cu:996-1000). Results are bit-exact.
 */
popcornStatus_t popcornDequantize_i8f32(
    float* out,
    const int8_t* qweight,
    const float* scale,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * The same expansion with bf16 output, for callers that keep expanded
 * weights in bf16 (half the bytes of f32): out[n, k] holds the bf16 bit
 * pattern of (float)qweight[n, k] * scale[n] -- the f32 product above,
 * rounded once to nearest even. Bit-exact.
 */
popcornStatus_t popcornDequantize_i8bf16(
    uint16_t* out,
    const int8_t* qweight,
    const float* scale,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * popcornDequantizeMatmul_i8f32 with the kernel path chosen by the caller.
 * Returns POPCORN_ERROR_INVALID_VALUE when `path` cannot run this shape or
 * these pointers (for example the tensor path with K % 16 != 0).
 */
popcornStatus_t popcornDequantizeMatmulPath_i8f32(
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    popcornMatmulPath_t path,
    cudaStream_t stream
);

/* The path popcornDequantizeMatmul_i8f32 takes for these sizes and pointers
 * (never POPCORN_MATMUL_PATH_AUTO). Pure host function, launches nothing. */
popcornMatmulPath_t popcornDequantizeMatmulSelectPath(
    const float* x,
    const int8_t* qweight,
    int64_t M,
    int64_t N,
    int64_t K
);

/* Number of kernel launches the call with these arguments enqueues (0 for a
 * no-op or an argument error). Pure host function. */
int popcornDequantizeMatmulLaunchCount(
    const float* x,
    const int8_t* qweight,
    int64_t M,
    int64_t N,
    int64_t K,
    popcornMatmulPath_t path
);

/*
 * popcornDequantizeMatmul_i8f32 on the tensor-core path for callers that
 * cannot let a library allocate device memory: processes that hand out all
 * GPU memory through their own allocator (a cgo service accounting for every
 * byte, a server reserving HBM for its caches) or that forbid allocation after
 * start-up so a steady-state step can never fail or stall on it. There is no
 * counterpart in the reference; popcorn's ABI has no scratch-free variant.
 *
 * It allocates nothing: its scratch is one fixed device array inside this
 * library (16 MiB for the converted activations, 64 KiB for row scales and
 * 10 MiB for split-K partial tiles) that every GPU loading the library holds
 * until the process exits. Limits: K % 16 == 0,
 * 16-byte aligned qweight, M <= 16384 and M*K*2 rounded up to 256 bytes
 * <= 16 MiB (for example M = 2048 with K = 4096); anything larger, or a shape
 * the tensor path cannot run, returns POPCORN_ERROR_INVALID_VALUE without
 * launching. It runs the same kernels, so its results equal
 * popcornDequantizeMatmulPath_i8f32 with POPCORN_MATMUL_PATH_TENSOR_F16.
 *
 * The first call on a device also looks up the array's device address and
 * sets kernel attributes for that device; make that first call before any
 * stream capture. Every call shares the one array and it keeps the last
 * call's contents (nothing in it needs to start at zero): calls whose kernels
 * overlap on the GPU -- on different streams, or from different host threads
 * -- race on it and must be serialised by the caller.
 */
popcornStatus_t popcornDequantizeMatmulNoAlloc_i8f32(
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/* Diagnostic: copies the current device's kernel error bits into *flags and
 * clears them (synchronous). Non-zero bits mean a bounded wait (1 s) inside
 * a kernel gave up -- the kernel ended early instead of hanging -- and the
 * results of that launch are not valid. Bits 0-15: tensor-core kernels
 * (pipeline barriers). Bits 16-31, shifted by 16: 0x100 a fused collective
 * waited for another rank's values, 0x200 a decode kernel waited for the
 * weight rows it staged in shared memory, 0x400 the int4 decode kernel
 * likewise, 0x1000 the per-group int8 decode kernel likewise. */
int popcornB200DeviceErrors(unsigned int* flags);

/*
 * Fused neighbours of the dequant-matmul in a transformer block: the same
 * results as the popcorn call sequences named below, in one pass over the
 * activations and without the intermediate tensors. Arithmetic: popcorn's
 * RMSNorm (src/reduction.cu:290-321: rms = sqrtf(sum(x^2) / K + eps),
 * x * (1 / rms) * norm_weight[k], norm_weight may be NULL) and SiLU
 * (src/unary.cu:76-81: g / (1 + expf(-g))); only the order of the sum of
 * squares and of the k-sum differ, so results agree with the sequence to f32
 * rounding (f32 path) or ~4e-4 normwise (tensor path, large M). Null
 * buffers other than norm_weight -> POPCORN_ERROR_INVALID_VALUE; any size
 * <= 0 -> no-op. Small problems, unaligned operands and K % 16 != 0 run the
 * unfused sequence inside the library (with stream-ordered scratch from its
 * pool).
 */

/* out = DequantizeMatmul(RMSNorm(x; norm_weight, eps), qweight, scale):
 * popcornRMSNorm_f32 followed by popcornDequantizeMatmul_i8f32. */
popcornStatus_t popcornRMSNormDequantizeMatmul_i8f32(
    float* out,
    const float* x,
    const float* norm_weight,
    float eps,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/* out = silu(x @ (q_gate * s_gate)^T) * (x @ (q_up * s_up)^T): two
 * popcornDequantizeMatmul_i8f32 calls, popcornSilu_f32 on the first result,
 * popcornMul_f32 of the two. q_gate/q_up are [N, K], s_gate/s_up [N]. */
popcornStatus_t popcornDequantizeMatmulSiluMul_i8f32(
    float* out,
    const float* x,
    const int8_t* q_gate,
    const float* s_gate,
    const int8_t* q_up,
    const float* s_up,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/* Both: out = silu(RMSNorm(x) @ W_gate^T) * (RMSNorm(x) @ W_up^T), the front
 * half of a gated MLP block. */
popcornStatus_t popcornRMSNormDequantizeMatmulSiluMul_i8f32(
    float* out,
    const float* x,
    const float* norm_weight,
    float eps,
    const int8_t* q_gate,
    const float* s_gate,
    const int8_t* q_up,
    const float* s_up,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

#ifdef __cplusplus
}
#endif

#endif /* POPCORN_B200_H */
