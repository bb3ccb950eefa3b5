/*
 * popcorn_tp_nccl.h -- tensor-parallel linear layers of any batch size M over
 * an NCCL communicator: one process (or host thread) per GPU of a node, each
 * rank holding its shard of the int8 weights. popcorn itself is single-GPU;
 * neither entry point has a counterpart in the reference (each replaces a
 * popcornDequantizeMatmul_i8f32 call followed by an NCCL collective, which a
 * cgo caller would otherwise have to issue itself).
 *
 * The communicator is the caller's (ncclCommInitRank or any other way); every
 * rank must make the same sequence of calls with the same sizes, each on the
 * stream it passes, which must be a stream of the communicator's GPU. The
 * library links NCCL dynamically (libnccl.so.2).
 *
 * Conventions are popcorn's: null buffers -> POPCORN_ERROR_INVALID_VALUE
 * (checked first), any size <= 0 -> POPCORN_SUCCESS with no work, a failed
 * kernel launch -> POPCORN_ERROR_CUDA (popcornGetLastCudaError); a failed
 * NCCL call -> POPCORN_ERROR_CUDA with the NCCL result kept per host thread
 * for popcornGetLastNcclError.
 */
#ifndef POPCORN_TP_NCCL_H
#define POPCORN_TP_NCCL_H

#include <nccl.h>

#include "popcorn.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Column-parallel layer: x [M, K] is replicated on every rank; this rank holds
 * output channels [rank * N / P, (rank + 1) * N / P) of the full [N, K]
 * weight (qweight [N / P, K], scale [N / P]; N % P == 0, P = communicator
 * size). Every rank ends with the full out [M, N] f32, the same bits on every
 * rank. Each channel is computed whole on one rank, so on the f32 CUDA-core
 * path (M <= 4) out equals a single-GPU popcornDequantizeMatmul_i8f32 over
 * the whole weight bit for bit; on the tensor path it agrees within that
 * path's tolerance (how K is split among a cluster depends on the shard's
 * width, which changes the order of the partial sums). `work` is
 * M * N floats of device scratch owned by the caller (the gathered shards
 * before they are interleaved into rows); it may be NULL when M == 1.
 */
popcornStatus_t popcornDequantizeMatmulColumnParallel_i8f32(
    ncclComm_t comm,
    float* out,
    float* work,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * Row-parallel layer: this rank holds input channels [k0, k0 + K) of the full
 * weight -- x [M, K] is its slice of the activations, qweight [N, K] its
 * column slice (contiguous), scale [N] the full per-channel scale. out
 * [M, N] f32 becomes, on every rank, the sum of all ranks' partial products
 * (ncclAllReduce, sum, in place on out), so it agrees with a single-GPU call
 * over the whole K to the rounding of the split sum.
 */
popcornStatus_t popcornDequantizeMatmulRowParallel_i8f32(
    ncclComm_t comm,
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/* The ncclResult_t of the last failed NCCL call made by this host thread
 * inside the two entry points above (ncclSuccess if none). */
ncclResult_t popcornGetLastNcclError(void);

#ifdef __cplusplus
}
#endif

#endif /* POPCORN_TP_NCCL_H */
