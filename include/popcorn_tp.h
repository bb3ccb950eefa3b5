/*
 * popcorn_tp.h -- tensor-parallel decode entry points of the B200 build: one
 * process (or host thread) per GPU of a node, each call a GEMV whose
 * collective is fused into the same kernel over NVLink peer memory.
 * popcorn itself is single-GPU; nothing here changes popcorn.h, and neither
 * entry point has a counterpart in the reference (each replaces a
 * popcornDequantizeMatmul_i8f32 call followed by an NCCL collective).
 */
#ifndef POPCORN_TP_H
#define POPCORN_TP_H

#include "popcorn.h"

#ifdef __cplusplus
extern "C" {
#endif

#define POPCORN_TP_MAX_RANKS 8

/*
 * One rank's view of a tensor-parallel group.
 *   recv[p]     rank p's receive area as mapped on this rank's GPU (its own
 *               for p == rank, a peer mapping over NVLink otherwise:
 *               CUDA IPC / symmetric memory). 8-byte aligned, recv_bytes
 *               long on every rank, zero-filled before the first call.
 *   recv_bytes  size of each receive area. A call uses one half of it
 *               (alternating halves), so an all-gather needs
 *               recv_bytes >= 16 * M * N and an all-reduce
 *               recv_bytes >= 16 * world * M * N.
 *   state       two uint32 in this rank's device memory, zero at set-up
 *               (the group's call count and a block counter).
 *
 * Protocol: every output value crosses NVLink once, as one 8-byte store that
 * carries the f32 bits together with the call's sequence number, into the
 * receiving rank's area. The receiver's kernel polls its own area until every
 * value of this call is present, so no flag, fence or barrier follows the
 * data. Every rank must make the same sequence of calls on a group, on one
 * stream per rank; consecutive calls alternate halves of the receive areas,
 * which is what lets a rank that is one call ahead write without disturbing
 * a slower one. A rank whose data does not arrive within 1 s makes the
 * waiting kernel stop, leave the missing outputs unwritten and set an error
 * bit (popcornB200DeviceErrors). Only one exchange kernel may run on a GPU
 * at a time (its blocks must all be resident while they wait).
 */
typedef struct {
    void* recv[POPCORN_TP_MAX_RANKS];
    int64_t recv_bytes;
    unsigned int* state;
    int rank;
    int world;
} popcornTpGroup_t;

/*
 * Column-parallel decode layer, all-gather fused: this rank multiplies x
 * [M, K] (replicated on every rank) by its shard of output channels
 * (qweight [n_local, K] int8 and scale [n_local], rows n_offset ..
 * n_offset + n_local of the full [N, K] weight), writes them into columns
 * n_offset .. n_offset + n_local of its own out [M, N] f32 and sends them to
 * every other rank; the kernel completes once every other rank's columns have
 * arrived in `out`. Arithmetic is that of popcornDequantizeMatmul_i8f32 on
 * the f32 CUDA-core path, so `out` equals a single-GPU call bit for bit.
 * Supported: 1 <= M <= 4, K % 16 == 0, K <= 16384 (M = 1), 8192 (M = 2),
 * 4096 (M <= 4), 16-byte aligned x and qweight; otherwise
 * POPCORN_ERROR_INVALID_VALUE.
 */
popcornStatus_t popcornDequantizeMatmulAllGather_i8f32(
    const popcornTpGroup_t* group,
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t n_offset,
    int64_t n_local,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

/*
 * Row-parallel decode layer, all-reduce fused: this rank multiplies its
 * slice of the input channels, x [M, K] with qweight [N, K] (the rank's
 * column slice of the full weight, contiguous) and scale [N] (the full
 * per-channel scale), sends the partial [M, N] to every rank, and writes
 * out [M, N] = the sum of all ranks' partials, added in rank order
 * 0, 1, ..., world-1, so every rank holds identical bits. Against a
 * single-GPU call over the whole K the result differs by f32 rounding of the
 * split sum only. Same shape limits as the all-gather.
 */
popcornStatus_t popcornDequantizeMatmulAllReduce_i8f32(
    const popcornTpGroup_t* group,
    float* out,
    const float* x,
    const int8_t* qweight,
    const float* scale,
    int64_t M,
    int64_t N,
    int64_t K,
    cudaStream_t stream
);

#ifdef __cplusplus
}
#endif

#endif /* POPCORN_TP_H */
