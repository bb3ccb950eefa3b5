// Tensor-parallel linear layers of any M over an NCCL communicator
// (include/popcorn_tp_nccl.h): the library's own matmul on this rank's shard,
// then the NCCL collective on the same stream.
//
// NCCL is resolved at run time, not linked: the process's already-loaded
// libnccl.so.2 is used when there is one (the one torch or a cgo program
// brought in), else libnccl.so.2 is opened. A hard dependency would let
// whichever libnccl.so.2 the loader found first serve every later user of
// that soname in the process.
#include <dlfcn.h>

#include <mutex>

#include "common.cuh"
#include "popcorn_tp_nccl.h"

namespace pcb {
namespace {

thread_local ncclResult_t t_last_nccl = ncclSuccess;

struct NcclApi {
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*count)(const ncclComm_t, int*);
    ncclResult_t (*user_rank)(const ncclComm_t, int*);
};

const NcclApi* nccl_api() {
    static NcclApi api = {};
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) return;
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.count = reinterpret_cast<decltype(api.count)>(dlsym(h, "ncclCommCount"));
        api.user_rank = reinterpret_cast<decltype(api.user_rank)>(dlsym(h, "ncclCommUserRank"));
        ok = api.all_gather && api.all_reduce && api.count && api.user_rank;
    });
    return ok ? &api : nullptr;
}

popcornStatus_t record_nccl(ncclResult_t r) {
    if (r != ncclSuccess) {
        t_last_nccl = r;
        return POPCORN_ERROR_CUDA;
    }
    return POPCORN_SUCCESS;
}

// out[m, p * w + j] = gathered[p][m][j]: the ranks' [M, w] shards, gathered
// rank after rank, interleaved into full rows.
__global__ void __launch_bounds__(256)
interleave_shards_kernel(float* __restrict__ out, const float* __restrict__ gathered, int64_t P, int64_t M,
                         int64_t w) {
    const int64_t total = P * M * w;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t p = t / (M * w);
        const int64_t r = t - p * M * w;
        const int64_t m = r / w;
        out[m * P * w + p * w + (r - m * w)] = gathered[t];
    }
}

}  // namespace
}  // namespace pcb

extern "C" popcornStatus_t popcornDequantizeMatmulColumnParallel_i8f32(ncclComm_t comm, float* out, float* work,
                                                                      const float* x, const int8_t* qweight,
                                                                      const float* scale, int64_t M, int64_t N,
                                                                      int64_t K, cudaStream_t stream) {
    using namespace pcb;
    if (comm == nullptr || out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (M > 1 && work == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    const NcclApi* nc = nccl_api();
    if (nc == nullptr) return record_nccl(ncclSystemError);
    int P = 0, rank = 0;
    popcornStatus_t st = record_nccl(nc->count(comm, &P));
    if (st == POPCORN_SUCCESS) st = record_nccl(nc->user_rank(comm, &rank));
    if (st != POPCORN_SUCCESS) return st;
    if (P < 1 || rank < 0 || rank >= P || N % P != 0) return POPCORN_ERROR_INVALID_VALUE;
    const int64_t w = N / P;
    // M == 1: the gathered shards [P][1][w] already are the output row.
    float* gathered = (M == 1) ? out : work;
    float* mine = gathered + static_cast<int64_t>(rank) * M * w;
    st = popcornDequantizeMatmul_i8f32(mine, x, qweight, scale, M, w, K, stream);
    if (st != POPCORN_SUCCESS) return st;
    if (P > 1) {
        st = record_nccl(nc->all_gather(mine, gathered, static_cast<size_t>(M * w), ncclFloat, comm, stream));
        if (st != POPCORN_SUCCESS) return st;
    }
    if (M > 1) {
        int64_t blocks = ceil_div(M * N, 256);
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
        if (blocks > cap) blocks = cap;
        interleave_shards_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(out, work, P, M, w);
        return check_launch();
    }
    return POPCORN_SUCCESS;
}

extern "C" popcornStatus_t popcornDequantizeMatmulRowParallel_i8f32(ncclComm_t comm, float* out, const float* x,
                                                                   const int8_t* qweight, const float* scale,
                                                                   int64_t M, int64_t N, int64_t K,
                                                                   cudaStream_t stream) {
    using namespace pcb;
    if (comm == nullptr || out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    const NcclApi* nc = nccl_api();
    if (nc == nullptr) return record_nccl(ncclSystemError);
    int P = 0;
    popcornStatus_t st = record_nccl(nc->count(comm, &P));
    if (st != POPCORN_SUCCESS) return st;
    st = popcornDequantizeMatmul_i8f32(out, x, qweight, scale, M, N, K, stream);
    if (st != POPCORN_SUCCESS || P == 1) return st;
    return record_nccl(nc->all_reduce(out, out, static_cast<size_t>(M * N), ncclFloat, ncclSum, comm, stream));
}

extern "C" ncclResult_t popcornGetLastNcclError(void) { return pcb::t_last_nccl; }
