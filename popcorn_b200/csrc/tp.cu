// Tensor-parallel decode entry points (include/popcorn_tp.h): argument checks
// and the translation of popcornTpGroup_t into the kernel's PeerArgs.
#include "common.cuh"
#include "popcorn_tp.h"

namespace {

using namespace pcb;

// Null and range checks shared by both entry points; `words` is how many
// 8-byte receive slots one call needs in each half of the receive areas.
popcornStatus_t check_group(const popcornTpGroup_t* group, int64_t words, PeerArgs& pa) {
    if (group->world < 1 || group->world > kPeerMaxRanks || group->rank < 0 || group->rank >= group->world) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (group->state == nullptr || group->recv_bytes < 0) return POPCORN_ERROR_INVALID_VALUE;
    for (int p = 0; p < group->world; ++p) {
        if (group->recv[p] == nullptr || (reinterpret_cast<uintptr_t>(group->recv[p]) & 7u) != 0) {
            return POPCORN_ERROR_INVALID_VALUE;
        }
        pa.recv[p] = static_cast<unsigned long long*>(group->recv[p]);
    }
    pa.half_words = group->recv_bytes / 16;
    if (words > pa.half_words) return POPCORN_ERROR_INVALID_VALUE;
    pa.state = group->state;
    pa.rank = group->rank;
    pa.world = group->world;
    return POPCORN_SUCCESS;
}

}  // namespace

extern "C" popcornStatus_t popcornDequantizeMatmulAllGather_i8f32(const popcornTpGroup_t* group, float* out,
                                                                 const float* x, const int8_t* qweight,
                                                                 const float* scale, int64_t M, int64_t n_offset,
                                                                 int64_t n_local, int64_t N, int64_t K,
                                                                 cudaStream_t stream) {
    if (group == nullptr || out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || n_local <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (n_offset < 0 || n_local > N || n_offset > N - n_local) return POPCORN_ERROR_INVALID_VALUE;
    if (!peer_supported(x, qweight, M, K) || N > (int64_t{1} << 31)) return POPCORN_ERROR_INVALID_VALUE;
    PeerArgs pa = {};
    const popcornStatus_t st = check_group(group, M * N, pa);
    if (st != POPCORN_SUCCESS) return st;
    pa.n_offset = n_offset;
    pa.n_total = N;
    return peer_dequant_matmul(kPeerGather, pa, out, x, qweight, scale, M, n_local, K, stream);
}

extern "C" popcornStatus_t popcornDequantizeMatmulAllReduce_i8f32(const popcornTpGroup_t* group, float* out,
                                                                 const float* x, const int8_t* qweight,
                                                                 const float* scale, int64_t M, int64_t N, int64_t K,
                                                                 cudaStream_t stream) {
    if (group == nullptr || out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (!peer_supported(x, qweight, M, K) || N > (int64_t{1} << 31)) return POPCORN_ERROR_INVALID_VALUE;
    PeerArgs pa = {};
    const popcornStatus_t st = check_group(group, group->world * M * N, pa);
    if (st != POPCORN_SUCCESS) return st;
    pa.n_offset = 0;
    pa.n_total = N;
    return peer_dequant_matmul(kPeerReduce, pa, out, x, qweight, scale, M, N, K, stream);
}
