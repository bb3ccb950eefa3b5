// tcgen05 tensor-core dequant-matmul path (large M). Not enabled yet.
#include "common.cuh"

namespace pcb {

bool tc_supported(const float*, const int8_t*, int64_t, int64_t, int64_t) { return false; }

popcornStatus_t tc_dequant_matmul(float*, const float*, const int8_t*, const float*, int64_t, int64_t,
                                  int64_t, cudaStream_t) {
    return POPCORN_ERROR_INVALID_VALUE;
}

int tc_launch_count(int64_t, int64_t, int64_t) { return 0; }

}  // namespace pcb
