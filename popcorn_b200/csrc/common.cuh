// Shared host/device plumbing of the B200 dequant-matmul library.
//
// Status handling follows popcorn's convention (src/common.cuh:16-27): a CUDA
// failure becomes POPCORN_ERROR_CUDA and the CUDA error code is remembered per
// host thread for popcornGetLastCudaError().
#ifndef POPCORN_B200_COMMON_CUH
#define POPCORN_B200_COMMON_CUH

#include <cuda_runtime.h>
#include <stdint.h>

#include "popcorn.h"
#include "popcorn_b200.h"

namespace pcb {

// Number of streaming multiprocessors on a B200.
constexpr int kB200Sms = 148;

// Ranks of one tensor-parallel group (GPUs of one node).
constexpr int kPeerMaxRanks = 8;

// Weight formats of the tensor-core path: per-channel int8 (one scale per
// row), per-group int8, per-group int4 with zero points.
enum WeightFormat : int { kFmtChannel = 0, kFmtGroup8 = 1, kFmtGroup4 = 2 };

// Collective fused into the decode GEMV.
enum PeerMode : int { kPeerNone = 0, kPeerGather = 1, kPeerReduce = 2 };

// Arguments of the fused decode GEMV + collective (passed by value to the kernel).
struct PeerArgs {
    unsigned long long* recv[kPeerMaxRanks];  // every rank's receive area, mapped on this GPU
    int64_t half_words;                       // 8-byte words in each half of a receive area
    unsigned int* state;                      // this rank's {call count, finished-block counter}
    int64_t n_offset;                         // all-gather: first output channel of this rank's shard
    int64_t n_total;                          // all-gather: output channels of the gathered result
    int rank;
    int world;
};

// Records `err` for popcornGetLastCudaError() and maps it to a status.
popcornStatus_t record_cuda(cudaError_t err);

// Launch-time check after a kernel launch: picks up launch-configuration
// errors (and, like popcorn, any sticky error left on the context).
inline popcornStatus_t check_launch() { return record_cuda(cudaGetLastError()); }

inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Streaming-multiprocessor count of the current device (cached per device).
int device_sm_count();

#ifdef __CUDACC__
// L2 prefetch hint for [p, p + bytes): the range is shrunk to 16-byte
// boundaries (the bulk prefetch's alignment; nothing outside the range is
// named) and split into `parts` pieces, of which the caller issues `part`.
__device__ __forceinline__ void prefetch_l2_range(const void* p, int64_t bytes, int part, int parts) {
    const uint64_t a = reinterpret_cast<uint64_t>(p);
    const uint64_t lo = (a + 15u) & ~uint64_t{15};
    const uint64_t hi = (a + static_cast<uint64_t>(bytes)) & ~uint64_t{15};
    if (hi <= lo) return;
    const uint64_t n = hi - lo;
    const uint64_t chunk = ((n + parts - 1) / parts + 15u) & ~uint64_t{15};
    const uint64_t c0 = static_cast<uint64_t>(part) * chunk;
    if (c0 >= n) return;
    const uint64_t c1 = (c0 + chunk < n) ? c0 + chunk : n;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo + c0), "r"(static_cast<uint32_t>(c1 - c0))
                 : "memory");
}

// Programmatic dependent launch, kernel side: let the next kernel of the
// stream begin launching now, and wait for the previous kernel's writes.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
#endif

// Host side: a launch configuration that allows programmatic dependent
// launch on `stream` (attr must outlive the launch call).
inline cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                     cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// ---------------------------------------------------------------------------
// Kernel-path entry points (implemented in gemv.cu / tc_gemm.cu).
// Each takes already validated arguments (non-null, all sizes > 0).
// ---------------------------------------------------------------------------

// f32 CUDA-core path, any shape and alignment.
popcornStatus_t simt_dequant_matmul(float* out, const float* x, const int8_t* q,
                                    const float* scale, int64_t M, int64_t N,
                                    int64_t K, cudaStream_t stream);
int simt_launch_count(const float* x, const int8_t* q, int64_t M, int64_t N, int64_t K);

// tcgen05 path; requires tc_supported(...).
bool tc_supported(const float* x, const int8_t* q, int64_t M, int64_t N, int64_t K);
popcornStatus_t tc_dequant_matmul(float* out, const float* x, const int8_t* q,
                                  const float* scale, int64_t M, int64_t N,
                                  int64_t K, cudaStream_t stream);
int tc_launch_count(int64_t M, int64_t N, int64_t K);

// tcgen05 path with the activation-side RMSNorm folded into the prologue
// (norm) and, with q_up, the gate/up pair: out = silu(x Wq^T) * (x Wup^T).
// Requires tc_supported(...) for q and q_up.
popcornStatus_t tc_dequant_matmul_fused(float* out, const float* x, const float* norm_w, float eps, bool norm,
                                        const int8_t* q, const float* scale, const int8_t* q_up, const float* s_up,
                                        int64_t M, int64_t N, int64_t K, cudaStream_t stream);

// Stream-ordered scratch from the library's private pool (kept between calls).
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t stream);
cudaError_t scratch_free(void* p, cudaStream_t stream);

// tcgen05 path for the per-group formats (int8 codes [N, K] or packed int4
// [N, K/2]; zero is null for int8); requires tc_grouped_supported(...).
bool tc_grouped_supported(const void* q, int64_t M, int64_t N, int64_t K, int64_t gs);
popcornStatus_t tc_dequant_matmul_grouped(WeightFormat fmt, float* out, const float* x, const void* q,
                                          const float* scale, const float* zero, int64_t M, int64_t N, int64_t K,
                                          int64_t gs, cudaStream_t stream);

// Fused decode GEMV + all-gather / all-reduce (gemv.cu). `rows` is the
// number of weight rows of this rank's call (n_local, or N for a reduce).
bool peer_supported(const float* x, const int8_t* q, int64_t M, int64_t K);
popcornStatus_t peer_dequant_matmul(PeerMode mode, const PeerArgs& pa, float* out, const float* x, const int8_t* q,
                                    const float* scale, int64_t M, int64_t rows, int64_t K, cudaStream_t stream);

// Read and clear the device error words of the bounded-wait kernels.
cudaError_t tc_take_errors(unsigned int* bits);
cudaError_t gemv_take_errors(unsigned int* bits);
cudaError_t i4_take_errors(unsigned int* bits);
cudaError_t grouped_take_errors(unsigned int* bits);

}  // namespace pcb

#endif  // POPCORN_B200_COMMON_CUH
