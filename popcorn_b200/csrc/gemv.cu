// f32 CUDA-core dequant-matmul path: out[m, n] = scale[n] * sum_k x[m, k] * q[n, k].
//
// This is the small-M (decode) kernel. Its arithmetic follows popcorn's
// dequantizeMatmulKernel_i8f32 (src/quantize.cu:18-84): int8 codes widened
// exactly to f32, products accumulated in f32. Two deliberate differences: the
// per-channel scale is applied once to the finished sum instead of to every
// code (the scale factors out of the k-sum), and the k-sum is split across
// lanes and combined by a shuffle tree, so rounding differs from popcorn's
// sequential sum by a few f32 ulps of the accumulated magnitude.
//
// Layout in HBM: x row-major [M, K] f32, q row-major [N, K] int8, out [M, N].
// Each warp owns NR weight rows and streams them with 16-byte loads (lane l
// reads bytes [16l, 16l+16) of every 512-byte segment, so one warp load
// instruction is one fully used 512-byte span). The activation chunk is staged
// once per block in shared memory with an XOR swizzle on 16-byte units so the
// lane-strided 16-byte reads are bank-conflict free. Codes are widened with
// the exponent trick: byte b^0x80 placed in the low mantissa of 2^23 gives
// the float 2^23 + 128 + code; subtracting 2^23 + 128 is exact.
//
// Roofline: HBM. Algorithmic bytes per launch = N*K (int8 weights); x, scale
// and out add 4*(M*K + N + M*N).
#include "common.cuh"

namespace pcb {
namespace {

constexpr int kGemvWarps = 4;              // warps per block
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kChunk = 4096;               // activations staged per pass (elements)
constexpr int kSeg = 512;                  // weight bytes one warp load covers
constexpr int kSegsPerChunk = kChunk / kSeg;
constexpr int kUnitsPerChunk = kChunk / 4; // 16-byte units per staged row

__device__ __forceinline__ int swz(int u) { return u ^ ((u >> 3) & 7); }

// Four int8 codes (one 32-bit word) -> four exact floats.
__device__ __forceinline__ void widen4(uint32_t word, float2& lo, float2& hi) {
    const uint32_t b = word ^ 0x80808080u;
    const float2 magic = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    float2 a, c;
    a.x = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440));
    a.y = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7441));
    c.x = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7442));
    c.y = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7443));
    lo = __fadd2_rn(a, magic);
    hi = __fadd2_rn(c, magic);
}

template <int MT, int NR>
__global__ void __launch_bounds__(kGemvThreads)
gemv_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
            const float* __restrict__ scale, int64_t M, int64_t N, int64_t K) {
    extern __shared__ float4 xs[];  // [MT][kUnitsPerChunk], swizzled
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t n0 = (static_cast<int64_t>(blockIdx.x) * kGemvWarps + warp) * NR;

    for (int64_t m0 = static_cast<int64_t>(blockIdx.y) * MT; m0 < M; m0 += static_cast<int64_t>(gridDim.y) * MT) {
        float2 acc[MT][NR];
        #pragma unroll
        for (int m = 0; m < MT; ++m)
            #pragma unroll
            for (int r = 0; r < NR; ++r) acc[m][r] = make_float2(0.0f, 0.0f);

        for (int64_t kc = 0; kc < K; kc += kChunk) {
            const int kn = static_cast<int>((K - kc) < kChunk ? (K - kc) : kChunk);  // multiple of 16

            // Issue this chunk's weight loads first so they are in flight while
            // the block stages the activations.
            uint4 w[kSegsPerChunk][NR];
            #pragma unroll
            for (int s = 0; s < kSegsPerChunk; ++s) {
                const int k = s * kSeg + lane * 16;
                #pragma unroll
                for (int r = 0; r < NR; ++r) {
                    if (k < kn && n0 + r < N) {
                        w[s][r] = __ldg(reinterpret_cast<const uint4*>(q + (n0 + r) * K + kc + k));
                    } else {
                        w[s][r] = make_uint4(0x0u, 0x0u, 0x0u, 0x0u);  // code 0
                    }
                }
            }

            __syncthreads();  // previous chunk's readers are done with xs
            const int units = ((kn + kSeg - 1) / kSeg) * (kSeg / 4);
            #pragma unroll
            for (int m = 0; m < MT; ++m) {
                const bool row_ok = (m0 + m) < M;
                const float4* xr = reinterpret_cast<const float4*>(x + (m0 + m) * K + kc);
                for (int u = threadIdx.x; u < units; u += kGemvThreads) {
                    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (row_ok && u * 4 < kn) v = __ldg(xr + u);
                    xs[m * kUnitsPerChunk + swz(u)] = v;
                }
            }
            __syncthreads();

            if (n0 < N) {
                #pragma unroll
                for (int s = 0; s < kSegsPerChunk; ++s) {
                    if (s * kSeg >= kn) break;
                    float2 xv[MT][8];
                    #pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        #pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const float4 v = xs[m * kUnitsPerChunk + swz(s * (kSeg / 4) + lane * 4 + c)];
                            xv[m][2 * c] = make_float2(v.x, v.y);
                            xv[m][2 * c + 1] = make_float2(v.z, v.w);
                        }
                    }
                    #pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        const uint32_t words[4] = {w[s][r].x, w[s][r].y, w[s][r].z, w[s][r].w};
                        #pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            float2 lo, hi;
                            widen4(words[c], lo, hi);
                            #pragma unroll
                            for (int m = 0; m < MT; ++m) {
                                acc[m][r] = __ffma2_rn(xv[m][2 * c], lo, acc[m][r]);
                                acc[m][r] = __ffma2_rn(xv[m][2 * c + 1], hi, acc[m][r]);
                            }
                        }
                    }
                }
            }
        }

        #pragma unroll
        for (int m = 0; m < MT; ++m) {
            #pragma unroll
            for (int r = 0; r < NR; ++r) {
                float v = acc[m][r].x + acc[m][r].y;
                #pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                if (lane == 0 && n0 + r < N && m0 + m < M) {
                    out[(m0 + m) * N + n0 + r] = v * __ldg(scale + n0 + r);
                }
            }
        }
    }
}

// Any shape, any alignment: one warp per (weight row, activation row) pair,
// scalar loads. Used when the vector kernel's K % 16 / alignment rules fail.
__global__ void __launch_bounds__(256)
generic_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
               const float* __restrict__ scale, int64_t M, int64_t N, int64_t K) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < M * N; t += nwarps) {
        const int64_t n = t % N;
        const int64_t m = t / N;
        const float* xr = x + m * K;
        const int8_t* qr = q + n * K;
        float acc = 0.0f;
        for (int64_t k = lane; k < K; k += 32) acc = fmaf(__ldg(xr + k), static_cast<float>(__ldg(qr + k)), acc);
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) out[m * N + n] = acc * __ldg(scale + n);
    }
}

bool vector_ok(const float* x, const int8_t* q, int64_t K) {
    return (K % 16 == 0) && aligned16(x) && aligned16(q);
}

constexpr int kMaxDevices = 64;
bool g_smem_set[kMaxDevices][3] = {};

template <int MT, int NR>
popcornStatus_t launch_gemv(int slot, float* out, const float* x, const int8_t* q, const float* scale,
                            int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    const int smem = MT * kChunk * static_cast<int>(sizeof(float));
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && dev >= 0 && dev < kMaxDevices && !g_smem_set[dev][slot]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<MT, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return record_cuda(e);
        g_smem_set[dev][slot] = true;
    }
    const int64_t gx = ceil_div(N, static_cast<int64_t>(kGemvWarps) * NR);
    int64_t gy = ceil_div(M, MT);
    if (gy > 65535) gy = 65535;
    if (gx > 0x7fffffff) return POPCORN_ERROR_INVALID_VALUE;
    dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
    gemv_kernel<MT, NR><<<grid, kGemvThreads, smem, stream>>>(out, x, q, scale, M, N, K);
    return check_launch();
}

}  // namespace

int simt_launch_count(const float*, const int8_t*, int64_t M, int64_t N, int64_t K) {
    return (M > 0 && N > 0 && K > 0) ? 1 : 0;
}

popcornStatus_t simt_dequant_matmul(float* out, const float* x, const int8_t* q, const float* scale,
                                    int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    if (!vector_ok(x, q, K)) {
        int64_t warps = M * N;
        int64_t blocks = ceil_div(warps, 8);
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
        if (blocks > cap) blocks = cap;
        generic_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(out, x, q, scale, M, N, K);
        return check_launch();
    }
    if (M == 1) return launch_gemv<1, 2>(0, out, x, q, scale, M, N, K, stream);
    if (M == 2) return launch_gemv<2, 2>(1, out, x, q, scale, M, N, K, stream);
    return launch_gemv<4, 2>(2, out, x, q, scale, M, N, K, stream);
}

}  // namespace pcb
