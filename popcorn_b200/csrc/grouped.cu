// Per-group int8: popcornDequantizeMatmulGrouped_i8f32 and
// popcornQuantizeGrouped_f32i8 (popcorn src/quantize.cu:114-218, :567-697).
//
// Semantics (popcorn): scale is [N, K / group_size]; the weight of (n, k) is
// code * scale[n, k / group_size]; quantization gives every group of a row
// its own symmetric scale max|v| / 127 (1 when 0, NaN skipped by the compare)
// and codes rint(v / scale) clamped to [-128, 127].
//
// Kernels:
//  * grouped_seq_kernel -- one thread per output walking k upward with
//    w = code * scale and acc = fma(x, w, acc): popcorn's operation sequence,
//    bit-identical to its kernel. Used for small problems, group sizes that
//    are not a multiple of 16 and unaligned operands.
//  * grouped_xs_kernel<MT, U, R> -- the x-stationary decode layout of the
//    f32 GEMV (each thread keeps U 16-element slices of x in registers and
//    reads one 16-byte chunk of R weight rows per slice): a slice lies inside
//    one group (group_size % 16 == 0), so its partial sum is multiplied by
//    that group's scale before the fixed-order warp and block reductions.
//    Arithmetic is f32 (exact code widening, packed FMA); results are within
//    f32 rounding of popcorn's.
//  * grouped_quantize_kernel -- one warp per (row, group): the group max by
//    shuffles with popcorn's NaN-skipping compare, then the codes; bit-
//    identical to popcorn's two kernels, with no temporary buffer.
#include "common.cuh"

namespace pcb {
namespace {

constexpr int kGThreads = 256;
constexpr int kGWarps = kGThreads / 32;

__device__ __forceinline__ int8_t quantize_code(float v, float sc) {
    float q = rintf(v / sc);
    if (q > 127.0f) q = 127.0f;
    if (q < -128.0f) q = -128.0f;
    return static_cast<int8_t>(q);
}

// Four int8 codes (one word) -> four exact floats: byte code ^ 0x80 in the low
// mantissa byte of 2^23 is 2^23 + 128 + code; subtracting 2^23 + 128 is exact.
__device__ __forceinline__ void widen4(uint32_t word, float2& lo, float2& hi) {
    const uint32_t b = word ^ 0x80808080u;
    const float2 magic = make_float2(-8388736.0f, -8388736.0f);
    float2 a, c;
    a.x = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440));
    a.y = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7441));
    c.x = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7442));
    c.y = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7443));
    lo = __fadd2_rn(a, magic);
    hi = __fadd2_rn(c, magic);
}

// Butterfly reduce-scatter of V values over a warp: afterwards the lanes with
// (lane % (32 / V)) == 0 hold the warp total of value lane / (32 / V).
template <int V>
__device__ __forceinline__ float reduce_scatter(float (&v)[V], int lane) {
    int cnt = V;
    #pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (cnt > 1) {
            const int half = cnt >> 1;
            const bool up = (lane & off) != 0;
            #pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < half) {
                    const float send = up ? v[i] : v[i + half];
                    const float keep = up ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
    return v[0];
}

__global__ void __launch_bounds__(256)
grouped_seq_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
                   const float* __restrict__ scale, int64_t M, int64_t N, int64_t K, int64_t gs) {
    const int64_t groups = K / gs;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < M * N; t += stride) {
        const int64_t n = t % N;
        const int64_t m = t / N;
        const float* xr = x + m * K;
        const int8_t* qr = q + n * K;
        const float* sr = scale + n * groups;
        float acc = 0.0f;
        for (int64_t k0 = 0; k0 < K; k0 += gs, ++sr) {  // group by group: k / gs without a division
            const float sc = __ldg(sr);
            for (int64_t k = k0; k < k0 + gs; ++k) {
                const float w = static_cast<float>(__ldg(qr + k)) * sc;
                acc = __fmaf_rn(__ldg(xr + k), w, acc);
            }
        }
        out[t] = acc;
    }
}

// MT activation rows (<= 4), U 16-element K slices per thread, R weight rows
// per block (one group of rows per block).
// M = 1 with one slice per thread fits 64 registers: four blocks per SM, so a
// decode-sized grid (N / 8 blocks) is resident in one wave.
template <int MT, int U, int R>
__global__ void __launch_bounds__(kGThreads, (MT == 1 && U == 1) ? 4 : 2)
grouped_xs_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
                  const float* __restrict__ scale, int64_t M, int64_t N, int64_t K, int64_t gs) {
    __shared__ float part[R * MT][kGWarps];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t units = K >> 4;
    const int64_t groups = K / gs;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * R;

    // Programmatic dependent launch: release the next kernel of the stream,
    // pull this block's weight rows and scales into L2 while the previous
    // kernel finishes (a hint; every real read follows the wait).
    pdl_launch_dependents();
    if (tid < kGWarps + 1 && blockIdx.y == 0) {
        const int64_t rows = (r0 + R <= N) ? R : N - r0;
        if (tid < kGWarps) {
            prefetch_l2_range(q + r0 * K, rows * K, tid, kGWarps);
        } else {
            prefetch_l2_range(scale + r0 * groups, rows * groups * 4, 0, 1);
        }
    }
    pdl_wait();

    // Weight rows of this block (independent of x: requested first), and the
    // group of each of this thread's slices (group_size is a multiple of 16).
    uint4 w[R][U];
    int grp[U];
    const int units_per_group = static_cast<int>(gs >> 4);
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        const int unit = tid + u * kGThreads;
        grp[u] = unit / units_per_group;
        #pragma unroll
        for (int r = 0; r < R; ++r) {
            w[r][u] = (r0 + r < N && unit < units) ? __ldg(reinterpret_cast<const uint4*>(q + (r0 + r) * K) + unit)
                                                    : make_uint4(0u, 0u, 0u, 0u);
        }
    }

    // One block per (row group, MT activation rows): gridDim.y = ceil(M / MT).
    // (A loop over activation-row chunks here keeps far more registers live.)
    {
        const int64_t m0 = static_cast<int64_t>(blockIdx.y) * MT;
        float acc[R * MT];
        #pragma unroll
        for (int i = 0; i < R * MT; ++i) acc[i] = 0.0f;
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kGThreads;
            float2 xv[MT][8];
            #pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (unit < units && m0 + m < M) {
                    const float4* p = reinterpret_cast<const float4*>(x + (m0 + m) * K + unit * 16);
                    #pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float4 v = __ldg(p + c);
                        xv[m][2 * c] = make_float2(v.x, v.y);
                        xv[m][2 * c + 1] = make_float2(v.z, v.w);
                    }
                } else {
                    #pragma unroll
                    for (int c = 0; c < 8; ++c) xv[m][c] = make_float2(0.0f, 0.0f);
                }
            }
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                const float sc = (r0 + r < N && unit < units) ? __ldg(scale + (r0 + r) * groups + grp[u]) : 0.0f;
                const uint32_t words[4] = {w[r][u].x, w[r][u].y, w[r][u].z, w[r][u].w};
                float2 a[MT];
                #pragma unroll
                for (int m = 0; m < MT; ++m) a[m] = make_float2(0.0f, 0.0f);
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float2 lo, hi;
                    widen4(words[c], lo, hi);
                    #pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        a[m] = __ffma2_rn(xv[m][2 * c], lo, a[m]);
                        a[m] = __ffma2_rn(xv[m][2 * c + 1], hi, a[m]);
                    }
                }
                #pragma unroll
                for (int m = 0; m < MT; ++m) acc[r * MT + m] = fmaf(a[m].x + a[m].y, sc, acc[r * MT + m]);
            }
        }
        constexpr int V = R * MT;
        const float total = reduce_scatter<V>(acc, lane);
        constexpr int span = 32 / V;
        if ((lane % span) == 0) part[lane / span][warp] = total;
        __syncthreads();
        if (tid < V) {
            const int r = tid / MT;
            const int m = tid % MT;
            float s = 0.0f;
            #pragma unroll
            for (int wv = 0; wv < kGWarps; ++wv) s += part[tid][wv];
            if (r0 + r < N && m0 + m < M) out[(m0 + m) * N + r0 + r] = s;
        }
        __syncthreads();
    }
}

// One warp per (row, group); grid-stride over all groups.
__global__ void __launch_bounds__(256)
grouped_quantize_kernel(int8_t* __restrict__ out, float* __restrict__ scale, const float* __restrict__ in,
                        int64_t N, int64_t K, int64_t gs) {
    const int lane = threadIdx.x & 31;
    const int64_t groups = K / gs;
    const int64_t total = N * groups;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < total;
         item += nwarps) {
        const int64_t row = item / groups;
        const int64_t g = item - row * groups;
        const float* r = in + row * K + g * gs;
        int8_t* o = out + row * K + g * gs;
        float mx = 0.0f;
        for (int64_t i = lane; i < gs; i += 32) {
            const float v = __ldg(r + i);
            const float a = v < 0 ? -v : v;
            if (a > mx) mx = a;  // NaN compares false and is skipped
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, mx, off);
            if (other > mx) mx = other;
        }
        float sc = mx / 127.0f;
        if (sc == 0.0f) sc = 1.0f;
        if (lane == 0) scale[item] = sc;
        for (int64_t i = lane; i < gs; i += 32) o[i] = quantize_code(__ldg(r + i), sc);
    }
}

template <int MT, int U, int R>
popcornStatus_t launch_grouped_xs(float* out, const float* x, const int8_t* q, const float* scale, int64_t M,
                                  int64_t N, int64_t K, int64_t gs, cudaStream_t stream) {
    const int64_t gx = ceil_div(N, R);
    const int64_t gy = ceil_div(M, MT);
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)),
                                              dim3(kGThreads), 0, stream, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, grouped_xs_kernel<MT, U, R>, out, x, q, scale, M, N, K, gs);
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

}  // namespace
}  // namespace pcb

extern "C" popcornStatus_t popcornDequantizeMatmulGrouped_i8f32(float* out, const float* x, const int8_t* qweight,
                                                               const float* scale, int64_t M, int64_t N, int64_t K,
                                                               int64_t group_size, cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (group_size <= 0 || K % group_size != 0) return POPCORN_ERROR_INVALID_VALUE;
    // More than four activation rows and >= 2^27 multiply-adds: tensor cores,
    // the group factors applied by the converters.
    if (M > 4 && static_cast<double>(M) * static_cast<double>(N) * static_cast<double>(K) >= 134217728.0 &&
        tc_grouped_supported(qweight, M, N, K, group_size)) {
        return tc_dequant_matmul_grouped(kFmtGroup8, out, x, qweight, scale, nullptr, M, N, K, group_size, stream);
    }
    const bool aligned = aligned16(x) && aligned16(qweight) && K % 16 == 0;
    const int64_t slices = ceil_div(K / 16, kGThreads);
    const bool tiny = M * N * K <= (int64_t{1} << 22);
    const bool grid_ok = ceil_div(M, 4) <= 65535 && ceil_div(N, 2) <= 0x7FFFFFFF;
    if (!tiny && aligned && group_size % 16 == 0 && slices <= 4 && grid_ok) {
        if (M == 1) {
            if (slices == 1) return launch_grouped_xs<1, 1, 8>(out, x, qweight, scale, M, N, K, group_size, stream);
            if (slices == 2) return launch_grouped_xs<1, 2, 4>(out, x, qweight, scale, M, N, K, group_size, stream);
            return launch_grouped_xs<1, 4, 2>(out, x, qweight, scale, M, N, K, group_size, stream);
        }
        if (M == 2 && slices <= 2) {
            if (slices == 1) return launch_grouped_xs<2, 1, 8>(out, x, qweight, scale, M, N, K, group_size, stream);
            return launch_grouped_xs<2, 2, 4>(out, x, qweight, scale, M, N, K, group_size, stream);
        }
        if (slices == 1) return launch_grouped_xs<4, 1, 4>(out, x, qweight, scale, M, N, K, group_size, stream);
    }
    int64_t blocks = ceil_div(M * N, 256);
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 32;
    if (blocks > cap) blocks = cap;
    grouped_seq_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(out, x, qweight, scale, M, N, K,
                                                                          group_size);
    return check_launch();
}

extern "C" popcornStatus_t popcornQuantizeGrouped_f32i8(int8_t* out, float* scale, const float* input, int64_t N,
                                                       int64_t K, int64_t group_size, cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || scale == nullptr || input == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (group_size <= 0 || K % group_size != 0) return POPCORN_ERROR_INVALID_VALUE;
    const int64_t items = N * (K / group_size);
    int64_t blocks = ceil_div(items, kGWarps);
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    grouped_quantize_kernel<<<static_cast<unsigned>(blocks), kGThreads, 0, stream>>>(out, scale, input, N, K,
                                                                                    group_size);
    return check_launch();
}
