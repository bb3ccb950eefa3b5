// Per-output-channel int8 quantize and dequantize (expand) kernels.
//
// Quantize follows popcorn's two-kernel algorithm (src/quantize.cu:458-528):
// row maximum of |w| with NaN skipped (the `abs_v > max` compare, :473-476),
// scale = max / 127 with 0 mapped to 1 (:513-515), code = rint(w / scale)
// clamped to [-128, 127] (:523-527). Here both steps run in one kernel, one
// warp per row, so no temporary buffer, no cudaMalloc/cudaFree and no device
// synchronisation is needed (popcorn allocates one, :547-562). The division
// and rint are the IEEE round-to-nearest-even operations popcorn uses, so
// codes and scales are bit-identical. The division itself is replaced by a
// multiply with the row's reciprocal except within 1e-4 of a rounding
// boundary (quantize_one_rcp states the bound), which keeps the codes
// identical while taking the division off the per-element path.
//
// For 1024 <= K <= 16384 (K % 16 == 0, aligned) one block handles a row and
// holds it in registers between the max and the quantize step; otherwise one
// warp per row makes two passes (the second served by L2).
// Traffic per element: 4 B read from HBM, 1 B written; plus 4 B per row.
#include <cuda_bf16.h>

#include "common.cuh"

namespace pcb {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kWarpsPerBlock = kQuantThreads / 32;

__device__ __forceinline__ float absmax_step(float m, float v) {
    // fmaxf returns the non-NaN operand, so a NaN |v| is skipped exactly like
    // popcorn's `if (abs_v > max)`; m itself is never NaN (it starts at 0).
    return fmaxf(m, fabsf(v));
}

__device__ __forceinline__ int8_t quantize_one(float v, float sc) {
    float q = rintf(v / sc);
    if (q > 127.0f) q = 127.0f;
    if (q < -128.0f) q = -128.0f;
    return static_cast<int8_t>(q);
}

// The same code as quantize_one(v, sc), with the division replaced by a
// multiply wherever that cannot change the result. rcp = 1 / sc rounded to
// nearest (a normal number: the caller checks that sc is normal and finite).
// With Q = v / sc exactly and |Q| <= 127 (sc = max / 127 >= |v| / 127
// within 2^-24), t = v * rcp lies within |Q| (2^-24 + 2^-24 + 2^-48) and
// popcorn's rounded quotient fl(Q) within |Q| 2^-24 of Q, so |t - fl(Q)| <
// 127 * 1.8e-7 < 2.3e-5. When t is more than 1e-4 away from every
// half-integer, rint(t) = rint(fl(Q)); otherwise (and for NaN t, where the
// compare is false) the exact division decides, ties to even included.
__device__ __forceinline__ int8_t quantize_one_rcp(float v, float sc, float rcp) {
    const float t = v * rcp;
    const float q = rintf(t);
    // |v| <= max |row| and rcp = 1/sc to 1 ulp put |t| within a few ulps of
    // 127 at most, so a q that passes the test needs no clamp.
    if (fabsf(t - q) <= 0.4999f) return static_cast<int8_t>(q);
    return quantize_one(v, sc);
}

// Rows whose scale is not a finite normal number (a zero, denormal or
// infinite row maximum) keep the division for every element.
__device__ __forceinline__ bool rcp_ok(float sc) {
    return sc >= 1.17549435e-38f && sc <= 3.40282347e38f;
}

// kVec: K % 16 == 0 and both row bases 16-byte aligned; each lane then owns
// 16 consecutive elements per step (four 16-byte loads, one 16-byte store).
template <bool kVec>
__global__ void __launch_bounds__(kQuantThreads)
quantize_rows_kernel(int8_t* __restrict__ out, float* __restrict__ scale,
                     const float* __restrict__ in, int64_t N, int64_t K) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock) + (threadIdx.x >> 5);
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;

    for (int64_t row = warp; row < N; row += nwarps) {
        const float* r = in + row * K;
        int8_t* o = out + row * K;

        float m = 0.0f;
        if (kVec) {
            const float4* r4 = reinterpret_cast<const float4*>(r);
            const int64_t n4 = K >> 2;
            #pragma unroll 4
            for (int64_t i = lane; i < n4; i += 32) {
                float4 v = __ldg(r4 + i);
                m = absmax_step(m, v.x);
                m = absmax_step(m, v.y);
                m = absmax_step(m, v.z);
                m = absmax_step(m, v.w);
            }
        } else {
            for (int64_t k = lane; k < K; k += 32) m = absmax_step(m, __ldg(r + k));
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            float other = __shfl_xor_sync(0xffffffffu, m, off);
            m = (other > m) ? other : m;
        }

        float sc = m / 127.0f;
        if (sc == 0.0f) sc = 1.0f;
        if (lane == 0) scale[row] = sc;

        const bool fast = rcp_ok(sc);
        const float rcp = fast ? __frcp_rn(sc) : 0.0f;
        auto code = [&](float v) { return fast ? quantize_one_rcp(v, sc, rcp) : quantize_one(v, sc); };
        if (kVec) {
            const float4* r4 = reinterpret_cast<const float4*>(r);
            uint4* o16 = reinterpret_cast<uint4*>(o);
            const int64_t n16 = K >> 4;
            for (int64_t c = lane; c < n16; c += 32) {
                uint32_t w[4];
                #pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float4 v = __ldg(r4 + c * 4 + j);
                    uint32_t b0 = static_cast<uint8_t>(code(v.x));
                    uint32_t b1 = static_cast<uint8_t>(code(v.y));
                    uint32_t b2 = static_cast<uint8_t>(code(v.z));
                    uint32_t b3 = static_cast<uint8_t>(code(v.w));
                    w[j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
                }
                o16[c] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
            for (int64_t k = lane; k < K; k += 32) o[k] = code(__ldg(r + k));
        }
    }
}

// One block per row, the whole row held in registers (U 16-float slices per
// thread, K <= 16 * 256 * U): HBM is read exactly once, and each thread keeps
// all of its loads in flight at once. Needs K % 16 == 0 and aligned bases.
constexpr int kRowThreads = 256;

template <int U>
__global__ void __launch_bounds__(kRowThreads)
quantize_row_block_kernel(int8_t* __restrict__ out, float* __restrict__ scale, const float* __restrict__ in,
                          int64_t N, int64_t K) {
    __shared__ float red[2][kRowThreads / 32];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int64_t units = K >> 4;
    int parity = 0;
    for (int64_t row = blockIdx.x; row < N; row += gridDim.x, parity ^= 1) {
        const float4* r4 = reinterpret_cast<const float4*>(in + row * K);
        float4 v[U][4];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                v[u][c] = (unit < units) ? __ldg(r4 + unit * 4 + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
        float m = 0.0f;
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                m = absmax_step(m, v[u][c].x);
                m = absmax_step(m, v[u][c].y);
                m = absmax_step(m, v[u][c].z);
                m = absmax_step(m, v[u][c].w);
            }
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, m, off);
            m = (other > m) ? other : m;
        }
        if (lane == 0) red[parity][warp] = m;
        __syncthreads();
        m = red[parity][0];
        #pragma unroll
        for (int w = 1; w < kRowThreads / 32; ++w) {
            const float other = red[parity][w];
            m = (other > m) ? other : m;
        }
        float sc = m / 127.0f;
        if (sc == 0.0f) sc = 1.0f;
        if (tid == 0) scale[row] = sc;

        uint4* o16 = reinterpret_cast<uint4*>(out + row * K);
        const bool fast = rcp_ok(sc);
        const float rcp = fast ? __frcp_rn(sc) : 0.0f;
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
            if (unit < units) {
                uint32_t w[4];
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t b0, b1, b2, b3;
                    if (fast) {
                        b0 = static_cast<uint8_t>(quantize_one_rcp(v[u][c].x, sc, rcp));
                        b1 = static_cast<uint8_t>(quantize_one_rcp(v[u][c].y, sc, rcp));
                        b2 = static_cast<uint8_t>(quantize_one_rcp(v[u][c].z, sc, rcp));
                        b3 = static_cast<uint8_t>(quantize_one_rcp(v[u][c].w, sc, rcp));
                    } else {
                        b0 = static_cast<uint8_t>(quantize_one(v[u][c].x, sc));
                        b1 = static_cast<uint8_t>(quantize_one(v[u][c].y, sc));
                        b2 = static_cast<uint8_t>(quantize_one(v[u][c].z, sc));
                        b3 = static_cast<uint8_t>(quantize_one(v[u][c].w, sc));
                    }
                    w[c] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
                }
                o16[unit] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
}

// out[n, k] = float(q[n, k]) * scale[n]. kVec (K % 16 == 0, aligned bases):
// a block walks rows, its warps take 512-code chunks of the row; lane l
// reads code words l, 32 + l, 64 + l, 96 + l of the chunk (four 128-byte
// loads per warp) and store j writes outputs [128 j, 128 j + 128) of the
// chunk, so every warp store covers 512 contiguous bytes.
constexpr int kDeqThreads = 256;
constexpr int kDeqWarps = kDeqThreads / 32;

__device__ __forceinline__ float4 expand4(uint32_t w, float sc) {
    float4 v;
    v.x = static_cast<float>(static_cast<int8_t>(w & 0xffu)) * sc;
    v.y = static_cast<float>(static_cast<int8_t>((w >> 8) & 0xffu)) * sc;
    v.z = static_cast<float>(static_cast<int8_t>((w >> 16) & 0xffu)) * sc;
    v.w = static_cast<float>(static_cast<int8_t>(w >> 24)) * sc;
    return v;
}

template <bool kVec>
__global__ void __launch_bounds__(kDeqThreads)
dequantize_kernel(float* __restrict__ out, const int8_t* __restrict__ q,
                  const float* __restrict__ scale, int64_t N, int64_t K) {
    if (kVec) {
        const int lane = threadIdx.x & 31;
        const int warp = threadIdx.x >> 5;
        const int64_t words = K >> 2;  // code words per row
        const int64_t chunks = (K + 511) >> 9;
        // This warp's (row, chunk) items in order, the next item's codes
        // requested before the current one is expanded and stored.
        auto load = [&](int64_t r, int64_t cc, uint32_t (&w)[4]) {
            const uint32_t* qr = reinterpret_cast<const uint32_t*>(q + r * K);
            #pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t i = cc * 128 + j * 32 + lane;
                w[j] = i < words ? __ldg(qr + i) : 0u;
            }
        };
        int64_t row = blockIdx.x;
        int64_t c = warp;
        uint32_t wn[4] = {0u, 0u, 0u, 0u};
        if (c < chunks && row < N) load(row, c, wn);
        while (c < chunks && row < N) {
            int64_t row2 = row, c2 = c + kDeqWarps;
            if (c2 >= chunks) {
                c2 = warp;
                row2 += gridDim.x;
            }
            const uint32_t w[4] = {wn[0], wn[1], wn[2], wn[3]};
            if (row2 < N) load(row2, c2, wn);
            const float sc = __ldg(scale + row);
            float4* orow = reinterpret_cast<float4*>(out + row * K);
            #pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t i = c * 128 + j * 32 + lane;
                if (i < words) orow[i] = expand4(w[j], sc);
            }
            row = row2;
            c = c2;
        }
    } else {
        const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
        const int64_t total = N * K;
        for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
            out[t] = static_cast<float>(q[t]) * __ldg(scale + t / K);
        }
    }
}

// The bf16 form: the same f32 product, rounded once to bf16 (nearest even,
// cvt.rn.bf16x2.f32). kVec: lane l reads code-word pairs l and 32 + l of a
// 512-code chunk (two 256-byte loads per warp) and store j writes bf16
// outputs [256 j, 256 j + 256) of the chunk (512 contiguous bytes).
template <bool kVec>
__global__ void __launch_bounds__(kDeqThreads)
dequantize_bf16_kernel(uint16_t* __restrict__ out, const int8_t* __restrict__ q,
                       const float* __restrict__ scale, int64_t N, int64_t K) {
    if (kVec) {
        const int lane = threadIdx.x & 31;
        const int warp = threadIdx.x >> 5;
        const int64_t pairs = K >> 3;  // 8-code pairs of words per row
        const int64_t chunks = (K + 511) >> 9;
        // This warp's (row, chunk) items in order; the codes of the next item
        // are requested before the current one is expanded and stored, so two
        // items' loads are in flight per warp.
        auto load = [&](int64_t r, int64_t cc, uint2 (&w)[2]) {
            const uint2* qr = reinterpret_cast<const uint2*>(q + r * K);
            #pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int64_t i = cc * 64 + j * 32 + lane;
                w[j] = i < pairs ? __ldg(qr + i) : make_uint2(0u, 0u);
            }
        };
        int64_t row = blockIdx.x;
        int64_t c = warp;
        uint2 wn[2] = {make_uint2(0u, 0u), make_uint2(0u, 0u)};
        if (c < chunks && row < N) load(row, c, wn);
        while (c < chunks && row < N) {
            int64_t row2 = row, c2 = c + kDeqWarps;
            if (c2 >= chunks) {
                c2 = warp;
                row2 += gridDim.x;
            }
            const uint2 w[2] = {wn[0], wn[1]};
            if (row2 < N) load(row2, c2, wn);
            const float sc = __ldg(scale + row);
            uint4* orow = reinterpret_cast<uint4*>(out + row * K);
            {
                #pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int64_t i = c * 64 + j * 32 + lane;
                    if (i < pairs) {
                        const float4 a = expand4(w[j].x, sc);
                        const float4 b = expand4(w[j].y, sc);
                        const __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y);  // first code in the low half
                        const __nv_bfloat162 p1 = __floats2bfloat162_rn(a.z, a.w);
                        const __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y);
                        const __nv_bfloat162 p3 = __floats2bfloat162_rn(b.z, b.w);
                        orow[i] = make_uint4(*reinterpret_cast<const uint32_t*>(&p0),
                                             *reinterpret_cast<const uint32_t*>(&p1),
                                             *reinterpret_cast<const uint32_t*>(&p2),
                                             *reinterpret_cast<const uint32_t*>(&p3));
                    }
                }
            }
            row = row2;
            c = c2;
        }
    } else {
        const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
        const int64_t total = N * K;
        for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
            const __nv_bfloat16 v = __float2bfloat16_rn(static_cast<float>(q[t]) * __ldg(scale + t / K));
            out[t] = *reinterpret_cast<const uint16_t*>(&v);
        }
    }
}

// Blocks for the row-walking expand kernels: one row per block up to eight
// resident blocks per SM.
int deq_rows_grid(int64_t N) {
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
    return static_cast<int>(N < cap ? N : cap);
}

int grid_for(int64_t work_items, int threads) {
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    int64_t g = ceil_div(work_items, threads);
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

}  // namespace
}  // namespace pcb

extern "C" popcornStatus_t popcornQuantize_f32i8(int8_t* out, float* scale, const float* input,
                                                 int64_t N, int64_t K, cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || scale == nullptr || input == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (N <= 0 || K <= 0) return POPCORN_SUCCESS;

    const bool vec = (K % 16 == 0) && aligned16(input) && aligned16(out);
    if (vec && K >= 1024 && K <= 16 * kRowThreads * 4) {
        // Block per row with the row in registers.
        int64_t blocks = N;
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
        if (blocks > cap) blocks = cap;
        const int64_t slices = ceil_div(K / 16, kRowThreads);
        const unsigned g = static_cast<unsigned>(blocks);
        if (slices == 1) quantize_row_block_kernel<1><<<g, kRowThreads, 0, stream>>>(out, scale, input, N, K);
        else if (slices == 2) quantize_row_block_kernel<2><<<g, kRowThreads, 0, stream>>>(out, scale, input, N, K);
        else if (slices == 3) quantize_row_block_kernel<3><<<g, kRowThreads, 0, stream>>>(out, scale, input, N, K);
        else quantize_row_block_kernel<4><<<g, kRowThreads, 0, stream>>>(out, scale, input, N, K);
        return check_launch();
    }
    // One warp per row; at most 16 resident blocks per SM worth of warps, the
    // grid-stride loop covers the rest.
    int64_t blocks = ceil_div(N, kWarpsPerBlock);
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    if (vec) {
        quantize_rows_kernel<true><<<static_cast<int>(blocks), kQuantThreads, 0, stream>>>(out, scale, input, N, K);
    } else {
        quantize_rows_kernel<false><<<static_cast<int>(blocks), kQuantThreads, 0, stream>>>(out, scale, input, N, K);
    }
    return check_launch();
}

extern "C" popcornStatus_t popcornDequantize_i8f32(float* out, const int8_t* qweight, const float* scale,
                                                   int64_t N, int64_t K, cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || qweight == nullptr || scale == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (N <= 0 || K <= 0) return POPCORN_SUCCESS;

    const bool vec = (K % 16 == 0) && aligned16(qweight) && aligned16(out);
    if (vec) {
        dequantize_kernel<true><<<deq_rows_grid(N), kDeqThreads, 0, stream>>>(out, qweight, scale, N, K);
    } else {
        dequantize_kernel<false><<<grid_for(N * K, 256), 256, 0, stream>>>(out, qweight, scale, N, K);
    }
    return check_launch();
}

extern "C" popcornStatus_t popcornDequantize_i8bf16(uint16_t* out, const int8_t* qweight, const float* scale,
                                                    int64_t N, int64_t K, cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || qweight == nullptr || scale == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (N <= 0 || K <= 0) return POPCORN_SUCCESS;

    const bool vec = (K % 16 == 0) && aligned16(qweight) && aligned16(out);
    if (vec) {
        dequantize_bf16_kernel<true><<<deq_rows_grid(N), kDeqThreads, 0, stream>>>(out, qweight, scale, N, K);
    } else {
        dequantize_bf16_kernel<false><<<grid_for(N * K, 256), 256, 0, stream>>>(out, qweight, scale, N, K);
    }
    return check_launch();
}
