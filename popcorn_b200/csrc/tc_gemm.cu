// tcgen05 tensor-core dequant-matmul path: out[m, n] = scale[n] * sum_k x[m, k] * q[n, k].
//
// Per-channel int8 weights with 4 < M <= 128 take the int8 path at the end
// of the device code (x_to_i8_*_kernel + tc_i8_kernel): activations as two
// signed 8-bit digits of a 16-bit fixed-point row, tcgen05.mma.kind::i8 on
// the raw weight codes, exact int32 sums. Everything else (M > 128, and the
// per-group int8 / int4 formats at any M) takes the f16 path described here.
//
// Same arithmetic contract as popcorn's dequantizeMatmulKernel_i8f32
// (src/quantize.cu:18-84) except that activations enter the tensor cores as
// f16: int8 codes are exact in f16, each activation row m is first scaled by
// a power of two 2^e_m (exact) so its largest |x| lands in [2^14, 2^15), then
// rounded to f16 (relative error <= 2^-11 per element); products are exact
// in the tensor core and accumulate in f32 in tensor memory; the epilogue
// multiplies by 2^-e_m (exact) and by scale[n] (one rounding).
//
// Two launches per call:
//  1. x_to_f16_kernel: x f32 [M, K] -> x16 f16 [M, K] + rowscale [M] = 2^-e_m
//     in stream-ordered scratch from a private memory pool.
//  2. tc_gemm_kernel<BM, FMT>: one CTA per 128 (weight rows) x BM (activation
//     rows) output tile (cluster split-K when the tiles fill less than half
//     the GPU), or tc_gemm_pair_kernel<RX, FMT>: a CTA pair per 256 x 2 RX
//     tile with tcgen05.mma.cta_group::2 (tc_gemm_pair_persist_kernel when
//     there are more tiles than resident pairs). Swap-AB, so the weight tile
//     is the MMA "A" operand; per 128-deep k-block stage:
//       warp 0      TMA producer: x16 tile (128B swizzle) and the weight-code
//                   tile [128 rows x 128 int8 (128B swizzle) or 64 bytes of
//                   packed int4 (64B swizzle)];
//       warp 1      tcgen05.mma issuer (A from tensor memory, B = x16 tile
//                   from shared memory, D = f32 in tensor memory);
//       warps 2-9   converters in two groups of four: each thread owns one
//                   weight row, group g converts codes [64 g, 64 g + 64) of
//                   every k-block to f16 and writes them to tensor memory
//                   (tcgen05.st) as the A operand;
//       warps 10-13 epilogue: tcgen05.ld of the accumulator, one row per
//                   lane, so each column m is a coalesced 128-byte store.
// Weight formats (FMT): per-channel int8 codes are exact in f16 and the
// epilogue multiplies by scale[n]; per-group int8 codes are written as
// code * scale[n, g] * 2^e_n and int4 codes as (code - zero[n, g]) *
// scale[n, g] * 2^e_n (one rounding to f16), 2^e_n a power of two per row
// that keeps the row inside f16's range, undone by the epilogue.
// Keeping the widened weights in tensor memory means shared memory carries
// only the weight codes and the f16 activations, not a second f16 copy.
//
// Roofline: tensor (dense f16) for large M; algorithmic work 2*M*N*K.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace pcb {

// Error bits set by bounded waits that timed out (read by popcornB200DeviceErrors).
__device__ unsigned int g_tc_error = 0;

namespace {

using namespace sm100;

constexpr int kTileN = 128;    // weight rows per CTA (MMA M)
constexpr int kThreads = 448;  // 14 warps
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpConv0 = 2;  // two groups of four converter warps: 2-5, 6-9
constexpr int kConvGroups = 2;  // group g converts codes [64 g, 64 g + 64) of every k-block
constexpr int kWarpEpi0 = 10;

// Per activation-tile height BM: k-blocks of 128 (one [128 x 128] int8 weight
// box, 128-byte swizzle, and a [BM x 128] f16 activation box per stage) in a
// ring of kStages stages; ring slot s is also tensor-memory A buffer s, so
// one barrier per slot says "its tiles and its A buffer are free again".
// Tensor memory: accumulator (BM columns) + kStages A buffers of 64 columns.
template <int BM, int FMT = kFmtChannel>
struct Cfg {
    static constexpr int kBK = 128;
    static constexpr int kSub = kBK / 64;           // 64-wide f16 swizzle atoms per stage
    static constexpr int kACols = kBK / 2;          // tensor-memory columns per A buffer
    static constexpr int kStages = BM >= 128 ? 4 : (BM >= 64 ? 6 : 7);
    static constexpr int kXBytes = BM * kBK * 2;   // f16 activation tile per stage
    static constexpr int kWRow = FMT == kFmtGroup4 ? kBK / 2 : kBK;  // weight bytes per row and stage
    static constexpr int kWBytes = kTileN * kWRow;  // weight tile per stage
    static constexpr int kTmemCols = 512;
    static constexpr int kNumBars = 3 * kStages + 2;
    // ring, barriers, tensor-memory slot (16 B), per-row output scales, and
    // the epilogue's [32 x 32] f32 staging tile per epilogue warp (tiles of
    // 64 or more activation rows; a single 32-column chunk stores directly)
    static constexpr bool kStaged = BM >= 64;
    static constexpr int kStageBytes = kStaged ? 4 * 32 * 32 * 4 : 0;
    static constexpr int kSmem = 1024 + kStages * (kXBytes + kWBytes) + kNumBars * 8 + 16 + kTileN * 4 + 16 + kStageBytes;
    // Split-K reduction buffer: [128 weight rows][BM + 4] f32 in the idle ring.
    static constexpr int kRedStride = BM + 4;
    static_assert(kXBytes % 1024 == 0, "x16 stages must stay 1024-byte aligned");
    // Two partial accumulators: k-steps alternate between them, so
    // consecutive MMAs of a k-block do not wait on each other's results.
    static constexpr int kAcc = 2;
    static_assert(kAcc * BM + kStages * kACols <= kTmemCols, "tensor memory holds 512 columns");
    static_assert(kSmem <= 227 * 1024, "shared memory per block");
    static_assert(kTileN * kRedStride * 4 <= kStages * (kXBytes + kWBytes), "reduction buffer fits the ring");
};

__device__ __forceinline__ float absmax_step(float m, float v) {
    float a = fabsf(v);
    return (a > m) ? a : m;
}

// Optional RMSNorm of the activation rows inside the prologue, with
// popcorn's arithmetic (src/reduction.cu:290-321): rms = sqrtf(sum(x^2) / K +
// eps), inv = 1 / rms, x' = (x * inv) * norm_w[k] (norm_w may be null). Only
// the order of the sum of squares differs from popcorn's sequential loop.
struct RowNorm {
    const float* w;  // [K] or null
    float eps;
    int on;
};

__device__ __forceinline__ float row_inv_rms(float sum_sq, int64_t K, float eps) {
    return 1.0f / sqrtf(sum_sq / static_cast<float>(K) + eps);
}

// x f32 [M, K] -> x16 f16 [M, K] with per-row power-of-two scaling; one warp per row.
__global__ void __launch_bounds__(256)
x_to_f16_kernel(__half* __restrict__ x16, float* __restrict__ rowscale, const float* __restrict__ x,
                int64_t M, int64_t K, int vec, RowNorm nrm) {
    // The GEMM that follows is launched as a programmatic dependent: let it
    // start its set-up now; it waits for this grid before reading x16.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
         row += nwarps) {
        const float* r = x + row * K;
        __half* o = x16 + row * K;
        float inv = 1.0f;
        if (nrm.on) {
            float ss = 0.0f;
            for (int64_t k = lane; k < K; k += 32) {
                const float v = __ldg(r + k);
                ss = fmaf(v, v, ss);
            }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            inv = row_inv_rms(ss, K, nrm.eps);
        }
        // The value entering the GEMM: x, or its normalised form.
        auto val = [&](int64_t k, float v) {
            if (!nrm.on) return v;
            v = v * inv;
            return nrm.w != nullptr ? v * __ldg(nrm.w + k) : v;
        };
        float m = 0.0f;
        if (vec && !nrm.on) {
            const float4* r4 = reinterpret_cast<const float4*>(r);
            #pragma unroll 4
            for (int64_t i = lane; i < (K >> 2); i += 32) {
                const float4 v = __ldg(r4 + i);
                m = absmax_step(absmax_step(absmax_step(absmax_step(m, v.x), v.y), v.z), v.w);
            }
        } else {
            for (int64_t k = lane; k < K; k += 32) m = absmax_step(m, val(k, __ldg(r + k)));
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, m, off);
            m = (other > m) ? other : m;
        }
        int e = 0;
        if (m > 0.0f && m <= 3.402823466e38f) {
            int p;
            frexpf(m, &p);  // m in [2^(p-1), 2^p)
            e = 15 - p;     // m * 2^e in [2^14, 2^15)
            e = e < -126 ? -126 : (e > 126 ? 126 : e);
        }
        const float up = __int_as_float((e + 127) << 23);
        if (lane == 0) rowscale[row] = __int_as_float((127 - e) << 23);
        if (vec && !nrm.on) {
            const float4* r4 = reinterpret_cast<const float4*>(r);
            uint4* o8 = reinterpret_cast<uint4*>(o);
            for (int64_t c = lane; c < (K >> 3); c += 32) {
                const float4 a = __ldg(r4 + 2 * c);
                const float4 b = __ldg(r4 + 2 * c + 1);
                __half2 h0 = __floats2half2_rn(a.x * up, a.y * up);
                __half2 h1 = __floats2half2_rn(a.z * up, a.w * up);
                __half2 h2 = __floats2half2_rn(b.x * up, b.y * up);
                __half2 h3 = __floats2half2_rn(b.z * up, b.w * up);
                uint4 packed;
                packed.x = *reinterpret_cast<uint32_t*>(&h0);
                packed.y = *reinterpret_cast<uint32_t*>(&h1);
                packed.z = *reinterpret_cast<uint32_t*>(&h2);
                packed.w = *reinterpret_cast<uint32_t*>(&h3);
                o8[c] = packed;
            }
        } else {
            for (int64_t k = lane; k < K; k += 32) o[k] = __float2half_rn(val(k, __ldg(r + k)) * up);
        }
    }
}

// Same conversion, one block per row with the row held in registers (U
// 16-float slices per thread, K <= 16 * 256 * U): x is read from HBM once and
// every thread has all of its loads in flight at once. Needs K % 16 == 0 and
// a 16-byte aligned x (and norm weights).
constexpr int kRowThreads = 256;

template <int U>
__global__ void __launch_bounds__(kRowThreads)
x_to_f16_row_kernel(__half* __restrict__ x16, float* __restrict__ rowscale, const float* __restrict__ x, int64_t M,
                    int64_t K, RowNorm nrm) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // see x_to_f16_kernel
    __shared__ float red[2][kRowThreads / 32];
    __shared__ float ssq[2][kRowThreads / 32];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int64_t units = K >> 4;
    int parity = 0;
    for (int64_t row = blockIdx.x; row < M; row += gridDim.x, parity ^= 1) {
        const float4* r4 = reinterpret_cast<const float4*>(x + row * K);
        float4 v[U][4];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                v[u][c] = (unit < units) ? __ldg(r4 + unit * 4 + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
        if (nrm.on) {
            float ss = 0.0f;
            #pragma unroll
            for (int u = 0; u < U; ++u)
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    ss = fmaf(v[u][c].x, v[u][c].x, ss);
                    ss = fmaf(v[u][c].y, v[u][c].y, ss);
                    ss = fmaf(v[u][c].z, v[u][c].z, ss);
                    ss = fmaf(v[u][c].w, v[u][c].w, ss);
                }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            if (lane == 0) ssq[parity][warp] = ss;
            __syncthreads();
            float total = 0.0f;
            #pragma unroll
            for (int w = 0; w < kRowThreads / 32; ++w) total += ssq[parity][w];
            const float inv = row_inv_rms(total, K, nrm.eps);
            #pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float4 a = v[u][c];
                    a.x *= inv;
                    a.y *= inv;
                    a.z *= inv;
                    a.w *= inv;
                    if (nrm.w != nullptr && unit < units) {
                        const float4 g = __ldg(reinterpret_cast<const float4*>(nrm.w) + unit * 4 + c);
                        a.x *= g.x;
                        a.y *= g.y;
                        a.z *= g.z;
                        a.w *= g.w;
                    }
                    v[u][c] = a;
                }
            }
        }
        float m = 0.0f;
        #pragma unroll
        for (int u = 0; u < U; ++u)
            #pragma unroll
            for (int c = 0; c < 4; ++c)
                m = absmax_step(absmax_step(absmax_step(absmax_step(m, v[u][c].x), v[u][c].y), v[u][c].z), v[u][c].w);
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
        int e = 0;
        if (m > 0.0f && m <= 3.402823466e38f) {
            int p;
            frexpf(m, &p);
            e = 15 - p;
            e = e < -126 ? -126 : (e > 126 ? 126 : e);
        }
        const float up = __int_as_float((e + 127) << 23);
        if (tid == 0) rowscale[row] = __int_as_float((127 - e) << 23);
        uint4* o8 = reinterpret_cast<uint4*>(x16 + row * K);
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
            if (unit < units) {
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 a = v[u][2 * h];
                    const float4 b = v[u][2 * h + 1];
                    __half2 h0 = __floats2half2_rn(a.x * up, a.y * up);
                    __half2 h1 = __floats2half2_rn(a.z * up, a.w * up);
                    __half2 h2 = __floats2half2_rn(b.x * up, b.y * up);
                    __half2 h3 = __floats2half2_rn(b.z * up, b.w * up);
                    uint4 packed;
                    packed.x = *reinterpret_cast<uint32_t*>(&h0);
                    packed.y = *reinterpret_cast<uint32_t*>(&h1);
                    packed.z = *reinterpret_cast<uint32_t*>(&h2);
                    packed.w = *reinterpret_cast<uint32_t*>(&h3);
                    o8[unit * 2 + h] = packed;
                }
            }
        }
    }
}

// Launch the x -> f16 prologue: block-per-row kernel where it applies.
popcornStatus_t launch_x_to_f16(__half* x16, float* rowscale, const float* x, int64_t M, int64_t K,
                                cudaStream_t stream, RowNorm nrm = RowNorm{nullptr, 0.0f, 0}) {
    const bool vec = aligned16(x) && (nrm.w == nullptr || aligned16(nrm.w));
    const int64_t slices = ceil_div(K / 16, kRowThreads);
    if (vec && K % 16 == 0 && K >= 1024 && slices <= 4) {
        int64_t blocks = M;
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
        if (blocks > cap) blocks = cap;
        const unsigned g = static_cast<unsigned>(blocks);
        if (slices == 1) x_to_f16_row_kernel<1><<<g, kRowThreads, 0, stream>>>(x16, rowscale, x, M, K, nrm);
        else if (slices == 2) x_to_f16_row_kernel<2><<<g, kRowThreads, 0, stream>>>(x16, rowscale, x, M, K, nrm);
        else x_to_f16_row_kernel<4><<<g, kRowThreads, 0, stream>>>(x16, rowscale, x, M, K, nrm);
        return check_launch();
    }
    int64_t blocks = ceil_div(M, 8);
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    x_to_f16_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x16, rowscale, x, M, K,
                                                                      aligned16(x) ? 1 : 0, nrm);
    return check_launch();
}

// ------------------------------------------- int8 digit prologue (M <= 128)
// For the int8 tensor path, activation row m becomes the 16-bit fixed-point
// row X[m, k] = rint(x[m, k] * 32512 / a_m), a_m = max_k |x[m, k]|, so
// |X| <= 32512 and x[m, k] = X[m, k] * f_m up to half a step, f_m = a_m / 32512.
// X is stored as two signed 8-bit digits X = 256 hi + lo, hi = (X + 128) >> 8
// in [-127, 127] and lo in [-128, 127]: hi digits of all rows in plane 0, lo
// digits in plane 1 of xd [2, M, K]. f_m is stored as a mantissa in [1, 2)
// (rowfactor[m]) and an exact power of two (rowpow[m]); the epilogue forms
// ((acc * mantissa) * scale[n]) * power, which overflows or underflows only
// where the result itself does. Rows with a NaN
// get f_m = NaN (every output of the row is NaN, as in popcorn's sum). Rows
// with infinities get f_m = inf and X = +-1 at the infinite entries, 0
// elsewhere: with one infinity each output is +-inf with the sign of x * w,
// or NaN where that code is 0 -- popcorn's result exactly; with several,
// every output is non-finite as popcorn's, but +-inf where popcorn's mixed
// signs give NaN. An all-zero row gets f_m = 0. Rows with a_m < 2^-100 are
// scaled by 2^100 (exact) before the division so 32512 / a stays finite.
struct DigitRow {
    float pre;   // exact power-of-two pre-scale
    float mult;  // 32512 / (a_m * pre)
    int mode;    // 0 finite, 1 infinities (no NaN), 2 NaN
    float fm;    // f_m = fm * pw: mantissa in [1, 2) (or NaN, inf, 0 for special rows)
    float pw;    //   and an exact power of two (0 below the smallest denormal)
};

__device__ __forceinline__ DigitRow digit_row(float a, bool has_nan) {
    DigitRow d{1.0f, 0.0f, 0, 0.0f, 1.0f};
    if (has_nan) {
        d.mode = 2;
        d.fm = __int_as_float(0x7fc00000);
    } else if (a > 3.402823466e38f) {
        d.mode = 1;
        d.fm = __int_as_float(0x7f800000);
    } else if (a > 0.0f) {
        const bool tiny = a < 0x1p-100f;
        d.pre = tiny ? 0x1p100f : 1.0f;
        const float ap = a * d.pre;
        d.mult = 32512.0f / ap;
        // ap / 32512 lies in [2^-64, 2^114): a normal float, split exactly.
        const uint32_t b = __float_as_uint(ap / 32512.0f);
        d.fm = __uint_as_float((b & 0x807FFFFFu) | (127u << 23));
        const int e = static_cast<int>((b >> 23) & 0xFFu) - 127 - (tiny ? 100 : 0);
        d.pw = e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23)
                         : (e >= -149 ? __uint_as_float(1u << (e + 149)) : 0.0f);
    }
    return d;
}

__device__ __forceinline__ int digit_value(float v, const DigitRow& d) {
    if (d.mode == 1) return (v == __int_as_float(0x7f800000)) ? 1 : ((v == __int_as_float(0xff800000)) ? -1 : 0);
    if (d.mode == 2) return 0;
    int X = __float2int_rn((v * d.pre) * d.mult);
    X = X > 32512 ? 32512 : (X < -32512 ? -32512 : X);
    return X;
}

// Four values -> their hi and lo digit bytes, k order.
__device__ __forceinline__ void digits4(float a, float b, float c, float e, const DigitRow& d, uint32_t& hi,
                                        uint32_t& lo) {
    const int X[4] = {digit_value(a, d), digit_value(b, d), digit_value(c, d), digit_value(e, d)};
    hi = 0;
    lo = 0;
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int h = (X[i] + 128) >> 8;
        const int l = X[i] - h * 256;
        hi |= (static_cast<uint32_t>(h) & 0xFFu) << (8 * i);
        lo |= (static_cast<uint32_t>(l) & 0xFFu) << (8 * i);
    }
}

// One block per row, the row held in registers (U 16-float slices per
// thread, K <= 16 * 256 * U); needs K % 16 == 0 and 16-byte aligned x (and
// norm weights).
template <int U>
__global__ void __launch_bounds__(kRowThreads)
x_to_i8_row_kernel(int8_t* __restrict__ xd, float* __restrict__ rowfactor, float* __restrict__ rowpow,
                   const float* __restrict__ x, int64_t M, int64_t K, RowNorm nrm) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the GEMM waits for this grid
    __shared__ float red[2][kRowThreads / 32];
    __shared__ float ssq[2][kRowThreads / 32];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int64_t units = K >> 4;
    int parity = 0;
    for (int64_t row = blockIdx.x; row < M; row += gridDim.x, parity ^= 1) {
        const float4* r4 = reinterpret_cast<const float4*>(x + row * K);
        float4 v[U][4];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                v[u][c] = (unit < units) ? __ldg(r4 + unit * 4 + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
        if (nrm.on) {
            float ss = 0.0f;
            #pragma unroll
            for (int u = 0; u < U; ++u)
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    ss = fmaf(v[u][c].x, v[u][c].x, ss);
                    ss = fmaf(v[u][c].y, v[u][c].y, ss);
                    ss = fmaf(v[u][c].z, v[u][c].z, ss);
                    ss = fmaf(v[u][c].w, v[u][c].w, ss);
                }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            if (lane == 0) ssq[parity][warp] = ss;
            __syncthreads();
            float total = 0.0f;
            #pragma unroll
            for (int w = 0; w < kRowThreads / 32; ++w) total += ssq[parity][w];
            const float inv = row_inv_rms(total, K, nrm.eps);
            #pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float4 a = v[u][c];
                    a.x *= inv;
                    a.y *= inv;
                    a.z *= inv;
                    a.w *= inv;
                    if (nrm.w != nullptr && unit < units) {
                        const float4 g = __ldg(reinterpret_cast<const float4*>(nrm.w) + unit * 4 + c);
                        a.x *= g.x;
                        a.y *= g.y;
                        a.z *= g.z;
                        a.w *= g.w;
                    }
                    v[u][c] = a;
                }
            }
        }
        float m = 0.0f;
        int nan_seen = 0;
        #pragma unroll
        for (int u = 0; u < U; ++u)
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 a = v[u][c];
                m = absmax_step(absmax_step(absmax_step(absmax_step(m, a.x), a.y), a.z), a.w);
                nan_seen |= (a.x != a.x) | (a.y != a.y) | (a.z != a.z) | (a.w != a.w);
            }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, m, off);
            m = (other > m) ? other : m;
        }
        if (lane == 0) red[parity][warp] = m;
        const bool has_nan = __syncthreads_or(nan_seen) != 0;
        m = red[parity][0];
        #pragma unroll
        for (int w = 1; w < kRowThreads / 32; ++w) {
            const float other = red[parity][w];
            m = (other > m) ? other : m;
        }
        const DigitRow d = digit_row(m, has_nan);
        if (tid == 0) {
            rowfactor[row] = d.fm;
            rowpow[row] = d.pw;
        }
        uint4* hi8 = reinterpret_cast<uint4*>(xd + row * K);
        uint4* lo8 = reinterpret_cast<uint4*>(xd + (M + row) * K);
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kRowThreads;
            if (unit < units) {
                uint32_t h[4], l[4];
                #pragma unroll
                for (int c = 0; c < 4; ++c) digits4(v[u][c].x, v[u][c].y, v[u][c].z, v[u][c].w, d, h[c], l[c]);
                hi8[unit] = make_uint4(h[0], h[1], h[2], h[3]);
                lo8[unit] = make_uint4(l[0], l[1], l[2], l[3]);
            }
        }
    }
}

// Any K (multiple of 16) and alignment of x: one warp per row, two passes
// over the row (the second from L2).
__global__ void __launch_bounds__(256)
x_to_i8_kernel(int8_t* __restrict__ xd, float* __restrict__ rowfactor, float* __restrict__ rowpow,
               const float* __restrict__ x, int64_t M, int64_t K, RowNorm nrm) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
         row += nwarps) {
        const float* r = x + row * K;
        float inv = 1.0f;
        if (nrm.on) {
            float ss = 0.0f;
            for (int64_t k = lane; k < K; k += 32) {
                const float v = __ldg(r + k);
                ss = fmaf(v, v, ss);
            }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            inv = row_inv_rms(ss, K, nrm.eps);
        }
        auto val = [&](int64_t k) {
            float v = __ldg(r + k);
            if (!nrm.on) return v;
            v = v * inv;
            return nrm.w != nullptr ? v * __ldg(nrm.w + k) : v;
        };
        float m = 0.0f;
        int nan_seen = 0;
        for (int64_t k = lane; k < K; k += 32) {
            const float v = val(k);
            m = absmax_step(m, v);
            nan_seen |= (v != v);
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, m, off);
            m = (other > m) ? other : m;
        }
        const bool has_nan = __any_sync(0xffffffffu, nan_seen) != 0;
        const DigitRow d = digit_row(m, has_nan);
        if (lane == 0) {
            rowfactor[row] = d.fm;
            rowpow[row] = d.pw;
        }
        uint32_t* hi4 = reinterpret_cast<uint32_t*>(xd + row * K);
        uint32_t* lo4 = reinterpret_cast<uint32_t*>(xd + (M + row) * K);
        for (int64_t c = lane; c < (K >> 2); c += 32) {
            uint32_t h, l;
            digits4(val(4 * c), val(4 * c + 1), val(4 * c + 2), val(4 * c + 3), d, h, l);
            hi4[c] = h;
            lo4[c] = l;
        }
    }
}

popcornStatus_t launch_x_to_i8(int8_t* xd, float* rowfactor, float* rowpow, const float* x, int64_t M, int64_t K,
                               cudaStream_t stream, RowNorm nrm) {
    const bool vec = aligned16(x) && (nrm.w == nullptr || aligned16(nrm.w));
    const int64_t slices = ceil_div(K / 16, kRowThreads);
    if (vec && K % 16 == 0 && slices <= 4) {
        const unsigned g = static_cast<unsigned>(M);  // M <= 128 on this path
        if (slices == 1) x_to_i8_row_kernel<1><<<g, kRowThreads, 0, stream>>>(xd, rowfactor, rowpow, x, M, K, nrm);
        else if (slices == 2) x_to_i8_row_kernel<2><<<g, kRowThreads, 0, stream>>>(xd, rowfactor, rowpow, x, M, K, nrm);
        else x_to_i8_row_kernel<4><<<g, kRowThreads, 0, stream>>>(xd, rowfactor, rowpow, x, M, K, nrm);
        return check_launch();
    }
    x_to_i8_kernel<<<static_cast<unsigned>(ceil_div(M, 8)), 256, 0, stream>>>(xd, rowfactor, rowpow, x, M, K,
                                                                         nrm);
    return check_launch();
}

// Four int8 codes (one word) -> two f16x2 words, exact:
// (code ^ 0x80) in the low byte of f16 0x6400 gives 1024 + 128 + code;
// subtracting 1152 leaves the code.
__device__ __forceinline__ void widen4_f16(uint32_t word, uint32_t& lo, uint32_t& hi) {
    const uint32_t b = word ^ 0x80808080u;
    const uint32_t plo = __byte_perm(b, 0x64646464u, 0x5140);
    const uint32_t phi = __byte_perm(b, 0x64646464u, 0x7362);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 l = __hsub2(*reinterpret_cast<const __half2*>(&plo), bias);
    __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&phi), bias);
    lo = *reinterpret_cast<uint32_t*>(&l);
    hi = *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t f16x2_bits(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Epilogue store: the value itself (epi = 0), or silu(g) * value (epi = 1)
// where g is what the previous GEMM of the same call wrote there -- the gate
// projection, so the up projection's epilogue finishes popcorn's
// popcornSilu_f32 (g / (1 + expf(-g)), src/unary.cu:76-81) and popcornMul_f32.
__device__ __forceinline__ void store_out(float* p, float v, int epi) {
    if (epi) {
        const float g = *p;
        v = (g / (1.0f + expf(-g))) * v;
    }
    *p = v;
}

// A 32-column chunk of a tile's accumulator: the sum (fixed order) of its
// kAcc partial accumulators, `stride` columns apart.
template <int kAcc>
__device__ __forceinline__ void acc_ld32(uint32_t taddr, int stride, uint32_t (&v)[32]) {
    tmem_ld_32x32b_x32(taddr, v);
    if constexpr (kAcc == 2) {
        uint32_t w[32];
        tmem_ld_32x32b_x32(taddr + stride, w);
        tmem_wait_ld();
        #pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
    } else {
        tmem_wait_ld();
    }
}

// Vector form of store_chunk (epi = 0) for a warp whose 32 weight rows
// n0w .. n0w + 31 all lie below N, with 16-byte aligned output rows: the
// chunk goes through the warp's [32 m][32 n] f32 staging tile in shared
// memory (lane l writes its row as column l, conflict-free) and back out as
// float4 runs along n: eight 16-byte stores per lane instead of 32 scalar
// ones.
__device__ __forceinline__ void store_chunk_v(float* __restrict__ out, const float* __restrict__ rowscale, int m0,
                                              int cnt, int n0w, int N, float sc, const uint32_t* v, float* stage,
                                              int lane) {
    float rs[32];
    if (cnt >= 32) {
        const float4* r4 = reinterpret_cast<const float4*>(rowscale + m0);
        #pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 r = __ldg(r4 + q);
            rs[4 * q] = r.x;
            rs[4 * q + 1] = r.y;
            rs[4 * q + 2] = r.z;
            rs[4 * q + 3] = r.w;
        }
    } else {
        #pragma unroll
        for (int j = 0; j < 32; ++j) rs[j] = (j < cnt) ? __ldg(rowscale + m0 + j) : 0.0f;
    }
    #pragma unroll
    for (int j = 0; j < 32; ++j) stage[j * 32 + lane] = (__uint_as_float(v[j]) * rs[j]) * sc;
    __syncwarp();
    const int q = lane & 7;
    const int mr = lane >> 3;
    #pragma unroll
    for (int it = 0; it < 8; ++it) {
        const int ml = it * 4 + mr;
        if (ml < cnt) {
            const float4 val = *reinterpret_cast<const float4*>(stage + ml * 32 + 4 * q);
            *reinterpret_cast<float4*>(out + static_cast<int64_t>(m0 + ml) * N + n0w + 4 * q) = val;
        }
    }
    __syncwarp();  // the tile is rewritten by the next chunk
}

// Epilogue of one 32-column accumulator chunk of weight row n:
// out[m0 + j, n] = (v[j] * rowscale[m0 + j]) * sc for j < cnt. The chunk's
// row scales are read first (broadcast float4 loads: every lane reads the
// same addresses; rowscale + m0 is 16-byte aligned since m0 % 32 == 0) and
// the epilogue mode is tested once, so the stores issue back to back
// instead of each waiting for its own load.
__device__ __forceinline__ void store_chunk(float* __restrict__ out, const float* __restrict__ rowscale, int m0,
                                            int cnt, int n, int N, float sc, const uint32_t* v, int epi) {
    float rs[32];
    if (cnt >= 32) {
        const float4* r4 = reinterpret_cast<const float4*>(rowscale + m0);
        #pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 r = __ldg(r4 + q);
            rs[4 * q] = r.x;
            rs[4 * q + 1] = r.y;
            rs[4 * q + 2] = r.z;
            rs[4 * q + 3] = r.w;
        }
    } else {
        #pragma unroll
        for (int j = 0; j < 32; ++j) rs[j] = (j < cnt) ? __ldg(rowscale + m0 + j) : 0.0f;
    }
    float* base = out + static_cast<int64_t>(m0) * N + n;
    if (epi) {
        #pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < cnt) store_out(base + static_cast<int64_t>(j) * N, (__uint_as_float(v[j]) * rs[j]) * sc, 1);
        }
    } else {
        #pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < cnt) base[static_cast<int64_t>(j) * N] = (__uint_as_float(v[j]) * rs[j]) * sc;
        }
    }
}

// Per-group formats: the converters write w * 2^e_n to tensor memory as f16
// and the epilogue multiplies by 2^-e_n (exact). 2^e_n brings the largest
// weight row n can hold -- 128 |s| for int8 codes, (15 + |z|) |s| for int4 --
// into [2^13, 2^14), far inside f16's range, whatever the scales' magnitude.
template <int FMT>
__device__ __forceinline__ int group_row_exp(const float* __restrict__ scale, const float* __restrict__ zero, int n,
                                             int N, int groups) {
    if (n >= N) return 0;
    const float* sr = scale + static_cast<int64_t>(n) * groups;
    const float* zr = zero + static_cast<int64_t>(n) * groups;
    float m = 0.0f;
    // 32 groups per pass, every load of a pass in flight at once (the scales
    // usually come from HBM: one round trip per pass).
    for (int g0 = 0; g0 < groups; g0 += 32) {
        float a[32], z[32];
        #pragma unroll
        for (int j = 0; j < 32; ++j) {
            a[j] = (g0 + j < groups) ? __ldg(sr + g0 + j) : 0.0f;
            if constexpr (FMT == kFmtGroup4) z[j] = (g0 + j < groups) ? __ldg(zr + g0 + j) : 0.0f;
        }
        #pragma unroll
        for (int j = 0; j < 32; ++j) {
            float b;
            if constexpr (FMT == kFmtGroup4) {
                b = (15.0f + fabsf(z[j])) * fabsf(a[j]);
            } else {
                b = 128.0f * fabsf(a[j]);
            }
            m = b > m ? b : m;  // NaN skipped
        }
    }
    int e = 0;
    if (m > 0.0f && m <= 3.402823466e38f) {
        int p;
        frexpf(m, &p);  // m in [2^(p-1), 2^p)
        e = 14 - p;     // m * 2^e in [2^13, 2^14)
        e = e < -126 ? -126 : (e > 126 ? 126 : e);
    }
    return e;
}

// Group factors of half `h` (64 codes) of a 128-deep k-block of weight row n,
// per 32-code quarter: f[j] = scale[n, g] * 2^e_n and (int4) zf[j] =
// zero[n, g] * f[j] for quarter 2h + j; zero for rows past N and quarters past
// K (whose codes and activations are zero-filled).
template <int FMT>
__device__ __forceinline__ void group_factors(const float* __restrict__ scale, const float* __restrict__ zero, int n,
                                              int N, int K, int gs, int kb, int h, float pw, float (&f)[2],
                                              float (&zf)[2]) {
    const int groups = K / gs;
    #pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int k = kb * 128 + h * 64 + q * 32;
        f[q] = 0.0f;
        zf[q] = 0.0f;
        if (n < N && k < K) {
            const int64_t i = static_cast<int64_t>(n) * groups + k / gs;
            f[q] = __ldg(scale + i) * pw;
            if constexpr (FMT == kFmtGroup4) zf[q] = __ldg(zero + i) * f[q];
        }
    }
}

// Four int8 codes -> two f16x2 words of code * f: the codes widen exactly
// (widen4_f16), then one packed f16 multiply by f rounded to f16 (f16x2 in
// both halves). Relative error <= 2^-11 per weight (f's rounding and the
// product's), normwise ~4e-4 with the f16 activations.
__device__ __forceinline__ void widen4_scaled(uint32_t word, __half2 f2, uint32_t& lo, uint32_t& hi) {
    uint32_t a, b;
    widen4_f16(word, a, b);
    __half2 l = __hmul2(*reinterpret_cast<const __half2*>(&a), f2);
    __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&b), f2);
    lo = *reinterpret_cast<uint32_t*>(&l);
    hi = *reinterpret_cast<uint32_t*>(&h);
}

// Eight int4 codes (one word, low nibble first) -> four f16x2 words of
// code * f - zero * f.
__device__ __forceinline__ void widen8_i4_scaled(uint32_t word, float f, float zf, uint32_t* h) {
    const uint32_t lo = word & 0x0F0F0F0Fu;         // even k
    const uint32_t hi = (word >> 4) & 0x0F0F0F0Fu;  // odd k
    const float2 bias = make_float2(-8388608.0f, -8388608.0f);  // -2^23
    const float2 ff = make_float2(f, f);
    const float2 nz = make_float2(-zf, -zf);
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        float2 c = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440 + j)),
                               __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440 + j)));
        c = __ffma2_rn(__fadd2_rn(c, bias), ff, nz);
        h[j] = f16x2_bits(c.x, c.y);
    }
}

// The codes of half g (codes [64 g, 64 g + 64)) of weight row r of a ring
// stage at `tile`, in k order: 16 words of int8 codes (128B swizzle: chunk ^=
// r & 7) or 8 words of packed int4 codes (64B swizzle: chunk ^= (r >> 1) & 3).
template <int FMT>
__device__ __forceinline__ void load_half(const uint8_t* tile, int r, int g, uint32_t (&w)[16]) {
    if constexpr (FMT == kFmtGroup4) {
        const uint8_t* row = tile + r * 64;
        #pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
            const int c = 2 * g + c2;
            const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ ((r >> 1) & 3)) << 4));
            w[4 * c2 + 0] = v.x;
            w[4 * c2 + 1] = v.y;
            w[4 * c2 + 2] = v.z;
            w[4 * c2 + 3] = v.w;
        }
    } else {
        const uint8_t* row = tile + r * 128;
        #pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
            const int c = g * 4 + c4;
            const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) << 4));
            w[4 * c4 + 0] = v.x;
            w[4 * c4 + 1] = v.y;
            w[4 * c4 + 2] = v.z;
            w[4 * c4 + 3] = v.w;
        }
    }
}

// Those 64 codes -> 32 f16x2 words of the A operand: int8 codes widened
// exactly (per-channel) or scaled per group, int4 codes with zero point and
// scale. f, zf: the factors of the half's two 32-code quarters.
template <int FMT>
__device__ __forceinline__ void widen_half(const uint32_t (&w)[16], const float (&f)[2], const float (&zf)[2],
                                           uint32_t (&h)[32]) {
    if constexpr (FMT == kFmtGroup4) {
        #pragma unroll
        for (int k = 0; k < 8; ++k) widen8_i4_scaled(w[k], f[k / 4], zf[k / 4], h + 4 * k);
    } else if constexpr (FMT == kFmtGroup8) {
        const __half2 f2[2] = {__float2half2_rn(f[0]), __float2half2_rn(f[1])};
        #pragma unroll
        for (int k = 0; k < 16; ++k) widen4_scaled(w[k], f2[k / 8], h[2 * k], h[2 * k + 1]);
    } else {
        #pragma unroll
        for (int k = 0; k < 16; ++k) widen4_f16(w[k], h[2 * k], h[2 * k + 1]);
    }
}

// Half g of a 128-deep k-block of weight row r into A-buffer columns
// [32 g, 32 g + 32) of tensor-memory lane r (`taddr` = the A buffer at this
// warp's lanes).
template <int FMT>
__device__ __forceinline__ void convert_half(const uint8_t* tile, int r, int g, uint32_t taddr, const float (&f)[2],
                                             const float (&zf)[2]) {
    uint32_t w[16];
    load_half<FMT>(tile, r, g, w);
    uint32_t h[32];
    widen_half<FMT>(w, f, zf, h);
    tmem_st_32x32b_x32(taddr + g * 32, h);
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(cluster_addr));
    return v;
}

// Split-K fix-up of rank `rank` of a CS-CTA cluster: weight rows
// [rank * rows, (rank + 1) * rows) of the tile, mq groups of four activation
// rows each, read from every rank's partial at `red_base` (row stride
// `red_stride` floats) and summed in rank order 0..CS-1. One unit = one weight
// row x four activation rows; each of the 128 threads takes units et,
// et + 128, ... two at a time, with all 2 x CS remote loads issued before
// the first sum (a distributed-shared-memory load costs several hundred
// cycles; issued one at a time they dominated the kernel).
template <int CS>
__device__ __forceinline__ void split_reduce(uint32_t red_base, int red_stride, int rank, int rows, int mq, int et,
                                             int n0, int M, int N, const float* rsc,
                                             const float* __restrict__ rowscale, float* __restrict__ out, int epi) {
    const int total = rows * mq;
    for (int u0 = et; u0 < total; u0 += 256) {
        float4 v[2][CS];
        #pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int unit = (u0 + h * 128 < total) ? u0 + h * 128 : u0;
            const int rl = rank * rows + unit % rows;
            const uint32_t off = static_cast<uint32_t>((rl * red_stride + 4 * (unit / rows)) * 4);
            #pragma unroll
            for (int p = 0; p < CS; ++p) v[h][p] = ld_dsmem_f4(mapa_shared(red_base + off, static_cast<uint32_t>(p)));
        }
        #pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int unit = u0 + h * 128;
            if (unit >= total) break;
            const int rl = rank * rows + unit % rows;  // weight row within the tile
            const int m = 4 * (unit / rows);
            float4 acc = v[h][0];
            #pragma unroll
            for (int p = 1; p < CS; ++p) {
                acc.x += v[h][p].x;
                acc.y += v[h][p].y;
                acc.z += v[h][p].z;
                acc.w += v[h][p].w;
            }
            const int nn = n0 + rl;
            if (nn < N) {
                const float sc = rsc[rl];
                const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
                #pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (m + k < M) {
                        store_out(out + static_cast<int64_t>(m + k) * N + nn, (a4[k] * __ldg(rowscale + m + k)) * sc,
                                  epi);
                    }
                }
            }
        }
    }
}

// Split-K over a cluster: with `splits` = C > 1 the C CTAs of a cluster
// (consecutive blockIdx.x) share one 128-row tile, rank r taking k-blocks
// [num_kb * r / C, num_kb * (r + 1) / C). Each rank copies its accumulator
// into its idle ring, and after a cluster barrier rank r adds the C partials
// of weight rows [128 r / C, 128 (r + 1) / C) in rank order 0..C-1 through
// distributed shared memory, so results do not depend on timing.
template <int BM, int FMT>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
               float* __restrict__ out, const float* __restrict__ scale, const float* __restrict__ rowscale,
               const float* __restrict__ zero, int gs, int M, int N, int K, int splits, int epi) {
    using C = Cfg<BM, FMT>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int kBK = C::kBK;
    uint8_t* xs = smem;                                  // S x kSub x [BM][64] f16, 128B swizzle
    uint8_t* ws = smem + S * C::kXBytes;                 // S x [128][kWRow] weight codes
    uint64_t* bars = reinterpret_cast<uint64_t*>(ws + S * C::kWBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    float* rsc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(tmem_slot) + 16);  // [128] output scales
    float* stage = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(rsc + kTileN) + 15) & ~uintptr_t(15));
    float* red = reinterpret_cast<float*>(smem);         // split-K partial, reuses the ring

    // full[s]: stage s landed (TMA). afull[s]: A buffer s written (8 converter
    // warps). release[s]: the MMAs reading stage s and A buffer s finished.
    const uint32_t full0 = smem_addr(bars);
    const uint32_t afull0 = full0 + 8 * S;
    const uint32_t release0 = afull0 + 8 * S;
    const uint32_t acc_full = release0 + 8 * S;
    const uint32_t drain = acc_full + 8;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rank = static_cast<int>(blockIdx.x) % splits;
    const int n0 = (static_cast<int>(blockIdx.x) / splits) * kTileN;
    const int num_kb = (K + kBK - 1) / kBK;
    const int kb0 = num_kb * rank / splits;
    const int n_kb = num_kb * (rank + 1) / splits - kb0;
    unsigned int* err = &g_tc_error;
    // Plain epilogue into 16-byte aligned rows: stores go out as float4 runs.
    const bool vec_out = C::kStaged && epi == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (N & 3) == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(afull0 + 8 * s, 4 * kConvGroups);
            mbar_init(release0 + 8 * s, 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == kWarpTma && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    // Launched as a programmatic dependent of the x -> f16 prologue: warm L2
    // with this CTA's first weight tiles (written before the prologue ran,
    // so already complete), then wait for x16 and rowscale.
    if (warp == kWarpTma && lane == 0) {
        for (int i = 0; i < S && i < n_kb; ++i) tma_prefetch_l2_2d(&tmap_w, (kb0 + i) * C::kWRow, n0);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t acc_tmem = tmem;               // partial accumulator p at columns [p BM, (p + 1) BM)
    const uint32_t a_tmem0 = tmem + C::kAcc * BM;  // A buffer s at columns kAcc BM + kACols s

    if (warp == kWarpTma) {
        if (lane == 0) {
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % S;
                if (i >= S && !mbar_wait(release0 + 8 * s, ((i / S) - 1) & 1, err, 1u)) break;
                const int kb = kb0 + i;
                mbar_arrive_expect_tx(full0 + 8 * s, C::kXBytes + C::kWBytes);
                #pragma unroll
                for (int sub = 0; sub < C::kSub; ++sub) {
                    tma_load_2d(smem_addr(xs + s * C::kXBytes + sub * BM * 128), &tmap_x, kb * kBK + sub * 64, 0,
                                full0 + 8 * s);
                }
                tma_load_2d(smem_addr(ws + s * C::kWBytes), &tmap_w, kb * C::kWRow, n0, full0 + 8 * s);
            }
            // Nothing of ours may still be landing in shared memory at exit:
            // wait (bounded) for the last fill of every stage.
            for (int i = (n_kb > S ? n_kb - S : 0); i < n_kb; ++i) {
                mbar_wait(full0 + 8 * (i % S), (i / S) & 1, err, 64u);
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kTileN, BM);
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % S;
                if (!mbar_wait(full0 + 8 * s, (i / S) & 1, err, 2u)) break;
                if (!mbar_wait(afull0 + 8 * s, (i / S) & 1, err, 4u)) break;
                tc_fence_after();
                #pragma unroll
                for (int j = 0; j < kBK / 16; ++j) {
                    // K step of 16 f16 = 32 bytes inside a 128-byte swizzle row of
                    // the (j / 4)-th 64-wide atom of the activation tile.
                    const uint64_t bdesc =
                        smem_desc_sw128_kmajor(smem_addr(xs + s * C::kXBytes + (j / 4) * BM * 128));
                    mma_f16_ts(acc_tmem + (j % C::kAcc) * BM, a_tmem0 + s * C::kACols + j * 8,
                               bdesc + static_cast<uint64_t>((j % 4) * 2), idesc, (i > 0 || j >= C::kAcc) ? 1u : 0u);
                }
                mma_commit(release0 + 8 * s);
            }
            mma_commit(acc_full);
            // Every MMA must be finished before tensor memory is released.
            mma_commit(drain);
            mbar_wait(drain, 0, err, 128u);
        }
    } else if (warp < kWarpEpi0) {
        // Converters: thread owns weight row r of the tile = tensor-memory lane r.
        // Both groups of four warps convert every k-block, group g its codes
        // [64 g, 64 g + 64), so a block is ready in half a conversion's time.
        const int quarter = warp & 3;
        const int group = (warp - kWarpConv0) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        float pw = 1.0f;
        if constexpr (FMT != kFmtChannel) {
            pw = __int_as_float((group_row_exp<FMT>(scale, zero, n0 + r, N, K / gs) + 127) << 23);
        }
        // Group factors one k-block ahead: the loads for the next block overlap
        // this block's wait and conversion.
        float f[2] = {}, zf[2] = {};
        if constexpr (FMT != kFmtChannel) {
            if (n_kb > 0) group_factors<FMT>(scale, zero, n0 + r, N, K, gs, kb0, group, pw, f, zf);
        }
        for (int i = 0; i < n_kb; ++i) {
            const int s = i % S;
            float fn[2] = {}, zn[2] = {};
            if constexpr (FMT != kFmtChannel) {
                if (i + 1 < n_kb) group_factors<FMT>(scale, zero, n0 + r, N, K, gs, kb0 + i + 1, group, pw, fn, zn);
            }
            bool ok = mbar_wait(full0 + 8 * s, (i / S) & 1, err, 8u);
            if (ok && i >= S) ok = mbar_wait(release0 + 8 * s, ((i / S) - 1) & 1, err, 16u);
            // tcgen05.st below is warp-collective: leave together or not at all.
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            convert_half<FMT>(ws + s * C::kWBytes, r, group, tmem + lane_addr + C::kAcc * BM + s * C::kACols, f, zf);
            #pragma unroll
            for (int q = 0; q < 2; ++q) {
                f[q] = fn[q];
                zf[q] = zn[q];
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(afull0 + 8 * s);
        }
    } else {
        // Epilogue: lane = weight row n, 32 accumulator columns (activation rows) per load.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int n = n0 + row;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        // Output scale of row n: scale[n], or 2^-e_n for a per-group format.
        float sc = 0.0f;
        if (n < N) {
            if constexpr (FMT == kFmtChannel) {
                sc = __ldg(scale + n);
            } else {
                sc = __int_as_float((127 - group_row_exp<FMT>(scale, zero, n, N, K / gs)) << 23);
            }
        }
        rsc[row] = sc;
        const bool ok = mbar_wait(acc_full, 0, err, 32u);
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            // The ring's last asynchronous (TMA, MMA) accesses are complete;
            // order them before this thread's generic stores into it.
            if (splits > 1) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            #pragma unroll 1
            for (int c0 = 0; c0 < BM; c0 += 32) {
                if (c0 >= M) break;
                uint32_t v[32];
                acc_ld32<C::kAcc>(acc_tmem + lane_addr + c0, BM, v);
                if (splits > 1) {
                    // The ring is idle: every MMA has finished reading it.
                    float4* dst = reinterpret_cast<float4*>(red + row * C::kRedStride + c0);
                    #pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        dst[q4] = make_float4(__uint_as_float(v[4 * q4]), __uint_as_float(v[4 * q4 + 1]),
                                              __uint_as_float(v[4 * q4 + 2]), __uint_as_float(v[4 * q4 + 3]));
                    }
                } else if (vec_out && n0 + quarter * 32 + 32 <= N) {
                    store_chunk_v(out, rowscale, c0, M - c0, n0 + quarter * 32, N, sc, v, stage + quarter * 1024,
                                  lane);
                } else if (n < N) {
                    store_chunk(out, rowscale, c0, M - c0, n, N, sc, v, epi);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (splits > 1) {
        // Every rank's partial is in its shared memory.
        cluster_sync();
        if (warp >= kWarpEpi0) {
            const int et = threadIdx.x - kWarpEpi0 * 32;  // 0..127
            const int rows = kTileN / splits;
            const int mq = ((M < BM ? M : BM) + 3) / 4;  // 4-column groups the epilogue wrote
            const uint32_t red_base = smem_addr(red);
            if (splits == 2) {
                split_reduce<2>(red_base, C::kRedStride, rank, rows, mq, et, n0, M, N, rsc, rowscale, out, epi);
            } else if (splits == 4) {
                split_reduce<4>(red_base, C::kRedStride, rank, rows, mq, et, n0, M, N, rsc, rowscale, out, epi);
            } else {
                split_reduce<8>(red_base, C::kRedStride, rank, rows, mq, et, n0, M, N, rsc, rowscale, out, epi);
            }
        }
        // No rank may leave while another still reads its shared memory.
        cluster_sync();
    }
    if (warp == kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ------------------------------------------------------------ CTA-pair kernel
// Large M: a cluster of two CTAs computes a 256 (weight rows) x 2*RX
// (activation rows) tile with tcgen05.mma.cta_group::2. CTA r of the pair
// converts its own 128 weight rows into its own tensor memory (the A operand
// is split by rows across the pair) and loads only its half of the
// activation tile (the B operand is split the same way), so each CTA moves
// half the tiles a single CTA with the same output tile would, and the
// pair's MMA work per k-step doubles.
// The leader CTA (rank 0) issues the MMAs; the pair synchronises through the
// leader's mbarriers:
//   full[s]   activation halves of both CTAs landed (TMA .cta_group::2 loads
//             complete their bytes on the leader's barrier; only the leader
//             posts the expected byte count);
//   wfull[s]  this CTA's weight tile landed (local);
//   afull[s]  both CTAs' converters wrote A buffer s (16 remote arrivals);
//   release[s], acc_full, drain: multicast tcgen05.commit from the leader to
//             the same barrier in both CTAs (release[s] frees ring slot s:
//             its shared-memory tiles and A buffer s).
// Stages are 128 deep in K: a CTA's TMA ring costs a roughly fixed time per
// iteration (measured on this part: ~0.4 us whether a stage carries 8 KB or
// 40 KB), so fewer, bigger stages move the same bytes in half the iterations.
// RX activation rows per CTA (the pair's MMA is 256 x 2*RX): 128 for
// prefill, 16/32/64 for skinny shapes with many weight tiles, where one MMA
// instruction now covers both CTAs' 128 weight rows.
// Persistent: a pair walks the output tiles t = pair, pair + pairs, ...; the
// ring's slots and barrier phases run on across tiles (a k-block counter
// shared by all roles), so the next tile's loads and conversions proceed
// while the epilogue of the previous one drains. The accumulator is single:
// acc_full (multicast commit) hands it to the epilogue, acc_empty (eight
// epilogue warps of both CTAs, on the leader) hands it back once read.
template <int RX, int FMT = kFmtChannel>
struct PairCfg {
    static constexpr int kBK = 128;
    static constexpr int kSub = kBK / 64;                  // 64-wide f16 swizzle atoms per stage
    static constexpr int kRowsX = RX;
    static constexpr int kXBytes = RX * kBK * 2;           // f16 activation half-tile per stage
    static constexpr int kWRow = FMT == kFmtGroup4 ? kBK / 2 : kBK;  // weight bytes per row and stage
    static constexpr int kWBytes = kTileN * kWRow;         // weight tile per stage (16 KB int8, 8 KB int4)
    static constexpr int kACols = kBK / 2;
    static constexpr int kTmemCols = 512;                  // 2*RX accumulator + A buffers
    // Ring slot s is also A buffer s (one release barrier frees both):
    // as many stages as both shared and tensor memory hold.
    static constexpr int kSmemStages = (RX >= 128) ? 4 : (RX >= 64 ? 6 : 8);
    // Two partial accumulators for narrow tiles (k-steps alternate between
    // them, so consecutive MMAs do not wait on each other's results); wide
    // tiles keep one, their MMAs are long enough to hide the dependency.
    static constexpr int kAcc = RX <= 32 ? 2 : 1;
    static constexpr int kTmemStages = (kTmemCols - kAcc * 2 * RX) / kACols;
    static constexpr int kStages = kSmemStages < kTmemStages ? kSmemStages : kTmemStages;
    static constexpr int kAStages = kStages;
    static constexpr int kNumBars = 4 * kStages + 3;
    // Epilogue [32 x 32] f32 staging tile per epilogue warp, for tiles of 64
    // or more activation rows (a single 32-column chunk stores directly).
    static constexpr bool kStaged = 2 * RX >= 64;
    static constexpr int kStageBytes = kStaged ? 4 * 32 * 32 * 4 : 0;
    static constexpr int kSmem = 1024 + kStages * (kXBytes + kWBytes) + kNumBars * 8 + 16 + 16 + kStageBytes;
    static_assert(kSmem <= 227 * 1024, "shared memory per block");
    static_assert(kAcc * 2 * RX + kAStages * kACols <= kTmemCols, "tensor memory holds 512 columns");
    static_assert(kXBytes % 1024 == 0, "x16 stages must stay 1024-byte aligned");
};

template <int RX, int FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
tc_gemm_pair_persist_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                    float* __restrict__ out, const float* __restrict__ scale, const float* __restrict__ rowscale,
                    const float* __restrict__ zero, int gs, int M, int N, int K, int epi) {
    using P = PairCfg<RX, FMT>;
    constexpr int kBK = P::kBK;
    constexpr int kSub = P::kSub;
    constexpr int kRowsX = P::kRowsX;
    constexpr int kXBytes = P::kXBytes;
    constexpr int kWBytes = P::kWBytes;
    constexpr int kACols = P::kACols;
    constexpr int kTmemCols = P::kTmemCols;
    constexpr int kNumBars = P::kNumBars;
    constexpr int S = P::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xs = smem;                                  // S x kSub x [RX][64] f16, 128B swizzle
    uint8_t* ws = smem + S * kXBytes;                    // S x [128][kWRow] weight codes
    uint64_t* bars = reinterpret_cast<uint64_t*>(ws + S * kWBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
    float* stage = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tmem_slot) + 16 + 15) & ~uintptr_t(15));

    // full[s]: both activation halves landed (leader). wfull[s]: this CTA's
    // weight tile landed. afull[s]: both CTAs' converters wrote A buffer s.
    // release[s]: the MMAs of slot s finished (multicast commit to both
    // CTAs): its tiles and A buffer may be refilled. acc_full / acc_empty:
    // the accumulator of a tile is complete / has been read.
    const uint32_t full0 = smem_addr(bars);
    const uint32_t wfull0 = full0 + 8 * S;
    const uint32_t release0 = wfull0 + 8 * S;
    const uint32_t afull0 = release0 + 8 * S;
    const uint32_t acc_full = afull0 + 8 * S;
    const uint32_t acc_empty = acc_full + 8;
    const uint32_t drain = acc_empty + 8;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int pairs = static_cast<int>(gridDim.x >> 1);
    const int tiles_n = (N + 2 * kTileN - 1) / (2 * kTileN);
    const int tiles = tiles_n * ((M + 2 * kRowsX - 1) / (2 * kRowsX));
    const int num_kb = (K + kBK - 1) / kBK;
    unsigned int* err = &g_tc_error;
    // Plain epilogue into 16-byte aligned rows: stores go out as float4 runs.
    const bool vec_out = P::kStaged && epi == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (N & 3) == 0;
    // Tile t: this CTA's weight rows n0 .. n0 + 127 and the pair's activation
    // rows mp .. mp + 2*RX - 1.
    auto tile_n0 = [&](int t) { return (t % tiles_n) * (2 * kTileN) + static_cast<int>(rank) * kTileN; };
    auto tile_mp = [&](int t) { return (t / tiles_n) * (2 * kRowsX); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(wfull0 + 8 * s, 1);
            mbar_init(release0 + 8 * s, 1);
            mbar_init(afull0 + 8 * s, 2 * 4 * kConvGroups);  // every converter warp of both CTAs
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * 4);  // the four epilogue warps of both CTAs
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == kWarpTma && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == kWarpMma) {
        tmem_alloc_pair(smem_addr(tmem_slot), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers exist before anyone arrives on them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t a_tmem0 = tmem + P::kAcc * 2 * kRowsX;  // A buffers after the accumulator columns

    // Launched as a programmatic dependent of the x -> f16 prologue. The
    // weights were written before the prologue ran, so the first ring of
    // weight tiles is requested (and converted) while the prologue still
    // runs; only the activation loads and the epilogue's row scales wait
    // for it (griddepcontrol.wait in those threads).
    if (warp == kWarpTma) {
        if (lane == 0) {
            const uint32_t full_leader0 = mapa_shared(full0, 0);
            const int first = (pair < tiles) ? (num_kb < S ? num_kb : S) : 0;
            for (int kb = 0; kb < first; ++kb) {
                mbar_arrive_expect_tx(wfull0 + 8 * kb, kWBytes);
                tma_load_2d(smem_addr(ws + kb * kWBytes), &tmap_w, kb * P::kWRow, tile_n0(pair), wfull0 + 8 * kb);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            int g = 0;  // k-blocks issued so far (all tiles)
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += pairs) {
                const int n0 = tile_n0(t);
                const int mp = tile_mp(t);
                for (int kb = 0; kb < num_kb; ++kb, ++g) {
                    const int s = g % S;
                    if (g >= S && !mbar_wait_cluster(release0 + 8 * s, ((g / S) - 1) & 1, err, 1u)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(full0 + 8 * s, 2 * kXBytes);
                    #pragma unroll
                    for (int sub = 0; sub < kSub; ++sub) {
                        tma_load_2d_pair(smem_addr(xs + s * kXBytes + sub * kRowsX * 128), &tmap_x,
                                         kb * kBK + sub * 64, mp + static_cast<int>(rank) * kRowsX,
                                         full_leader0 + 8 * s);
                    }
                    if (g >= first) {
                        mbar_arrive_expect_tx(wfull0 + 8 * s, kWBytes);
                        tma_load_2d(smem_addr(ws + s * kWBytes), &tmap_w, kb * P::kWRow, n0, wfull0 + 8 * s);
                    }
                }
            }
            // Leave no copy of ours in flight: the weight tiles signal this CTA;
            // the activation halves are covered by the drain below (the leader
            // consumes every stage before it commits the drain).
            for (int i = (g > S ? g - S : 0); i < g; ++i) mbar_wait(wfull0 + 8 * (i % S), (i / S) & 1, err, 64u);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_f16_f32(2 * kTileN, 2 * kRowsX);
            int g = 0;
            int it = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += pairs, ++it) {
                // The previous tile's accumulator must have been read out.
                if (it > 0 && !mbar_wait_cluster(acc_empty, (it - 1) & 1, err, 4u)) break;
                tc_fence_after();
                for (int kb = 0; kb < num_kb; ++kb, ++g) {
                    const int s = g % S;
                    if (!mbar_wait_cluster(full0 + 8 * s, (g / S) & 1, err, 2u) ||
                        !mbar_wait_cluster(afull0 + 8 * s, (g / S) & 1, err, 4u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    #pragma unroll
                    for (int j = 0; j < kBK / 16; ++j) {
                        const uint64_t bdesc =
                            smem_desc_sw128_kmajor(smem_addr(xs + s * kXBytes + (j / 4) * kRowsX * 128));
                        mma_f16_ts_pair(tmem + (j % P::kAcc) * 2 * kRowsX, a_tmem0 + s * kACols + j * 8,
                                        bdesc + static_cast<uint64_t>((j % 4) * 2), idesc,
                                        (kb > 0 || j >= P::kAcc) ? 1u : 0u);
                    }
                    mma_commit_pair(release0 + 8 * s, 0x3);
                }
                if (ok) mma_commit_pair(acc_full, 0x3);
            }
            mma_commit_pair(drain, 0x3);
        }
    } else if (warp < kWarpEpi0) {
        // Converters: thread owns weight row r of this CTA's 128 = tensor-memory
        // lane r; both groups convert every k-block, group g its codes
        // [64 g, 64 g + 64).
        const int quarter = warp & 3;
        const int group = (warp - kWarpConv0) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t afull_leader0 = mapa_shared(afull0, 0);
        int g = 0;
        bool ok = true;
        for (int t = pair; t < tiles && ok; t += pairs) {
            const int n0 = tile_n0(t);
            float pw = 1.0f;
            if constexpr (FMT != kFmtChannel) {
                pw = __int_as_float((group_row_exp<FMT>(scale, zero, n0 + r, N, K / gs) + 127) << 23);
            }
            // Group factors one k-block ahead, their loads overlapping this
            // block's waits and conversion.
            float f[2] = {}, zf[2] = {};
            if constexpr (FMT != kFmtChannel) group_factors<FMT>(scale, zero, n0 + r, N, K, gs, 0, group, pw, f, zf);
            for (int kb = 0; kb < num_kb; ++kb, ++g) {
                const int s = g % S;
                float fn[2] = {}, zn[2] = {};
                if constexpr (FMT != kFmtChannel) {
                    if (kb + 1 < num_kb) {
                        group_factors<FMT>(scale, zero, n0 + r, N, K, gs, kb + 1, group, pw, fn, zn);
                    }
                }
                bool w_ok = mbar_wait(wfull0 + 8 * s, (g / S) & 1, err, 8u);
                if (w_ok && g >= S) w_ok = mbar_wait_cluster(release0 + 8 * s, ((g / S) - 1) & 1, err, 16u);
                // tcgen05.st is warp-collective: leave together or not at all.
                if (!__all_sync(0xffffffffu, w_ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                convert_half<FMT>(ws + s * kWBytes, r, group, tmem + lane_addr + P::kAcc * 2 * kRowsX + s * kACols, f,
                                  zf);
                #pragma unroll
                for (int q = 0; q < 2; ++q) {
                    f[q] = fn[q];
                    zf[q] = zn[q];
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(afull_leader0 + 8 * s);
            }
        }
    } else {
        // Epilogue: lane = weight row n of this CTA, 2*RX accumulator columns =
        // activation rows mp .. mp + 2*RX - 1 of the pair.
        const int quarter = warp & 3;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t acc_empty_leader = mapa_shared(acc_empty, 0);
        asm volatile("griddepcontrol.wait;" ::: "memory");  // row scales come from the prologue
        int it = 0;
        for (int t = pair; t < tiles; t += pairs, ++it) {
            const int n = tile_n0(t) + quarter * 32 + lane;
            const int mp = tile_mp(t);
            // Output scale of row n: scale[n], or 2^-e_n for a per-group format.
            float sc = 0.0f;
            if (n < N) {
                if constexpr (FMT == kFmtChannel) {
                    sc = __ldg(scale + n);
                } else {
                    sc = __int_as_float((127 - group_row_exp<FMT>(scale, zero, n, N, K / gs)) << 23);
                }
            }
            const bool ok = mbar_wait_cluster(acc_full, it & 1, err, 32u);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            // 32 accumulator columns per read; the accumulator is handed back
            // to the MMA warp as soon as its last columns are in registers.
            const int rows_m = (M - mp < 2 * kRowsX) ? M - mp : 2 * kRowsX;  // activation rows of the tile
            const int n0w = tile_n0(t) + quarter * 32;                      // the warp's first weight row
            #pragma unroll 1
            for (int c0 = 0; c0 < rows_m; c0 += 32) {
                uint32_t v[32];
                acc_ld32<P::kAcc>(tmem + lane_addr + c0, 2 * kRowsX, v);
                if (c0 + 32 >= rows_m) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
                }
                if (vec_out && n0w + 32 <= N) {
                    store_chunk_v(out, rowscale, mp + c0, rows_m - c0, n0w, N, sc, v, stage + quarter * 1024, lane);
                } else if (n < N) {
                    store_chunk(out, rowscale, mp + c0, rows_m - c0, n, N, sc, v, epi);
                }
            }
        }
    }

    // Every MMA of the pair must be finished before either CTA releases its
    // tensor memory or shared memory: wait for the drain commit, then meet.
    if (warp == kWarpMma && lane == 0) mbar_wait_cluster(drain, 0, err, 128u);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTmemCols);
    }
}

// One output tile per pair (grid = every tile): used when all tiles are
// resident at once, so there is nothing to overlap between tiles and the
// single-tile loops are the cheaper ones to issue.
template <int RX, int FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                    float* __restrict__ out, const float* __restrict__ scale, const float* __restrict__ rowscale,
                    const float* __restrict__ zero, int gs, int M, int N, int K, int epi) {
    using P = PairCfg<RX, FMT>;
    constexpr int kBK = P::kBK;
    constexpr int kSub = P::kSub;
    constexpr int kRowsX = P::kRowsX;
    constexpr int kXBytes = P::kXBytes;
    constexpr int kWBytes = P::kWBytes;
    constexpr int kACols = P::kACols;
    constexpr int kTmemCols = P::kTmemCols;
    constexpr int kNumBars = P::kNumBars;
    constexpr int S = P::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xs = smem;                                  // S x kSub x [RX][64] f16, 128B swizzle
    uint8_t* ws = smem + S * kXBytes;                    // S x [128][kWRow] weight codes
    uint64_t* bars = reinterpret_cast<uint64_t*>(ws + S * kWBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
    float* stage = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tmem_slot) + 16 + 15) & ~uintptr_t(15));

    // full[s]: both activation halves landed (leader). wfull[s]: this CTA's
    // weight tile landed. afull[s]: both CTAs' converters wrote A buffer s.
    // release[s]: the MMAs of slot s finished (multicast commit to both
    // CTAs): its tiles and A buffer may be refilled.
    const uint32_t full0 = smem_addr(bars);
    const uint32_t wfull0 = full0 + 8 * S;
    const uint32_t release0 = wfull0 + 8 * S;
    const uint32_t afull0 = release0 + 8 * S;
    const uint32_t acc_full = afull0 + 8 * S;
    const uint32_t drain = acc_full + 8;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int n0 = (blockIdx.x >> 1) * (2 * kTileN) + static_cast<int>(rank) * kTileN;  // this CTA's weight rows
    const int mp = blockIdx.y * (2 * kRowsX);                                          // pair's activation rows
    const int num_kb = (K + kBK - 1) / kBK;
    unsigned int* err = &g_tc_error;
    // Plain epilogue into 16-byte aligned rows: stores go out as float4 runs.
    const bool vec_out = P::kStaged && epi == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (N & 3) == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(wfull0 + 8 * s, 1);
            mbar_init(release0 + 8 * s, 1);
            mbar_init(afull0 + 8 * s, 2 * 4 * kConvGroups);  // every converter warp of both CTAs
        }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == kWarpTma && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == kWarpMma) {
        tmem_alloc_pair(smem_addr(tmem_slot), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers exist before anyone arrives on them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t a_tmem0 = tmem + P::kAcc * 2 * kRowsX;  // A buffers after the accumulator columns

    // Launched as a programmatic dependent of the x -> f16 prologue. The
    // weights were written before the prologue ran, so the first ring of
    // weight tiles is requested (and converted) while the prologue still
    // runs; only the activation loads and the epilogue's row scales wait
    // for it (griddepcontrol.wait in those threads).
    if (warp == kWarpTma) {
        if (lane == 0) {
            const uint32_t full_leader0 = mapa_shared(full0, 0);
            const int first = num_kb < S ? num_kb : S;
            for (int kb = 0; kb < first; ++kb) {
                mbar_arrive_expect_tx(wfull0 + 8 * kb, kWBytes);
                tma_load_2d(smem_addr(ws + kb * kWBytes), &tmap_w, kb * P::kWRow, n0, wfull0 + 8 * kb);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % S;
                if (kb >= S && !mbar_wait_cluster(release0 + 8 * s, ((kb / S) - 1) & 1, err, 1u)) break;
                if (leader) mbar_arrive_expect_tx(full0 + 8 * s, 2 * kXBytes);
                #pragma unroll
                for (int sub = 0; sub < kSub; ++sub) {
                    tma_load_2d_pair(smem_addr(xs + s * kXBytes + sub * kRowsX * 128), &tmap_x, kb * kBK + sub * 64,
                                     mp + static_cast<int>(rank) * kRowsX, full_leader0 + 8 * s);
                }
                if (kb >= first) {
                    mbar_arrive_expect_tx(wfull0 + 8 * s, kWBytes);
                    tma_load_2d(smem_addr(ws + s * kWBytes), &tmap_w, kb * P::kWRow, n0, wfull0 + 8 * s);
                }
            }
            // Leave no copy of ours in flight: the weight tiles signal this CTA;
            // the activation halves are covered by the drain below (the leader
            // consumes every stage before it commits the drain).
            for (int kb = (num_kb > S ? num_kb - S : 0); kb < num_kb; ++kb) {
                mbar_wait(wfull0 + 8 * (kb % S), (kb / S) & 1, err, 64u);
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_f16_f32(2 * kTileN, 2 * kRowsX);
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % S;
                const int a = s;
                if (!mbar_wait_cluster(full0 + 8 * s, (kb / S) & 1, err, 2u)) break;
                if (!mbar_wait_cluster(afull0 + 8 * a, (kb / S) & 1, err, 4u)) break;
                tc_fence_after();
                #pragma unroll
                for (int j = 0; j < kBK / 16; ++j) {
                    const uint64_t bdesc = smem_desc_sw128_kmajor(smem_addr(xs + s * kXBytes + (j / 4) * kRowsX * 128));
                    mma_f16_ts_pair(tmem + (j % P::kAcc) * 2 * kRowsX, a_tmem0 + a * kACols + j * 8,
                                    bdesc + static_cast<uint64_t>((j % 4) * 2), idesc,
                                    (kb > 0 || j >= P::kAcc) ? 1u : 0u);
                }
                mma_commit_pair(release0 + 8 * s, 0x3);
            }
            mma_commit_pair(acc_full, 0x3);
            mma_commit_pair(drain, 0x3);
        }
    } else if (warp < kWarpEpi0) {
        // Converters: thread owns weight row r of this CTA's 128 = tensor-memory
        // lane r; both groups convert every k-block, group g its codes
        // [64 g, 64 g + 64).
        const int quarter = warp & 3;
        const int group = (warp - kWarpConv0) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t afull_leader0 = mapa_shared(afull0, 0);
        float pw = 1.0f;
        if constexpr (FMT != kFmtChannel) {
            pw = __int_as_float((group_row_exp<FMT>(scale, zero, n0 + r, N, K / gs) + 127) << 23);
        }
        // Group factors one k-block ahead, their loads overlapping this block's
        // waits and conversion.
        float f[2] = {}, zf[2] = {};
        if constexpr (FMT != kFmtChannel) {
            if (num_kb > 0) group_factors<FMT>(scale, zero, n0 + r, N, K, gs, 0, group, pw, f, zf);
        }
        for (int kb = 0; kb < num_kb; ++kb) {
            const int s = kb % S;
            const int a = s;
            float fn[2] = {}, zn[2] = {};
            if constexpr (FMT != kFmtChannel) {
                if (kb + 1 < num_kb) group_factors<FMT>(scale, zero, n0 + r, N, K, gs, kb + 1, group, pw, fn, zn);
            }
            bool ok = mbar_wait(wfull0 + 8 * s, (kb / S) & 1, err, 8u);
            if (ok && kb >= S) ok = mbar_wait_cluster(release0 + 8 * s, ((kb / S) - 1) & 1, err, 16u);
            // tcgen05.st is warp-collective: leave together or not at all.
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            convert_half<FMT>(ws + s * kWBytes, r, group, tmem + lane_addr + P::kAcc * 2 * kRowsX + a * kACols, f, zf);
            #pragma unroll
            for (int q = 0; q < 2; ++q) {
                f[q] = fn[q];
                zf[q] = zn[q];
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(afull_leader0 + 8 * a);
        }
    } else {
        // Epilogue: lane = weight row n of this CTA, 2*RX accumulator columns =
        // activation rows mp .. mp + 2*RX - 1 of the pair.
        const int quarter = warp & 3;
        const int n = n0 + quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        // Output scale of row n: scale[n], or 2^-e_n for a per-group format.
        float sc = 0.0f;
        if (n < N) {
            if constexpr (FMT == kFmtChannel) {
                sc = __ldg(scale + n);
            } else {
                sc = __int_as_float((127 - group_row_exp<FMT>(scale, zero, n, N, K / gs)) << 23);
            }
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");  // row scales come from the prologue
        const bool ok = mbar_wait_cluster(acc_full, 0, err, 32u);
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            // Activation rows of this tile: 2*RX, or fewer in the last tile row.
            const int rows_m = (M - mp < 2 * kRowsX) ? M - mp : 2 * kRowsX;
            #pragma unroll 1
            for (int c0 = 0; c0 < rows_m; c0 += 32) {
                uint32_t v[32];
                acc_ld32<P::kAcc>(tmem + lane_addr + c0, 2 * kRowsX, v);
                const int n0w = n0 + quarter * 32;  // the warp's first weight row
                if (vec_out && n0w + 32 <= N) {
                    store_chunk_v(out, rowscale, mp + c0, rows_m - c0, n0w, N, sc, v, stage + quarter * 1024, lane);
                } else if (n < N) {
                    store_chunk(out, rowscale, mp + c0, rows_m - c0, n, N, sc, v, epi);
                }
            }
        }
    }

    // Every MMA of the pair must be finished before either CTA releases its
    // tensor memory or shared memory: wait for the drain commit, then meet.
    if (warp == kWarpMma && lane == 0) mbar_wait_cluster(drain, 0, err, 128u);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTmemCols);
    }
}

// ---------------------------------------------- int8 tensor path (M <= 128)
// Per-channel int8 weights, M <= 128 activation rows: the weight codes go
// from TMA straight into tcgen05.mma.kind::i8 as the A operand (shared
// memory, 128B swizzle), with no conversion. The B operand of a k-block is
// the [2 BM x 128] int8 tile of the prologue's digit planes (hi digits of
// the BM rows, then their lo digits), so each M=128, N=2 BM, K=32
// instruction adds the exact int32 dot products of both digits. The
// epilogue forms ((256 hi + lo) * mantissa_m) * scale[n] * 2^e_m in f32.
//
// Bounds: |code * digit| <= 128 * 128, so the int32 sums cannot wrap for
// K <= 131071 (the path is taken for K <= 65536).
//
// Warp roles (6 warps): 0 TMA producer, 1 MMA issuer (and tensor-memory
// owner), 2-5 epilogue (warp w reads tensor-memory lanes 32 (w % 4) ..).
// Split-K over a cluster of C CTAs when the 128-row tiles fill less than
// half the GPU: each rank writes its f32 partial tile [BM][128] to global
// scratch (L2), and after a cluster barrier rank r sums weight rows
// [128 r / C, 128 (r + 1) / C) over the C partials in rank order.
constexpr int kI8Threads = 192;
constexpr int kI8WarpEpi0 = 2;

template <int BM>
struct CfgI8 {
    static constexpr int kBK = 128;                  // k-block depth (int8 elements = bytes)
    static constexpr int kN = 2 * BM;                // MMA N: hi and lo digit rows
    static constexpr int kXBytes = kN * kBK;         // digit tile per stage
    static constexpr int kWBytes = kTileN * kBK;     // weight tile per stage
    static constexpr int kStages = BM >= 128 ? 4 : (BM >= 64 ? 6 : 8);
    static constexpr int kAcc = 2;                   // k-steps alternate between two accumulators
    static constexpr int kTmemCols = kAcc * kN;      // 128, 256 or 512
    static constexpr int kNumBars = 2 * kStages + 2;
    static constexpr bool kStaged = BM >= 64;
    static constexpr int kStageBytes = kStaged ? 4 * 32 * 32 * 4 : 0;
    // ring, barriers, tensor-memory slot, staging tiles, row factors [2][BM]
    static constexpr int kSmem =
        1024 + kStages * (kXBytes + kWBytes) + kNumBars * 8 + 16 + 16 + kStageBytes + 2 * BM * 4;
    static_assert(kXBytes % 1024 == 0 && kWBytes % 1024 == 0, "stages stay 1024-byte aligned");
    static_assert(kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512, "tensor-memory allocation");
    static_assert(kSmem <= 227 * 1024, "shared memory per block");
};

template <int BM>
__global__ void __launch_bounds__(kI8Threads, 1)
tc_i8_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
             float* __restrict__ out, const float* __restrict__ scale, const float* __restrict__ rowfactor,
             const float* __restrict__ rowpow, float* __restrict__ part, int M, int N, int K, int splits, int epi) {
    using C = CfgI8<BM>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xs = smem;                                  // S x [2 BM][128] digits, 128B swizzle
    uint8_t* ws = smem + S * C::kXBytes;                 // S x [128][128] weight codes, 128B swizzle
    uint64_t* bars = reinterpret_cast<uint64_t*>(ws + S * C::kWBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    float* stage = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tmem_slot + 4) + 15) & ~uintptr_t(15));

    // full[s]: stage s landed. release[s]: the MMAs reading stage s finished.
    const uint32_t full0 = smem_addr(bars);
    const uint32_t release0 = full0 + 8 * S;
    const uint32_t acc_full = release0 + 8 * S;
    const uint32_t drain = acc_full + 8;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rank = static_cast<int>(blockIdx.x) % splits;
    const int n0 = (static_cast<int>(blockIdx.x) / splits) * kTileN;
    const int num_kb = (K + C::kBK - 1) / C::kBK;
    const int kb0 = num_kb * rank / splits;
    const int n_kb = num_kb * (rank + 1) / splits - kb0;
    unsigned int* err = &g_tc_error;
    const bool vec_out = C::kStaged && epi == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (N & 3) == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(release0 + 8 * s, 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
        // Weights were written before the prologue ran: warm L2 with this
        // CTA's first tiles while the prologue finishes.
        for (int i = 0; i < S && i < n_kb; ++i) tma_prefetch_l2_2d(&tmap_w, (kb0 + i) * C::kBK, n0);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    float* rf_s = stage + C::kStageBytes / 4;  // row factors: [BM] mantissas, then [BM] powers
    asm volatile("griddepcontrol.wait;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // accumulator p at columns [p 2BM, (p + 1) 2BM): hi at +0, lo at +BM

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % S;
                if (i >= S && !mbar_wait(release0 + 8 * s, ((i / S) - 1) & 1, err, 1u)) break;
                const int kb = kb0 + i;
                mbar_arrive_expect_tx(full0 + 8 * s, C::kXBytes + C::kWBytes);
                tma_load_2d(smem_addr(xs + s * C::kXBytes), &tmap_x, kb * C::kBK, 0, full0 + 8 * s);
                tma_load_2d(smem_addr(xs + s * C::kXBytes + BM * C::kBK), &tmap_x, kb * C::kBK, M, full0 + 8 * s);
                tma_load_2d(smem_addr(ws + s * C::kWBytes), &tmap_w, kb * C::kBK, n0, full0 + 8 * s);
            }
            // Nothing of ours may still be landing in shared memory at exit.
            for (int i = (n_kb > S ? n_kb - S : 0); i < n_kb; ++i) {
                mbar_wait(full0 + 8 * (i % S), (i / S) & 1, err, 64u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8_s32(kTileN, C::kN);
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % S;
                if (!mbar_wait(full0 + 8 * s, (i / S) & 1, err, 2u)) break;
                tc_fence_after();
                const uint64_t adesc = smem_desc_sw128_kmajor(smem_addr(ws + s * C::kWBytes));
                const uint64_t bdesc = smem_desc_sw128_kmajor(smem_addr(xs + s * C::kXBytes));
                #pragma unroll
                for (int j = 0; j < C::kBK / 32; ++j) {
                    // K step of 32 int8 = 32 bytes inside the 128-byte swizzle rows.
                    mma_i8_ss(tmem + (j % C::kAcc) * C::kN, adesc + static_cast<uint64_t>(2 * j),
                              bdesc + static_cast<uint64_t>(2 * j), idesc, (i > 0 || j >= C::kAcc) ? 1u : 0u);
                }
                mma_commit(release0 + 8 * s);
            }
            mma_commit(acc_full);
            // Every MMA must be finished before tensor memory is released.
            mma_commit(drain);
            mbar_wait(drain, 0, err, 128u);
        }
    } else {
        // Epilogue: lane = weight row n, 32 activation rows per chunk.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int n = n0 + row;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const float sc = n < N ? __ldg(scale + n) : 0.0f;
        // This CTA's row factors, once, into shared memory while the k-loop
        // runs (named barrier 1: the four epilogue warps only). Loading them
        // before the block-wide barrier above instead delayed the first
        // digit tile.
        for (int i = threadIdx.x - kI8WarpEpi0 * 32; i < BM; i += 128) {
            rf_s[i] = i < M ? __ldg(rowfactor + i) : 0.0f;
            rf_s[BM + i] = i < M ? __ldg(rowpow + i) : 0.0f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool ok = mbar_wait(acc_full, 0, err, 32u) && n_kb > 0;
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            #pragma unroll 1
            for (int c0 = 0; c0 < BM; c0 += 32) {
                if (c0 >= M) break;
                uint32_t h0[32], h1[32];
                tmem_ld_32x32b_x32(tmem + lane_addr + c0, h0);
                tmem_ld_32x32b_x32(tmem + lane_addr + C::kN + c0, h1);
                tmem_wait_ld();
                #pragma unroll
                for (int j = 0; j < 32; ++j) {
                    h0[j] = static_cast<uint32_t>(static_cast<int>(h0[j]) + static_cast<int>(h1[j]));
                }
                uint32_t l0[32];
                tmem_ld_32x32b_x32(tmem + lane_addr + BM + c0, l0);
                tmem_ld_32x32b_x32(tmem + lane_addr + C::kN + BM + c0, h1);
                tmem_wait_ld();
                uint32_t v[32];
                #pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int lo = static_cast<int>(l0[j]) + static_cast<int>(h1[j]);
                    v[j] = __float_as_uint(fmaf(256.0f, static_cast<float>(static_cast<int>(h0[j])),
                                                static_cast<float>(lo)));
                }
                const int cnt = M - c0;
                if (splits > 1) {
                    // Partial tile of this rank: [BM activation rows][128 weight rows].
                    float* dst = part + (static_cast<size_t>(blockIdx.x) * BM + c0) * kTileN + row;
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) dst[j * kTileN] = __uint_as_float(v[j]);
                    continue;
                }
                // ((acc * mantissa_m) * scale[n]) * 2^e_m, row factors from shared memory.
                float o[32];
                #pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = ((__uint_as_float(v[j]) * rf_s[c0 + j]) * sc) * rf_s[BM + c0 + j];
                if (vec_out && n0 + quarter * 32 + 32 <= N) {
                    // [32 m][32 n] staging tile of this warp, out as float4 runs along n.
                    float* st = stage + quarter * 1024;
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) st[j * 32 + lane] = o[j];
                    __syncwarp();
                    const int q4 = lane & 7;
                    const int mr = lane >> 3;
                    #pragma unroll
                    for (int it = 0; it < 8; ++it) {
                        const int ml = it * 4 + mr;
                        if (ml < cnt) {
                            float* dst = out + static_cast<int64_t>(c0 + ml) * N + n0 + quarter * 32 + 4 * q4;
                            *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(st + ml * 32 + 4 * q4);
                        }
                    }
                    __syncwarp();
                } else if (n < N) {
                    float* base = out + static_cast<int64_t>(c0) * N + n;
                    if (epi) {
                        #pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (j < cnt) store_out(base + static_cast<int64_t>(j) * N, o[j], 1);
                        }
                    } else {
                        #pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (j < cnt) base[static_cast<int64_t>(j) * N] = o[j];
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (splits > 1) {
        // Every rank's partial is in global memory (release/acquire at
        // cluster scope orders the stores before the loads below).
        cluster_sync();
        if (warp >= kI8WarpEpi0) {
            const int et = threadIdx.x - kI8WarpEpi0 * 32;  // 0..127
            const int rows = kTileN / splits;
            const int mq = ((M < BM ? M : BM) + 3) / 4;
            const int tile = static_cast<int>(blockIdx.x) / splits;
            for (int unit = et; unit < rows * mq; unit += 128) {
                const int rl = rank * rows + unit % rows;  // weight row within the tile
                const int m = 4 * (unit / rows);
                float p4[8][4];
                #pragma unroll
                for (int p = 0; p < 8; ++p) {
                    if (p < splits) {
                        const float* src = part + (static_cast<size_t>(tile * splits + p) * BM + m) * kTileN + rl;
                        #pragma unroll
                        for (int k = 0; k < 4; ++k) p4[p][k] = __ldcg(src + k * kTileN);
                    }
                }
                const int nn = n0 + rl;
                if (nn < N) {
                    const float s_n = __ldg(scale + nn);
                    #pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        float acc = p4[0][k];
                        #pragma unroll
                        for (int p = 1; p < 8; ++p) {
                            if (p < splits) acc += p4[p][k];
                        }
                        if (m + k < M) {
                            store_out(out + static_cast<int64_t>(m + k) * N + nn,
                                      ((acc * __ldg(rowfactor + m + k)) * s_n) * __ldg(rowpow + m + k), epi);
                        }
                    }
                }
            }
        }
    }
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ------------------------------- int8 tensor path on CTA pairs (32 < M <= 128)
// The same arithmetic as tc_i8_kernel with tcgen05.mma.cta_group::2: a pair
// of CTAs (cluster of two) computes 256 weight rows. CTA r holds its own 128
// weight rows (the A operand is split by rows across the pair) and only
// digit plane r of the activation tile -- rank 0 the hi digits, rank 1 the
// lo digits -- as its half of the B operand, so the pair's N = 2 BM columns
// are hi then lo, exactly the single-CTA layout, and each CTA's tensor
// memory receives its 128 weight rows x 2 BM columns. Per 128-deep k-block
// a CTA loads 16 KB of weights and BM x 128 digit bytes instead of 2 BM x
// 128: at BM = 128 that is 32 KB instead of 48 KB per SM, the stream that
// bounds the single-CTA kernel when M = 128 (the MMAs of a k-block need
// ~540 cycles; 48 KB at the ~70 bytes per cycle an SM receives takes ~700).
// Used for 128-row activation tiles when the 128-row weight tiles already
// fill half the GPU (no split-K); instantiated for BM = 128 only.
//
// All four TMA loads of a stage (weights and digits of both CTAs) complete
// on the leader's full[s]; the leader alone posts the expected bytes and
// issues the MMAs; release[s], acc_full and drain are multicast commits to
// both CTAs. The first ring of weight tiles is requested before the
// dependent-launch wait (the prologue writes only the digit planes and row
// factors); the digit tiles and the epilogue's row factors come after it.
template <int BM>
struct CfgI8Pair {
    static constexpr int kBK = 128;
    static constexpr int kN = 2 * BM;                // pair MMA N: hi rows (rank 0), then lo rows (rank 1)
    static constexpr int kXBytes = BM * kBK;         // this CTA's digit plane tile per stage
    static constexpr int kWBytes = kTileN * kBK;     // this CTA's weight tile per stage
    static constexpr int kStages = 6;
    static constexpr int kAcc = 1;                   // one accumulator: each k-step is 128 x 256 x 32 per CTA
    static constexpr int kTmemCols = kAcc * kN;      // 256
    static constexpr int kNumBars = 2 * kStages + 2;
    static constexpr int kStageBytes = 4 * 32 * 32 * 4;
    static constexpr int kSmem = 1024 + kStages * (kXBytes + kWBytes) + kNumBars * 8 + 16 + 16 + kStageBytes + 2 * BM * 4;
    static_assert(kXBytes % 1024 == 0 && kWBytes % 1024 == 0, "stages stay 1024-byte aligned");
    static_assert(BM == 128 && kTmemCols == 256, "tensor-memory allocation");
    static_assert(kSmem <= 227 * 1024, "shared memory per block");
};

template <int BM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kI8Threads, 1)
tc_i8_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                  float* __restrict__ out, const float* __restrict__ scale, const float* __restrict__ rowfactor,
                  const float* __restrict__ rowpow, int M, int N, int K, int epi) {
    using C = CfgI8Pair<BM>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xs = smem;                                  // S x [BM][128] digits of plane `rank`, 128B swizzle
    uint8_t* ws = smem + S * C::kXBytes;                 // S x [128][128] weight codes, 128B swizzle
    uint64_t* bars = reinterpret_cast<uint64_t*>(ws + S * C::kWBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    float* stage = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tmem_slot + 4) + 15) & ~uintptr_t(15));
    float* rf_s = stage + C::kStageBytes / 4;            // row factors: [BM] mantissas, then [BM] powers

    // full[s] (leader): all four tiles of stage s landed. release[s] (both):
    // the MMAs reading stage s finished. acc_full, drain (both): multicast.
    const uint32_t full0 = smem_addr(bars);
    const uint32_t release0 = full0 + 8 * S;
    const uint32_t acc_full = release0 + 8 * S;
    const uint32_t drain = acc_full + 8;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int n0 = static_cast<int>(blockIdx.x >> 1) * (2 * kTileN) + static_cast<int>(rank) * kTileN;
    const int num_kb = (K + C::kBK - 1) / C::kBK;
    unsigned int* err = &g_tc_error;
    const bool vec_out = epi == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (N & 3) == 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(release0 + 8 * i, 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the leader's barriers exist before the peer's loads complete on them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // accumulator: hi at columns [0, BM), lo at [BM, 2 BM)

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full_leader0 = mapa_shared(full0, 0);
            constexpr uint32_t kStageTx = 2 * (C::kXBytes + C::kWBytes);
            const int first = num_kb < S ? num_kb : S;
            for (int kb = 0; kb < first; ++kb) {
                if (leader) mbar_arrive_expect_tx(full0 + 8 * kb, kStageTx);
                tma_load_2d_pair(smem_addr(ws + kb * C::kWBytes), &tmap_w, kb * C::kBK, n0, full_leader0 + 8 * kb);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");  // the digit planes come from the prologue
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % S;
                if (kb >= S) {
                    if (!mbar_wait_cluster(release0 + 8 * s, ((kb / S) - 1) & 1, err, 1u)) break;
                    if (leader) mbar_arrive_expect_tx(full0 + 8 * s, kStageTx);
                    tma_load_2d_pair(smem_addr(ws + s * C::kWBytes), &tmap_w, kb * C::kBK, n0, full_leader0 + 8 * s);
                }
                tma_load_2d_pair(smem_addr(xs + s * C::kXBytes), &tmap_x, kb * C::kBK, static_cast<int>(rank) * M,
                                 full_leader0 + 8 * s);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_i8_s32(2 * kTileN, C::kN);
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % S;
                if (!mbar_wait_cluster(full0 + 8 * s, (kb / S) & 1, err, 2u)) break;
                tc_fence_after();
                const uint64_t adesc = smem_desc_sw128_kmajor(smem_addr(ws + s * C::kWBytes));
                const uint64_t bdesc = smem_desc_sw128_kmajor(smem_addr(xs + s * C::kXBytes));
                #pragma unroll
                for (int j = 0; j < C::kBK / 32; ++j) {
                    // K step of 32 int8 = 32 bytes inside the 128-byte swizzle rows.
                    mma_i8_ss_pair(tmem + (j % C::kAcc) * C::kN, adesc + static_cast<uint64_t>(2 * j),
                                   bdesc + static_cast<uint64_t>(2 * j), idesc, (kb > 0 || j >= C::kAcc) ? 1u : 0u);
                }
                mma_commit_pair(release0 + 8 * s, 0x3);
            }
            mma_commit_pair(acc_full, 0x3);
            // Every MMA (and so every load it consumed) is finished before the
            // pair releases tensor or shared memory.
            mma_commit_pair(drain, 0x3);
        }
    } else {
        // Epilogue: lane = weight row n of this CTA, 32 activation rows per chunk.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int n = n0 + row;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const float sc = n < N ? __ldg(scale + n) : 0.0f;
        asm volatile("griddepcontrol.wait;" ::: "memory");  // row factors come from the prologue
        for (int i = threadIdx.x - kI8WarpEpi0 * 32; i < BM; i += 128) {
            rf_s[i] = i < M ? __ldg(rowfactor + i) : 0.0f;
            rf_s[BM + i] = i < M ? __ldg(rowpow + i) : 0.0f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool ok = mbar_wait_cluster(acc_full, 0, err, 32u) && num_kb > 0;
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            #pragma unroll 1
            for (int c0 = 0; c0 < BM; c0 += 32) {
                if (c0 >= M) break;
                // Exact int32 hi and lo digit sums of activation rows c0 .. c0 + 31.
                uint32_t h[32], l[32];
                tmem_ld_32x32b_x32(tmem + lane_addr + c0, h);
                tmem_ld_32x32b_x32(tmem + lane_addr + BM + c0, l);
                tmem_wait_ld();
                const int cnt = M - c0;
                // ((acc * mantissa_m) * scale[n]) * 2^e_m, acc = 256 hi + lo.
                float o[32];
                #pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float acc = fmaf(256.0f, static_cast<float>(static_cast<int>(h[j])),
                                           static_cast<float>(static_cast<int>(l[j])));
                    o[j] = ((acc * rf_s[c0 + j]) * sc) * rf_s[BM + c0 + j];
                }
                if (vec_out && n0 + quarter * 32 + 32 <= N) {
                    // [32 m][32 n] staging tile of this warp, out as float4 runs along n.
                    float* st = stage + quarter * 1024;
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) st[j * 32 + lane] = o[j];
                    __syncwarp();
                    const int q4 = lane & 7;
                    const int mr = lane >> 3;
                    #pragma unroll
                    for (int it = 0; it < 8; ++it) {
                        const int ml = it * 4 + mr;
                        if (ml < cnt) {
                            float* dst = out + static_cast<int64_t>(c0 + ml) * N + n0 + quarter * 32 + 4 * q4;
                            *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(st + ml * 32 + 4 * q4);
                        }
                    }
                    __syncwarp();
                } else if (n < N) {
                    float* base = out + static_cast<int64_t>(c0) * N + n;
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (j < cnt) store_out(base + static_cast<int64_t>(j) * N, o[j], epi);
                    }
                }
            }
        }
    }

    if (warp == 1 && lane == 0) mbar_wait_cluster(drain, 0, err, 128u);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem, C::kTmemCols);
    }
}

// ------------------------------------------------------------------ host side
constexpr int kMaxDevices = 64;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    return fn;
}

// Stream-ordered scratch for x16 + rowscale: a private pool per device that
// keeps its memory between calls (no trimming at synchronisation points).
std::mutex g_pool_mu;
cudaMemPool_t g_pool[kMaxDevices] = {};

cudaError_t scratch_pool(cudaMemPool_t* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_pool_mu);
    if (g_pool[dev] == nullptr) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool;
        e = cudaMemPoolCreate(&pool, &props);
        if (e != cudaSuccess) return e;
        uint64_t keep = UINT64_MAX;
        e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) return e;
        g_pool[dev] = pool;
    }
    *out = g_pool[dev];
    return cudaSuccess;
}

bool g_attr_set[kMaxDevices][24] = {};  // [device][launch slot + 8 * weight format]

// Cluster size for the split-K launch of a tile grid: the largest C in
// {8, 4, 2} that keeps every CTA resident at once (tiles * C clusters' worth
// of SMs, checked with the occupancy API) and leaves each rank >= 4 k-blocks;
// 1 when the tiles alone already fill half the GPU.
template <int BM, int FMT>
int pick_splits(int slot, int64_t tiles, int64_t num_kb) {
    using C = Cfg<BM, FMT>;
    static int cache[kMaxDevices][3][4] = {};  // [dev][slot][log2 C - 1]: 0 unknown, 1 no, 2 + clusters
    const int64_t sms = device_sm_count();
    if (tiles * 2 > sms) return 1;
    int dev = 0;
    cudaGetDevice(&dev);
    for (int c = 8; c >= 2; c >>= 1) {
        if (tiles * c > sms || num_kb < 4 * c) continue;
        const int li = c == 8 ? 2 : (c == 4 ? 1 : 0);
        int* known = (dev >= 0 && dev < kMaxDevices) ? &cache[dev][slot][li] : nullptr;
        int clusters = 0;
        if (known == nullptr || *known == 0) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(c));
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = C::kSmem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(c);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_kernel<BM, FMT>, &cfg) != cudaSuccess) {
                cudaGetLastError();
                clusters = 0;
            }
            if (known != nullptr) *known = clusters > 0 ? 2 + clusters : 1;
        } else {
            clusters = *known >= 2 ? *known - 2 : 0;
        }
        if (clusters >= tiles) return c;
    }
    return 1;
}

template <int BM, int FMT>
popcornStatus_t launch_gemm(int slot, const CUtensorMap& tx, const CUtensorMap& tw, float* out, const float* scale,
                            const float* rowscale, const float* zero, int gs, int64_t M, int64_t N, int64_t K,
                            int epi, cudaStream_t stream) {
    using C = Cfg<BM, FMT>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDevices && !g_attr_set[dev][slot + 8 * FMT]) {
        cudaError_t e =
            cudaFuncSetAttribute(tc_gemm_kernel<BM, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return record_cuda(e);
        g_attr_set[dev][slot + 8 * FMT] = true;
    }
    const int64_t tiles = ceil_div(N, kTileN);
    const int splits = pick_splits<BM, FMT>(slot, tiles, ceil_div(K, C::kBK));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles * splits));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BM, FMT>, tx, tw, out, scale, rowscale, zero, gs,
                                             static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), splits, epi);
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

int pick_bm(int64_t M) {
    if (M <= 32) return 32;
    if (M <= 64) return 64;
    if (M <= 128) return 128;
    return 256;
}

// Tensor maps of one call: x16 [M, K] f16 in [xrows x 64] boxes (128B
// swizzle), weight codes [N, wcols] bytes (wcols = K for int8, K / 2 for
// packed int4) in [128 x bk] boxes (bk = 64: 64B swizzle, bk = 128: 128B
// swizzle).
bool make_maps(PFN_cuTensorMapEncodeTiled_v12000 encode, __half* x16, const void* q, int64_t M, int64_t N,
               int64_t K, int64_t wcols, int xrows, int bk, CUtensorMap* tx, CUtensorMap* tw) {
    const int bm = xrows;
    const cuuint64_t xdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t xstride[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t xbox[2] = {64, static_cast<cuuint32_t>(bm)};
    const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(wcols), static_cast<cuuint64_t>(N)};
    const cuuint64_t wstride[1] = {static_cast<cuuint64_t>(wcols)};
    const cuuint32_t wbox[2] = {static_cast<cuuint32_t>(bk), kTileN};
    const cuuint32_t estride[2] = {1, 1};
    CUresult r1 = encode(tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, xdims, xstride, xbox, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = encode(tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), wdims, wstride, wbox, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r1 == CUDA_SUCCESS && r2 == CUDA_SUCCESS;
}

template <int RX, int FMT>
popcornStatus_t launch_pair(int slot, const CUtensorMap& tx, const CUtensorMap& tw, float* out, const float* scale,
                            const float* rowscale, const float* zero, int gs, int64_t M, int64_t N, int64_t K,
                            int epi, cudaStream_t stream) {
    using P = PairCfg<RX, FMT>;
    int dev = 0;
    cudaGetDevice(&dev);
    const bool known = dev >= 0 && dev < kMaxDevices;
    // Both pair kernels take the same shared memory (attribute set once each).
    static bool persist_attr[kMaxDevices][24] = {};
    if (known && !g_attr_set[dev][slot + 8 * FMT]) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_pair_kernel<RX, FMT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, P::kSmem);
        if (e == cudaSuccess && !persist_attr[dev][slot + 8 * FMT]) {
            e = cudaFuncSetAttribute(tc_gemm_pair_persist_kernel<RX, FMT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, P::kSmem);
            persist_attr[dev][slot + 8 * FMT] = e == cudaSuccess;
        }
        if (e != cudaSuccess) return record_cuda(e);
        g_attr_set[dev][slot + 8 * FMT] = true;
    }
    // Pairs resident at once (occupancy query, cached per device and config).
    static int resident[kMaxDevices][4][3] = {};  // [dev][log2(RX / 16)][FMT]: pairs, 0 = unknown
    const int rxi = RX == 16 ? 0 : (RX == 32 ? 1 : (RX == 64 ? 2 : 3));
    int pairs = known ? resident[dev][rxi][FMT] : 0;
    if (pairs == 0) {
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(2);
        q.blockDim = dim3(kThreads);
        q.dynamicSmemBytes = P::kSmem;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_pair_persist_kernel<RX, FMT>, &q) != cudaSuccess ||
            clusters < 1) {
            cudaGetLastError();
            clusters = device_sm_count() / 2;
        }
        pairs = clusters;
        if (known) resident[dev][rxi][FMT] = pairs;
    }
    const int64_t tiles_n = ceil_div(N, 2 * kTileN);
    const int64_t tiles_m = ceil_div(M, 2 * RX);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = P::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (tiles_n * tiles_m > pairs) {
        // More tiles than resident pairs: persistent pairs, so the next tile's
        // loads and conversions overlap the previous tile's epilogue.
        cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
        e = cudaLaunchKernelEx(&cfg, tc_gemm_pair_persist_kernel<RX, FMT>, tx, tw, out, scale, rowscale, zero, gs,
                               static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), epi);
    } else {
        cfg.gridDim = dim3(static_cast<unsigned>(2 * tiles_n), static_cast<unsigned>(tiles_m));
        e = cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<RX, FMT>, tx, tw, out, scale, rowscale, zero, gs,
                               static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), epi);
    }
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

// The GEMM launch of the tensor path once x16 and rowscale are in place:
// CTA pairs (256 x 256 tiles) for M > 128, single CTAs with BM activation
// rows otherwise.
template <int FMT>
popcornStatus_t launch_tc_gemm(PFN_cuTensorMapEncodeTiled_v12000 encode, __half* x16, const float* rowscale,
                               float* out, const void* q, const float* scale, const float* zero, int gs, int64_t M,
                               int64_t N, int64_t K, int epi, cudaStream_t stream) {
    const int bm = pick_bm(M);
    const int64_t wcols = FMT == kFmtGroup4 ? K / 2 : K;
    const int bk = FMT == kFmtGroup4 ? 64 : 128;
    CUtensorMap tx, tw;
    // CTA pairs: always for M > 128; for smaller M when there are more
    // 128-row weight tiles than half the SMs (the single-CTA kernel with
    // cluster split-K serves the rest).
    if (bm >= 256 || ceil_div(N, kTileN) * 2 > device_sm_count()) {
        const int rx = bm / 2;
        if (!make_maps(encode, x16, q, M, N, K, wcols, rx, bk, &tx, &tw)) return POPCORN_ERROR_INVALID_VALUE;
        switch (rx) {
            case 16: return launch_pair<16, FMT>(4, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
            case 32: return launch_pair<32, FMT>(5, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
            case 64: return launch_pair<64, FMT>(6, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
            default: return launch_pair<128, FMT>(7, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
        }
    }
    if (!make_maps(encode, x16, q, M, N, K, wcols, bm, bk, &tx, &tw)) return POPCORN_ERROR_INVALID_VALUE;
    switch (bm) {
        case 32: return launch_gemm<32, FMT>(0, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
        case 64: return launch_gemm<64, FMT>(1, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
        default: return launch_gemm<128, FMT>(2, tx, tw, out, scale, rowscale, zero, gs, M, N, K, epi, stream);
    }
}

// ---------------------------------------------------- int8 path, host side
bool g_i8_attr_set[kMaxDevices][3] = {};

template <int BM>
int i8_slot() {
    return BM == 32 ? 0 : (BM == 64 ? 1 : 2);
}

template <int BM>
popcornStatus_t i8_set_attr() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDevices && !g_i8_attr_set[dev][i8_slot<BM>()]) {
        const cudaError_t e =
            cudaFuncSetAttribute(tc_i8_kernel<BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, CfgI8<BM>::kSmem);
        if (e != cudaSuccess) return record_cuda(e);
        g_i8_attr_set[dev][i8_slot<BM>()] = true;
    }
    return POPCORN_SUCCESS;
}

// Cluster size for the int8 path's split-K: the largest C in {8, 4, 2}
// that keeps every CTA of the grid resident at once and leaves each rank
// >= 4 k-blocks; 1 when the tiles alone fill half the GPU.
template <int BM>
int pick_splits_i8(int64_t tiles, int64_t num_kb) {
    using C = CfgI8<BM>;
    static int cache[kMaxDevices][3][3] = {};  // [dev][slot][log2 C - 1]: 0 unknown, 1 no, 2 + clusters
    const int64_t sms = device_sm_count();
    if (tiles * 2 > sms) return 1;
    // The occupancy query needs the kernel's shared-memory size allowed first
    // (without it the query fails and "no split" would be cached for good).
    if (i8_set_attr<BM>() != POPCORN_SUCCESS) return 1;
    int dev = 0;
    cudaGetDevice(&dev);
    for (int c = 8; c >= 2; c >>= 1) {
        if (tiles * c > sms || num_kb < 4 * c) continue;
        const int li = c == 8 ? 2 : (c == 4 ? 1 : 0);
        int* known = (dev >= 0 && dev < kMaxDevices) ? &cache[dev][i8_slot<BM>()][li] : nullptr;
        int clusters = 0;
        if (known == nullptr || *known == 0) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(c));
            cfg.blockDim = dim3(kI8Threads);
            cfg.dynamicSmemBytes = C::kSmem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(c);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&clusters, tc_i8_kernel<BM>, &cfg) != cudaSuccess) {
                cudaGetLastError();
                clusters = 0;
            }
            if (known != nullptr) *known = clusters > 0 ? 2 + clusters : 1;
        } else {
            clusters = *known >= 2 ? *known - 2 : 0;
        }
        if (clusters >= tiles) return c;
    }
    return 1;
}

// The pair form of the int8 GEMM: 256 weight rows per cluster of two CTAs.
template <int BM>
popcornStatus_t launch_i8_pair(const CUtensorMap& tx, const CUtensorMap& tw, float* out, const float* scale,
                               const float* rowfactor, const float* rowpow, int64_t M, int64_t N, int64_t K, int epi,
                               cudaStream_t stream) {
    using C = CfgI8Pair<BM>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool known = dev >= 0 && dev < kMaxDevices;
    if (!known || !attr_set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(tc_i8_pair_kernel<BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return record_cuda(e);
        if (known) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * ceil_div(N, 2 * kTileN)));
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, tc_i8_pair_kernel<BM>, tx, tw, out, scale, rowfactor, rowpow,
                                             static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), epi);
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

template <int BM>
popcornStatus_t launch_i8(PFN_cuTensorMapEncodeTiled_v12000 encode, const int8_t* xd, const float* rowfactor,
                          const float* rowpow, float* part, int splits, float* out, const void* q,
                          const float* scale, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t stream) {
    using C = CfgI8<BM>;
    popcornStatus_t st = i8_set_attr<BM>();
    if (st != POPCORN_SUCCESS) return st;
    // Digit planes xd [2 M, K] in [BM x 128] boxes; weight codes [N, K] in
    // [128 x 128] boxes; both 128-byte swizzled, zero fill past the edges.
    CUtensorMap tx, tw;
    const cuuint64_t xdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(2 * M)};
    const cuuint64_t xstride[1] = {static_cast<cuuint64_t>(K)};
    const cuuint32_t xbox[2] = {static_cast<cuuint32_t>(C::kBK), static_cast<cuuint32_t>(BM)};
    const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
    const cuuint64_t wstride[1] = {static_cast<cuuint64_t>(K)};
    const cuuint32_t wbox[2] = {static_cast<cuuint32_t>(C::kBK), kTileN};
    const cuuint32_t estride[2] = {1, 1};
    if (encode(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(xd), xdims, xstride, xbox, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), wdims, wstride, wbox, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    const int64_t tiles = ceil_div(N, kTileN);
    if constexpr (BM == 128) {
        // Tiles that fill half the GPU without split-K: CTA pairs (measured
        // ~10 % faster at M = 128; at 64-row tiles the pair's fixed cost
        // outweighs the smaller stream, so those keep single CTAs).
        if (splits == 1) return launch_i8_pair<BM>(tx, tw, out, scale, rowfactor, rowpow, M, N, K, epi, stream);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles * splits));
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, tc_i8_kernel<BM>, tx, tw, out, scale, rowfactor, rowpow, part,
                                             static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), splits,
                                             epi);
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

// The int8 path applies to per-channel weights with 4 < M <= 128 and
// K <= 65536 (int32 sums cannot wrap).
bool i8_path(int64_t M, int64_t K) { return M <= 128 && K <= 65536; }

template <int BM>
int i8_splits(int64_t N, int64_t K) {
    return pick_splits_i8<BM>(ceil_div(N, kTileN), ceil_div(K, CfgI8<BM>::kBK));
}

// Launch plan of one int8-path call: activation tile height, split-K
// cluster size and the scratch it needs -- digit planes [2, M, K] int8, row
// mantissas and powers [M] f32 each, split-K partials [tiles * splits][BM][128]
// f32 -- each region 256-byte aligned.
struct I8Plan {
    int bm;
    int splits;
    size_t xd_bytes;
    size_t rf_bytes;
    size_t part_bytes;
    size_t total() const { return xd_bytes + 2 * rf_bytes + part_bytes; }
};

I8Plan i8_plan(int64_t M, int64_t N, int64_t K) {
    I8Plan p;
    p.bm = pick_bm(M);
    p.splits = p.bm == 32 ? i8_splits<32>(N, K) : (p.bm == 64 ? i8_splits<64>(N, K) : i8_splits<128>(N, K));
    p.xd_bytes = (static_cast<size_t>(2 * M) * K + 255) & ~size_t(255);
    p.rf_bytes = (static_cast<size_t>(M) * 4 + 255) & ~size_t(255);
    p.part_bytes =
        p.splits > 1 ? static_cast<size_t>(ceil_div(N, kTileN)) * p.splits * p.bm * kTileN * sizeof(float) : 0;
    return p;
}

// Digit prologue, then the GEMM (and, with q_up, the up-projection GEMM whose
// epilogue multiplies by silu of the first result), with the plan's scratch
// regions at xd, rowfactor, rowpow and part.
popcornStatus_t i8_launch_all(const I8Plan& p, PFN_cuTensorMapEncodeTiled_v12000 encode, int8_t* xd,
                              float* rowfactor, float* rowpow, float* part, float* out, const float* x,
                              const int8_t* q, const float* scale, int64_t M, int64_t N, int64_t K,
                              cudaStream_t stream, RowNorm nrm, const int8_t* q_up, const float* s_up) {
    auto gemm = [&](const int8_t* qq, const float* ss, int epi) {
        if (p.bm == 32) {
            return launch_i8<32>(encode, xd, rowfactor, rowpow, part, p.splits, out, qq, ss, M, N, K, epi, stream);
        }
        if (p.bm == 64) {
            return launch_i8<64>(encode, xd, rowfactor, rowpow, part, p.splits, out, qq, ss, M, N, K, epi, stream);
        }
        return launch_i8<128>(encode, xd, rowfactor, rowpow, part, p.splits, out, qq, ss, M, N, K, epi, stream);
    };
    popcornStatus_t st = launch_x_to_i8(xd, rowfactor, rowpow, x, M, K, stream, nrm);
    if (st == POPCORN_SUCCESS) st = gemm(q, scale, 0);
    if (st == POPCORN_SUCCESS && q_up != nullptr) st = gemm(q_up, s_up, 1);
    return st;
}

// The int8 path with its scratch from the stream-ordered pool.
popcornStatus_t tc_run_i8(float* out, const float* x, const int8_t* q, const float* scale, int64_t M, int64_t N,
                          int64_t K, cudaStream_t stream, RowNorm nrm, const int8_t* q_up, const float* s_up) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
    if (encode == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    const I8Plan p = i8_plan(M, N, K);
    cudaMemPool_t pool;
    cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return record_cuda(e);
    void* scratch = nullptr;
    e = cudaMallocFromPoolAsync(&scratch, p.total(), pool, stream);
    if (e != cudaSuccess) return record_cuda(e);
    uint8_t* base = static_cast<uint8_t*>(scratch);
    popcornStatus_t st = i8_launch_all(
        p, encode, reinterpret_cast<int8_t*>(base), reinterpret_cast<float*>(base + p.xd_bytes),
        reinterpret_cast<float*>(base + p.xd_bytes + p.rf_bytes),
        p.splits > 1 ? reinterpret_cast<float*>(base + p.xd_bytes + 2 * p.rf_bytes) : nullptr, out, x, q, scale, M,
        N, K, stream, nrm, q_up, s_up);
    e = cudaFreeAsync(scratch, stream);
    if (st == POPCORN_SUCCESS && e != cudaSuccess) st = record_cuda(e);
    return st;
}

// x -> f16 prologue into stream-ordered scratch, then the GEMM.
// x -> f16 prologue (with the optional RMSNorm), then the GEMM; with q_up a
// second GEMM over the same activations whose epilogue multiplies by
// silu of the first one's result (gate/up fusion).
template <int FMT>
popcornStatus_t tc_run(float* out, const float* x, const void* q, const float* scale, const float* zero, int gs,
                       int64_t M, int64_t N, int64_t K, cudaStream_t stream, RowNorm nrm = RowNorm{nullptr, 0.0f, 0},
                       const void* q_up = nullptr, const float* s_up = nullptr) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
    if (encode == nullptr) return POPCORN_ERROR_INVALID_VALUE;

    // Scratch: x16 [M, K] f16, then rowscale [M] f32, each 256-byte aligned.
    const size_t x16_bytes = (static_cast<size_t>(M) * K * 2 + 255) & ~size_t(255);
    const size_t bytes = x16_bytes + ((static_cast<size_t>(M) * 4 + 255) & ~size_t(255));
    cudaMemPool_t pool;
    cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return record_cuda(e);
    void* scratch = nullptr;
    e = cudaMallocFromPoolAsync(&scratch, bytes, pool, stream);
    if (e != cudaSuccess) return record_cuda(e);
    __half* x16 = static_cast<__half*>(scratch);
    float* rowscale = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + x16_bytes);

    popcornStatus_t st = launch_x_to_f16(x16, rowscale, x, M, K, stream, nrm);
    if (st == POPCORN_SUCCESS) {
        st = launch_tc_gemm<FMT>(encode, x16, rowscale, out, q, scale, zero, gs, M, N, K, 0, stream);
    }
    if (st == POPCORN_SUCCESS && q_up != nullptr) {
        st = launch_tc_gemm<FMT>(encode, x16, rowscale, out, q_up, s_up, zero, gs, M, N, K, 1, stream);
    }
    e = cudaFreeAsync(scratch, stream);
    if (st == POPCORN_SUCCESS && e != cudaSuccess) st = record_cuda(e);
    return st;
}

}  // namespace

bool tc_supported(const float*, const int8_t* q, int64_t M, int64_t N, int64_t K) {
    // TMA: 16-byte aligned weight base and row pitch; int32 tile coordinates.
    return (K % 16 == 0) && aligned16(q) && M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX &&
           M * K <= (int64_t(1) << 40) && encode_fn() != nullptr;
}

int tc_launch_count(int64_t, int64_t, int64_t) { return 2; }

popcornStatus_t tc_dequant_matmul(float* out, const float* x, const int8_t* q, const float* scale, int64_t M,
                                  int64_t N, int64_t K, cudaStream_t stream) {
    if (i8_path(M, K)) return tc_run_i8(out, x, q, scale, M, N, K, stream, RowNorm{nullptr, 0.0f, 0}, nullptr, nullptr);
    return tc_run<kFmtChannel>(out, x, q, scale, nullptr, 0, M, N, K, stream);
}

cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t stream) {
    cudaMemPool_t pool;
    const cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    return cudaMallocFromPoolAsync(p, bytes, pool, stream);
}

cudaError_t scratch_free(void* p, cudaStream_t stream) { return cudaFreeAsync(p, stream); }

popcornStatus_t tc_dequant_matmul_fused(float* out, const float* x, const float* norm_w, float eps, bool norm,
                                        const int8_t* q, const float* scale, const int8_t* q_up, const float* s_up,
                                        int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    const RowNorm nrm{norm_w, eps, norm ? 1 : 0};
    if (i8_path(M, K)) return tc_run_i8(out, x, q, scale, M, N, K, stream, nrm, q_up, s_up);
    return tc_run<kFmtChannel>(out, x, q, scale, nullptr, 0, M, N, K, stream, nrm, q_up, s_up);
}

bool tc_grouped_supported(const void* q, int64_t M, int64_t N, int64_t K, int64_t gs) {
    // Group factors are taken per 32 codes; 16-byte aligned base and row
    // pitch for TMA (K % 32 == 0 follows from gs % 32 == 0 and gs | K).
    return gs % 32 == 0 && K % gs == 0 && aligned16(q) && M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX &&
           M * K <= (int64_t(1) << 40) && encode_fn() != nullptr;
}

popcornStatus_t tc_dequant_matmul_grouped(WeightFormat fmt, float* out, const float* x, const void* q,
                                          const float* scale, const float* zero, int64_t M, int64_t N, int64_t K,
                                          int64_t gs, cudaStream_t stream) {
    if (fmt == kFmtGroup4) {
        return tc_run<kFmtGroup4>(out, x, q, scale, zero, static_cast<int>(gs), M, N, K, stream);
    }
    return tc_run<kFmtGroup8>(out, x, q, scale, nullptr, static_cast<int>(gs), M, N, K, stream);
}

}  // namespace pcb

// ---------------------------------------------------------------------------
// Allocation-free variant of the tensor path.
//
// Some callers cannot let a library allocate device memory: a process whose
// GPU memory is carved up once at start-up by its own allocator (a Go/cgo
// service that accounts for every byte, or an inference server that reserves
// almost all of HBM for its KV cache), or a real-time loop that forbids any
// allocation after initialisation so it can never fail or stall mid-run. For
// them, popcornDequantizeMatmulNoAlloc_i8f32 runs the same kernels as the
// tensor path with its scratch in the fixed array below instead of the pool.
//
// The array is a file-scope device variable: every GPU that loads this
// library holds it (26 MiB + 64 KiB) until the process exits. In host code
// its name is only a host-side stand-in, not a device address, so the entry
// point looks up the real address with cudaGetSymbolAddress once per device
// (with that device current) and passes that pointer to the kernels.
// ---------------------------------------------------------------------------
namespace pcb {
namespace {

constexpr size_t kNoAllocX16Bytes = size_t(16) << 20;   // f16 activations, or int8 digit planes
constexpr size_t kNoAllocRowBytes = size_t(64) << 10;   // f32 row scales (row mantissas and powers)
constexpr size_t kNoAllocPartBytes = size_t(10) << 20;  // split-K partials of the int8 path

static __device__ __align__(256) unsigned char
    g_noalloc_scratch[kNoAllocX16Bytes + kNoAllocRowBytes + kNoAllocPartBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up on
// the first call per device, cached after).
cudaError_t noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace pcb

extern "C" popcornStatus_t popcornDequantizeMatmulNoAlloc_i8f32(float* out, const float* x, const int8_t* qweight,
                                                               const float* scale, int64_t M, int64_t N, int64_t K,
                                                               cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (!tc_supported(x, qweight, M, N, K)) return POPCORN_ERROR_INVALID_VALUE;
    if (M > static_cast<int64_t>(kNoAllocRowBytes / 4) || K > static_cast<int64_t>(kNoAllocX16Bytes / 2)) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    const size_t x16_bytes = (static_cast<size_t>(M) * K * 2 + 255) & ~size_t(255);
    if (x16_bytes > kNoAllocX16Bytes) return POPCORN_ERROR_INVALID_VALUE;
    PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
    if (encode == nullptr) return POPCORN_ERROR_INVALID_VALUE;

    void* scratch = nullptr;
    cudaError_t e = noalloc_scratch(&scratch);
    if (e != cudaSuccess) return record_cuda(e);
    __half* x16 = static_cast<__half*>(scratch);
    float* rowscale = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kNoAllocX16Bytes);

    // The prologue writes every activation element and row scale the GEMM
    // reads (tile edges past M or K are zero-filled by TMA, not read from the
    // array), and every split-K partial is written before it is read, so
    // nothing left in the array by an earlier call needs clearing.
    if (i8_path(M, K)) {
        const I8Plan p = i8_plan(M, N, K);
        if (p.xd_bytes > kNoAllocX16Bytes || 2 * p.rf_bytes > kNoAllocRowBytes || p.part_bytes > kNoAllocPartBytes) {
            return POPCORN_ERROR_INVALID_VALUE;
        }
        uint8_t* base = static_cast<uint8_t*>(scratch);
        float* rows = reinterpret_cast<float*>(base + kNoAllocX16Bytes);
        return i8_launch_all(p, encode, reinterpret_cast<int8_t*>(base), rows,
                             reinterpret_cast<float*>(base + kNoAllocX16Bytes + p.rf_bytes),
                             reinterpret_cast<float*>(base + kNoAllocX16Bytes + kNoAllocRowBytes), out, x, qweight,
                             scale, M, N, K, stream, RowNorm{nullptr, 0.0f, 0}, nullptr, nullptr);
    }
    popcornStatus_t st = launch_x_to_f16(x16, rowscale, x, M, K, stream);
    if (st != POPCORN_SUCCESS) return st;

    return launch_tc_gemm<kFmtChannel>(encode, x16, rowscale, out, qweight, scale, nullptr, 0, M, N, K, 0, stream);
}

namespace pcb {
cudaError_t tc_take_errors(unsigned int* bits) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(bits, g_tc_error, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(unsigned int));
    return e;
}
}  // namespace pcb
