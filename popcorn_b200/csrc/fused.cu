// Fused neighbours of the per-channel dequant-matmul in a transformer block:
//   popcornRMSNormDequantizeMatmul_i8f32        RMSNorm(x) @ W^T
//   popcornDequantizeMatmulSiluMul_i8f32        silu(x @ Wg^T) * (x @ Wu^T)
//   popcornRMSNormDequantizeMatmulSiluMul_i8f32 both
// They replace the popcorn call sequences RMSNorm (src/reduction.cu:290-321)
// -> DequantizeMatmul (src/quantize.cu:18-112) -> Silu (src/unary.cu:76-81)
// -> Mul (src/binary.cu:89-95) with one pass over the activations and no
// intermediate tensors.
//
// Paths:
//  * fused_xs_kernel<MT, U, R, NORM, GLU> (M <= 4): the x-stationary decode
//    layout of the f32 GEMV; a block spans all of K, so it forms the row's sum
//    of squares itself (NORM) and normalises its x slices in registers; with
//    GLU it streams R rows of both weight matrices and writes silu(g) * u.
//    At M = 1 the dot products are exact dp2a sums on 30-bit fixed-point
//    slices, as in the per-channel decode GEMV.
//  * tensor cores (M > 4, >= 2^27 multiply-adds): the RMSNorm runs inside the
//    x -> f16 prologue; the gate GEMM writes g to `out` and the up GEMM's
//    epilogue turns it into silu(g) * u (tc_gemm.cu).
//  * anything else runs the unfused sequence with this library's kernels and
//    stream-ordered scratch.
#include "common.cuh"

namespace pcb {
namespace {

constexpr int kFThreads = 256;
constexpr int kFWarps = kFThreads / 32;

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// dp2a with unsigned 16-bit halves in the first operand (low or high pair
// of signed bytes in the second).
__device__ __forceinline__ int dp2a_lo_u(uint32_t a, int b, int c) {
    int d;
    asm("dp2a.lo.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_u(uint32_t a, int b, int c) {
    int d;
    asm("dp2a.hi.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Four int8 codes (one word) -> four exact floats (byte ^ 0x80 in the low
// mantissa byte of 2^23 is 2^23 + 128 + code).
__device__ __forceinline__ void widen4f(uint32_t word, float2& lo, float2& hi) {
    const uint32_t b = word ^ 0x80808080u;
    const float2 magic = make_float2(-8388736.0f, -8388736.0f);
    const float2 a = make_float2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440)),
                                 __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7441)));
    const float2 c = make_float2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7442)),
                                 __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7443)));
    lo = __fadd2_rn(a, magic);
    hi = __fadd2_rn(c, magic);
}

// Butterfly reduce-scatter of V values over a warp: afterwards the lanes with
// (lane % (32 / V)) == 0 hold the warp total of value lane / (32 / V).
template <int V>
__device__ __forceinline__ float fused_reduce_scatter(float (&v)[V], int lane) {
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

// MT activation rows (<= 4), U 16-element K slices per thread, R weight rows
// per block (of each matrix); gridDim.y = ceil(M / MT). NORM: RMSNorm the
// activation rows first. GLU: second matrix (qb, sb), out = silu(g) * u.
template <int MT, int U, int R, bool NORM, bool GLU>
__global__ void __launch_bounds__(kFThreads, (MT == 1 && U == 1 && R * (GLU ? 2 : 1) <= 8) ? 4 : 2)
fused_xs_kernel(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ nw, float eps,
                const int8_t* __restrict__ qa, const float* __restrict__ sa, const int8_t* __restrict__ qb,
                const float* __restrict__ sb, int64_t M, int64_t N, int64_t K) {
    constexpr int NM = GLU ? 2 : 1;  // weight matrices
    constexpr int V = NM * R * MT;   // partial sums per thread
    __shared__ float part[V][kFWarps];
    __shared__ float ssq[MT][kFWarps];
    __shared__ float fin[V];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t units = K >> 4;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * R;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * MT;

    // Programmatic dependent launch: release the next kernel, pull this
    // block's weight rows into L2 while the previous kernel finishes.
    pdl_launch_dependents();
    if (tid < NM * kFWarps && blockIdx.y == 0) {
        const int64_t rows = (r0 + R <= N) ? R : N - r0;
        prefetch_l2_range((tid < kFWarps ? qa : qb) + r0 * K, rows * K, tid % kFWarps, kFWarps);
    }
    pdl_wait();

    uint4 w[NM][R][U];
    #pragma unroll
    for (int mat = 0; mat < NM; ++mat) {
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kFThreads;
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                const int8_t* qm = mat == 0 ? qa : qb;
                w[mat][r][u] = (r0 + r < N && unit < units)
                                   ? __ldg(reinterpret_cast<const uint4*>(qm + (r0 + r) * K) + unit)
                                   : make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
    float4 xr[MT][U][4];
    #pragma unroll
    for (int m = 0; m < MT; ++m) {
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kFThreads;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                xr[m][u][c] = (unit < units && m0 + m < M)
                                  ? __ldg(reinterpret_cast<const float4*>(x + (m0 + m) * K + unit * 16) + c)
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
    }

    if constexpr (NORM) {
        // The block holds every column of its activation rows: sum of squares
        // per row, then x * (1 / rms) * weight in popcorn's order.
        #pragma unroll
        for (int m = 0; m < MT; ++m) {
            float ss = 0.0f;
            #pragma unroll
            for (int u = 0; u < U; ++u)
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 v = xr[m][u][c];
                    ss = fmaf(v.x, v.x, ss);
                    ss = fmaf(v.y, v.y, ss);
                    ss = fmaf(v.z, v.z, ss);
                    ss = fmaf(v.w, v.w, ss);
                }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            if (lane == 0) ssq[m][warp] = ss;
        }
        __syncthreads();
        #pragma unroll
        for (int m = 0; m < MT; ++m) {
            float total = 0.0f;
            #pragma unroll
            for (int wv = 0; wv < kFWarps; ++wv) total += ssq[m][wv];
            const float inv = 1.0f / sqrtf(total / static_cast<float>(K) + eps);
            #pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t unit = tid + static_cast<int64_t>(u) * kFThreads;
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float4 v = xr[m][u][c];
                    v.x *= inv;
                    v.y *= inv;
                    v.z *= inv;
                    v.w *= inv;
                    if (nw != nullptr && unit < units) {
                        const float4 g = __ldg(reinterpret_cast<const float4*>(nw) + unit * 4 + c);
                        v.x *= g.x;
                        v.y *= g.y;
                        v.z *= g.z;
                        v.w *= g.w;
                    }
                    xr[m][u][c] = v;
                }
            }
        }
    }

    float acc[V];
    #pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.0f;
    // M = 1: each thread's (normalised) slices as 30-bit fixed point from
    // the slices' max |x|, X = hi * 2^16 + lo, and exact dp2a products with
    // the codes (the per-channel decode GEMV's arithmetic); a warp holding a
    // non-finite value or a max |x| outside [2^-90, 2^100] keeps the float
    // path below.
    bool fixed = false;
    float up = 1.0f, down = 1.0f;
    if constexpr (MT == 1) {
        uint32_t mb = 0;
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 v = xr[0][u][c];
                mb = max(mb, max(max(__float_as_uint(v.x) & 0x7FFFFFFFu, __float_as_uint(v.y) & 0x7FFFFFFFu),
                                 max(__float_as_uint(v.z) & 0x7FFFFFFFu, __float_as_uint(v.w) & 0x7FFFFFFFu)));
            }
        }
        const bool bad = mb != 0u && (mb < 0x12800000u || mb > 0x71800000u);
        fixed = !__any_sync(0xffffffffu, bad);
        if (fixed && mb != 0u) {
            const int ex = 156 - static_cast<int>(mb >> 23);  // max |x| * 2^ex in [2^29, 2^30)
            up = __int_as_float((ex + 127) << 23);
            down = __int_as_float((127 - ex) << 23);
        }
    }
    if (MT == 1 && fixed) {
        uint32_t xh[U][8], xl[U][8];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 v = xr[0][u][c];
                const uint32_t a0 = static_cast<uint32_t>(__float2int_rn(v.x * up));
                const uint32_t a1 = static_cast<uint32_t>(__float2int_rn(v.y * up));
                const uint32_t a2 = static_cast<uint32_t>(__float2int_rn(v.z * up));
                const uint32_t a3 = static_cast<uint32_t>(__float2int_rn(v.w * up));
                xl[u][2 * c] = __byte_perm(a0, a1, 0x5410);
                xh[u][2 * c] = __byte_perm(a0, a1, 0x7632);
                xl[u][2 * c + 1] = __byte_perm(a2, a3, 0x5410);
                xh[u][2 * c + 1] = __byte_perm(a2, a3, 0x7632);
            }
        }
        #pragma unroll
        for (int mat = 0; mat < NM; ++mat) {
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                int sh = 0, sl = 0;
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int words[4] = {static_cast<int>(w[mat][r][u].x), static_cast<int>(w[mat][r][u].y),
                                          static_cast<int>(w[mat][r][u].z), static_cast<int>(w[mat][r][u].w)};
                    #pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        sh = __dp2a_lo(static_cast<int>(xh[u][2 * c]), words[c], sh);
                        sh = __dp2a_hi(static_cast<int>(xh[u][2 * c + 1]), words[c], sh);
                        sl = dp2a_lo_u(xl[u][2 * c], words[c], sl);
                        sl = dp2a_hi_u(xl[u][2 * c + 1], words[c], sl);
                    }
                }
                acc[mat * R + r] = fmaf(static_cast<float>(sh), 65536.0f, static_cast<float>(sl)) * down;
            }
        }
    } else {
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        #pragma unroll
        for (int mat = 0; mat < NM; ++mat) {
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint32_t words[4] = {w[mat][r][u].x, w[mat][r][u].y, w[mat][r][u].z, w[mat][r][u].w};
                float2 a[MT];
                #pragma unroll
                for (int m = 0; m < MT; ++m) a[m] = make_float2(0.0f, 0.0f);
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float2 lo, hi;
                    widen4f(words[c], lo, hi);
                    #pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const float4 v = xr[m][u][c];
                        a[m] = __ffma2_rn(make_float2(v.x, v.y), lo, a[m]);
                        a[m] = __ffma2_rn(make_float2(v.z, v.w), hi, a[m]);
                    }
                }
                #pragma unroll
                for (int m = 0; m < MT; ++m) acc[(mat * R + r) * MT + m] += a[m].x + a[m].y;
            }
        }
    }
    }
    const float total = fused_reduce_scatter<V>(acc, lane);
    constexpr int span = 32 / V;
    if ((lane % span) == 0) part[lane / span][warp] = total;
    __syncthreads();
    if (tid < V) {
        const int mat = tid / (R * MT);
        const int r = (tid / MT) % R;
        float s = 0.0f;
        #pragma unroll
        for (int wv = 0; wv < kFWarps; ++wv) s += part[tid][wv];
        fin[tid] = (r0 + r < N) ? s * __ldg((mat == 0 ? sa : sb) + r0 + r) : 0.0f;
    }
    __syncthreads();
    if (tid < R * MT) {
        const int r = tid / MT;
        const int m = tid % MT;
        if (r0 + r < N && m0 + m < M) {
            const float g = fin[tid];
            out[(m0 + m) * N + r0 + r] = GLU ? silu(g) * fin[R * MT + tid] : g;
        }
    }
}

// RMSNorm of each row (one warp per row), popcorn's arithmetic.
__global__ void __launch_bounds__(256)
rmsnorm_rows_kernel(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ nw, float eps,
                    int64_t M, int64_t K) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
         row += nwarps) {
        const float* r = x + row * K;
        float ss = 0.0f;
        for (int64_t k = lane; k < K; k += 32) ss = fmaf(__ldg(r + k), __ldg(r + k), ss);
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
        for (int64_t k = lane; k < K; k += 32) {
            float v = __ldg(r + k) * inv;
            if (nw != nullptr) v *= __ldg(nw + k);
            out[row * K + k] = v;
        }
    }
}

// out[i] = silu(out[i]) * u[i].
__global__ void __launch_bounds__(256) silu_mul_kernel(float* __restrict__ out, const float* __restrict__ u,
                                                       int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        out[i] = silu(out[i]) * u[i];
    }
}

template <int MT, int U, int R, bool NORM, bool GLU>
popcornStatus_t launch_fused_xs(float* out, const float* x, const float* nw, float eps, const int8_t* qa,
                                const float* sa, const int8_t* qb, const float* sb, int64_t M, int64_t N, int64_t K,
                                cudaStream_t stream) {
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(
        dim3(static_cast<unsigned>(ceil_div(N, R)), static_cast<unsigned>(ceil_div(M, MT))), dim3(kFThreads), 0,
        stream, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fused_xs_kernel<MT, U, R, NORM, GLU>, out, x, nw, eps, qa, sa, qb,
                                             sb, M, N, K);
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

// Decode layout for M <= 4 and one to four 4096-column slices per thread;
// returns false (nothing launched) when no variant fits.
template <bool NORM, bool GLU>
bool try_fused_decode(popcornStatus_t* st, float* out, const float* x, const float* nw, float eps, const int8_t* qa,
                      const float* sa, const int8_t* qb, const float* sb, int64_t M, int64_t N, int64_t K,
                      cudaStream_t stream) {
    const int64_t slices = ceil_div(K / 16, kFThreads);
    constexpr int R1 = GLU ? 4 : 8;  // rows per block of each matrix at one slice
    if (M == 1) {
        // One slice: 8 rows of each matrix per block (with GLU 16 rows, two
        // blocks per SM), so the block's x, norm weight and sum of squares
        // serve twice the rows: 22.9 -> 21.6 us at K = 4096, N = 11008.
        if (slices == 1) *st = launch_fused_xs<1, 1, 8, NORM, GLU>(out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else if (slices == 2) *st = launch_fused_xs<1, 2, R1 / 2, NORM, GLU>(out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else if (slices <= 4) *st = launch_fused_xs<1, 4, R1 / 4, NORM, GLU>(out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else return false;
        return true;
    }
    if (M == 2) {
        if (slices == 1) *st = launch_fused_xs<2, 1, R1, NORM, GLU>(out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else if (slices == 2) *st = launch_fused_xs<2, 2, R1 / 2, NORM, GLU>(out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else return false;
        return true;
    }
    if (M <= 4 && slices == 1) {
        *st = launch_fused_xs<4, 1, R1 / 2, NORM, GLU>(out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        return true;
    }
    return false;
}

// The unfused sequence with this library's kernels.
popcornStatus_t fused_sequence(float* out, const float* x, const float* nw, float eps, bool norm, const int8_t* qa,
                               const float* sa, const int8_t* qb, const float* sb, int64_t M, int64_t N, int64_t K,
                               cudaStream_t stream) {
    float* xn = nullptr;
    float* u = nullptr;
    cudaError_t e = cudaSuccess;
    popcornStatus_t st = POPCORN_SUCCESS;
    const float* xin = x;
    if (norm) {
        e = scratch_alloc(reinterpret_cast<void**>(&xn), sizeof(float) * static_cast<size_t>(M * K), stream);
        if (e != cudaSuccess) return record_cuda(e);
        int64_t blocks = ceil_div(M, 8);
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
        if (blocks > cap) blocks = cap;
        rmsnorm_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(xn, x, nw, eps, M, K);
        st = check_launch();
        xin = xn;
    }
    if (st == POPCORN_SUCCESS) st = popcornDequantizeMatmul_i8f32(out, xin, qa, sa, M, N, K, stream);
    if (st == POPCORN_SUCCESS && qb != nullptr) {
        e = scratch_alloc(reinterpret_cast<void**>(&u), sizeof(float) * static_cast<size_t>(M * N), stream);
        if (e != cudaSuccess) {
            st = record_cuda(e);
        } else {
            st = popcornDequantizeMatmul_i8f32(u, xin, qb, sb, M, N, K, stream);
            if (st == POPCORN_SUCCESS) {
                int64_t blocks = ceil_div(M * N, 256);
                const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
                if (blocks > cap) blocks = cap;
                silu_mul_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(out, u, M * N);
                st = check_launch();
            }
        }
    }
    if (u != nullptr) {
        e = scratch_free(u, stream);
        if (st == POPCORN_SUCCESS && e != cudaSuccess) st = record_cuda(e);
    }
    if (xn != nullptr) {
        e = scratch_free(xn, stream);
        if (st == POPCORN_SUCCESS && e != cudaSuccess) st = record_cuda(e);
    }
    return st;
}

popcornStatus_t fused_dispatch(float* out, const float* x, const float* nw, float eps, bool norm, const int8_t* qa,
                               const float* sa, const int8_t* qb, const float* sb, int64_t M, int64_t N, int64_t K,
                               cudaStream_t stream) {
    const bool glu = qb != nullptr;
    const bool aligned = aligned16(x) && aligned16(qa) && (!glu || aligned16(qb)) &&
                         (!norm || nw == nullptr || aligned16(nw)) && K % 16 == 0;
    const bool tiny = static_cast<double>(M) * static_cast<double>(N) * static_cast<double>(K) <= 4194304.0;
    if (M <= 4 && aligned && !tiny && ceil_div(N, 2) <= 0x7FFFFFFF) {
        popcornStatus_t st = POPCORN_SUCCESS;
        bool done;
        if (norm && glu) done = try_fused_decode<true, true>(&st, out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else if (norm) done = try_fused_decode<true, false>(&st, out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        else done = try_fused_decode<false, true>(&st, out, x, nw, eps, qa, sa, qb, sb, M, N, K, stream);
        if (done) return st;
    }
    if (M > 4 && static_cast<double>(M) * static_cast<double>(N) * static_cast<double>(K) >= 134217728.0 &&
        tc_supported(x, qa, M, N, K) && (!glu || tc_supported(x, qb, M, N, K))) {
        return tc_dequant_matmul_fused(out, x, nw, eps, norm, qa, sa, qb, sb, M, N, K, stream);
    }
    return fused_sequence(out, x, nw, eps, norm, qa, sa, qb, sb, M, N, K, stream);
}

}  // namespace
}  // namespace pcb

extern "C" popcornStatus_t popcornRMSNormDequantizeMatmul_i8f32(float* out, const float* x, const float* norm_weight,
                                                               float eps, const int8_t* qweight, const float* scale,
                                                               int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    return pcb::fused_dispatch(out, x, norm_weight, eps, true, qweight, scale, nullptr, nullptr, M, N, K, stream);
}

extern "C" popcornStatus_t popcornDequantizeMatmulSiluMul_i8f32(float* out, const float* x, const int8_t* q_gate,
                                                               const float* s_gate, const int8_t* q_up,
                                                               const float* s_up, int64_t M, int64_t N, int64_t K,
                                                               cudaStream_t stream) {
    if (out == nullptr || x == nullptr || q_gate == nullptr || s_gate == nullptr || q_up == nullptr ||
        s_up == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    return pcb::fused_dispatch(out, x, nullptr, 0.0f, false, q_gate, s_gate, q_up, s_up, M, N, K, stream);
}

extern "C" popcornStatus_t popcornRMSNormDequantizeMatmulSiluMul_i8f32(
    float* out, const float* x, const float* norm_weight, float eps, const int8_t* q_gate, const float* s_gate,
    const int8_t* q_up, const float* s_up, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    if (out == nullptr || x == nullptr || q_gate == nullptr || s_gate == nullptr || q_up == nullptr ||
        s_up == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    return pcb::fused_dispatch(out, x, norm_weight, eps, true, q_gate, s_gate, q_up, s_up, M, N, K, stream);
}
