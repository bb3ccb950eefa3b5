// Int4 packed asymmetric per-group: popcornDequantizeMatmulGrouped_i4f32 and
// popcornQuantizeGrouped_f32i4 (popcorn src/quantize.cu:329-446, :699-888).
//
// Format (popcorn): qweight is [N, K/2] bytes, two 4-bit codes per byte, the
// even k in the low nibble; scale and zero are [N, K/group_size] f32; the
// weight of (n, k) is (code - zero[n, g]) * scale[n, g], g = k / group_size.
// Quantization: per group min and max (NaN skipped), scale = (max - min) / 15
// (1 when 0), zero = -min / scale, code = clamp(rint(v / scale + zero), 0, 15).
//
// Kernels:
//  * i4_seq_kernel -- one thread per output walking k upward with
//    w = (code - zero) * scale and acc = fma(x, w, acc): popcorn's operation
//    sequence, bit-identical to its kernel. Used for small problems, group
//    sizes that are not a multiple of 16 and unaligned operands.
//  * i4_xs_kernel<MT, U, R> -- x-stationary decode layout: each thread keeps
//    U 16-element slices of x in registers and reads the matching 8 bytes of
//    R weight rows per slice. A slice lies inside one group, so the zero
//    point leaves the inner loop:
//        sum_k x_k (c_k - z) s = s * (sum_k x_k (c_k - 8) - (z - 8) sum_k x_k)
//    with c_k - 8 exact in f32 (centred codes keep the two terms small). The
//    codes become floats without a conversion instruction: a nibble placed in
//    the low mantissa bits of 2^23 reads as 2^23 + c; the high nibble is taken
//    in place (2^23 + 16 c) and its activation pre-scaled by 1/16, exactly.
//  * i4_mma_kernel -- decode (M = 1, K = 1024, 2048 or 4096, group size a
//    multiple of 64, of 128 at K = 4096): staged rows, codes unpacked to bytes and summed against
//    fixed-point digits of x with mma.sync (u8 x s8), the zero point applied
//    through the exact group sum of x.
//  * i4_quantize_kernel -- one warp per (row, group): min and max by shuffles,
//    ties between +0 and -0 broken the way popcorn's 256-thread block breaks
//    them, then (even group sizes) the packed codes of the group;
//    i4_pack_kernel packs bytes that straddle two groups (odd group sizes)
//    from the stored parameters. Codes, scales and zero points are
//    bit-identical to popcorn's kernels; no temporary buffer.
#include "common.cuh"
#include "mma_frag.cuh"
#include "sm100.cuh"

namespace pcb {

// Error bits of bounded waits in this file's kernels (read by
// popcornB200DeviceErrors).
__device__ unsigned int g_i4_error = 0;

namespace {

constexpr int kI4Threads = 256;
constexpr unsigned int kI4StageTimeoutBit = 0x400u;  // staged int4 rows did not land within 1 s
constexpr int kI4Warps = kI4Threads / 32;

// Butterfly reduce-scatter of V values over a warp: afterwards the lanes with
// (lane % (32 / V)) == 0 hold the warp total of value lane / (32 / V).
template <int V>
__device__ __forceinline__ float i4_reduce_scatter(float (&v)[V], int lane) {
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
i4_seq_kernel(float* __restrict__ out, const float* __restrict__ x, const uint8_t* __restrict__ q,
              const float* __restrict__ scale, const float* __restrict__ zero, int64_t M, int64_t N, int64_t K,
              int64_t gs) {
    const int64_t groups = K / gs;
    const int64_t row_bytes = K >> 1;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < M * N; t += stride) {
        const int64_t n = t % N;
        const int64_t m = t / N;
        const float* xr = x + m * K;
        const uint8_t* qr = q + n * row_bytes;
        const float* sr = scale + n * groups;
        const float* zr = zero + n * groups;
        float acc = 0.0f;
        int64_t k = 0;
        for (int64_t g = 0; g < groups; ++g) {  // group by group: k / gs without a division
            const float sc = __ldg(sr + g);
            const float zp = __ldg(zr + g);
            for (const int64_t end = k + gs; k < end; ++k) {
                const uint32_t b = __ldg(qr + (k >> 1));
                const uint32_t code = (k & 1) ? (b >> 4) : (b & 0x0Fu);
                const float w = __fmul_rn(__fsub_rn(static_cast<float>(code), zp), sc);
                acc = __fmaf_rn(__ldg(xr + k), w, acc);
            }
        }
        out[t] = acc;
    }
}

// Eight codes (one word, k = 0..7) -> four float2 pairs (c_2j - 8, 16 (c_2j+1 - 8)).
__device__ __forceinline__ void widen8(uint32_t word, float2 (&c)[4]) {
    const uint32_t lo = word & 0x0F0F0F0Fu;  // even k, in place
    const uint32_t hi = word & 0xF0F0F0F0u;  // odd k, times 16
    const float2 bias = make_float2(-8388616.0f, -8388736.0f);  // -(2^23 + 8), -(2^23 + 128)
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440 + j)),
                                     __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440 + j)));
        c[j] = __fadd2_rn(f, bias);
    }
}

// A slice holding an infinity or a NaN: popcorn's per-element form
// w = (c - z) * s, acc = fma(x, w, acc) over the 16 elements in k order, so
// the slice gives +-inf or NaN exactly where popcorn's sum does (the
// factored form below would turn inf * (c - 8) - (z - 8) * inf into NaN).
__device__ __forceinline__ float i4_direct_slice(uint2 w, const float4 (&xr)[4], float sc, float zp) {
    const uint32_t words[2] = {w.x, w.y};
    const float xk[16] = {xr[0].x, xr[0].y, xr[0].z, xr[0].w, xr[1].x, xr[1].y, xr[1].z, xr[1].w,
                          xr[2].x, xr[2].y, xr[2].z, xr[2].w, xr[3].x, xr[3].y, xr[3].z, xr[3].w};
    float acc = 0.0f;
    #pragma unroll
    for (int e = 0; e < 16; ++e) {
        const uint32_t code = (words[e >> 3] >> (4 * (e & 7))) & 0xFu;
        const float wk = __fmul_rn(__fsub_rn(static_cast<float>(code), zp), sc);
        acc = __fmaf_rn(xk[e], wk, acc);
    }
    return acc;
}

__device__ __forceinline__ bool slice_finite(const float4 (&xr)[4]) {
    bool ok = true;
    #pragma unroll
    for (int c = 0; c < 4; ++c) {
        ok = ok && isfinite(xr[c].x) && isfinite(xr[c].y) && isfinite(xr[c].z) && isfinite(xr[c].w);
    }
    return ok;
}

// MT activation rows (<= 4), U 16-element K slices per thread, R weight rows
// per block; gridDim.y = ceil(M / MT).
template <int MT, int U, int R>
__global__ void __launch_bounds__(kI4Threads, (MT == 1 && U == 1) ? 4 : 2)
i4_xs_kernel(float* __restrict__ out, const float* __restrict__ x, const uint8_t* __restrict__ q,
             const float* __restrict__ scale, const float* __restrict__ zero, int64_t M, int64_t N, int64_t K,
             int64_t gs) {
    __shared__ float part[R * MT][kI4Warps];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t units = K >> 4;
    const int64_t groups = K / gs;
    const int64_t row_bytes = K >> 1;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * R;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * MT;

    // Programmatic dependent launch: release the next kernel of the stream,
    // pull this block's weight rows and group parameters into L2 while the
    // previous kernel finishes (a hint; every real read follows the wait).
    pdl_launch_dependents();
    if (tid < kI4Warps + 2 && blockIdx.y == 0) {
        const int64_t rows = (r0 + R <= N) ? R : N - r0;
        if (tid < kI4Warps) {
            prefetch_l2_range(q + r0 * row_bytes, rows * row_bytes, tid, kI4Warps);
        } else {
            prefetch_l2_range((tid == kI4Warps ? scale : zero) + r0 * groups, rows * groups * 4, 0, 1);
        }
    }
    pdl_wait();

    // Weight bytes of this block first (independent of x), then the group
    // parameters, all requested before any of them is needed.
    uint2 w[R][U];
    float sc[R][U], zc[R][U];
    const int units_per_group = static_cast<int>(gs >> 4);
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        const int unit = tid + u * kI4Threads;
        #pragma unroll
        for (int r = 0; r < R; ++r) {
            w[r][u] = (r0 + r < N && unit < units)
                          ? __ldg(reinterpret_cast<const uint2*>(q + (r0 + r) * row_bytes) + unit)
                          : make_uint2(0u, 0u);
        }
    }
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        const int unit = tid + u * kI4Threads;
        const int g = unit / units_per_group;
        #pragma unroll
        for (int r = 0; r < R; ++r) {
            const bool ok = r0 + r < N && unit < units;
            sc[r][u] = ok ? __ldg(scale + (r0 + r) * groups + g) : 0.0f;
            zc[r][u] = ok ? __ldg(zero + (r0 + r) * groups + g) - 8.0f : 0.0f;
        }
    }

    // Activations of this thread's slices, as loaded.
    float4 xr[MT][U][4];
    #pragma unroll
    for (int m = 0; m < MT; ++m) {
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kI4Threads;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                xr[m][u][c] = (unit < units && m0 + m < M)
                                  ? __ldg(reinterpret_cast<const float4*>(x + (m0 + m) * K + unit * 16) + c)
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
    }

    float acc[R * MT];
    #pragma unroll
    for (int i = 0; i < R * MT; ++i) acc[i] = 0.0f;

    // f32 layout: codes widened exactly, activations as pairs
    // (x_2j, x_2j+1 / 16), packed multiply-adds.
    auto dot_float = [&]() {
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            float2 xv[MT][8];
            float xsum[MT];
            #pragma unroll
            for (int m = 0; m < MT; ++m) {
                float s = 0.0f;
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 v = xr[m][u][c];
                    s += (v.x + v.y) + (v.z + v.w);
                    xv[m][2 * c] = make_float2(v.x, v.y * 0.0625f);
                    xv[m][2 * c + 1] = make_float2(v.z, v.w * 0.0625f);
                }
                xsum[m] = s;
            }
            bool fin[MT];
            #pragma unroll
            for (int m = 0; m < MT; ++m) fin[m] = slice_finite(xr[m][u]);
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                float2 a[MT];
                #pragma unroll
                for (int m = 0; m < MT; ++m) a[m] = make_float2(0.0f, 0.0f);
                const uint32_t words[2] = {w[r][u].x, w[r][u].y};
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float2 c[4];
                    widen8(words[h], c);
                    #pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        #pragma unroll
                        for (int m = 0; m < MT; ++m) a[m] = __ffma2_rn(xv[m][4 * h + j], c[j], a[m]);
                    }
                }
                #pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (fin[m]) {
                        const float d = fmaf(-zc[r][u], xsum[m], a[m].x + a[m].y);
                        acc[r * MT + m] = fmaf(sc[r][u], d, acc[r * MT + m]);
                    } else {
                        acc[r * MT + m] += i4_direct_slice(w[r][u], xr[m][u], sc[r][u], zc[r][u] + 8.0f);
                    }
                }
            }
        }
    };

    if constexpr (MT == 1) {
        // M = 1: the slice of x becomes 22-bit fixed point X (scaled by a
        // power of two from the thread's max |x|), written as three bytes
        // X = d2 * 2^16 + d1 * 2^8 + d0 (d0, d1 unsigned, d2 signed). The
        // codes are bytes after one mask (even k) or a shift and a mask
        // (odd k), so each dp4a multiplies four codes by four digits exactly:
        // six dp4a finish eight codes. Per row and slice the int32 sum
        // S = sum X c (|S| < 2^30) is exact; S - 8 sum X is rounded once to
        // f32, the zero point enters as (z - 8) * sum X, and the power of two
        // is undone exactly. A warp holding a non-finite x or a slice max
        // outside [2^-90, 2^100] keeps the f32 layout.
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
        if (!__any_sync(0xffffffffu, bad)) {
            float up = 1.0f, down = 1.0f;
            if (mb != 0u) {
                const int ex = 148 - static_cast<int>(mb >> 23);  // max |x| * 2^ex < 2^22
                up = __int_as_float((ex + 127) << 23);
                down = __int_as_float((127 - ex) << 23);
            }
            // digit[u][h][p][d]: digit d of the four activations that meet
            // the even (p = 0) or odd (p = 1) codes of weight word h.
            uint32_t digit[U][2][2][3];
            int xs[U];
            #pragma unroll
            for (int u = 0; u < U; ++u) {
                int xi[16];
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 v = xr[0][u][c];
                    xi[4 * c] = __float2int_rn(v.x * up);
                    xi[4 * c + 1] = __float2int_rn(v.y * up);
                    xi[4 * c + 2] = __float2int_rn(v.z * up);
                    xi[4 * c + 3] = __float2int_rn(v.w * up);
                }
                int s = 0;
                #pragma unroll
                for (int e = 0; e < 16; ++e) s += xi[e];
                xs[u] = s;
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    #pragma unroll
                    for (int p = 0; p < 2; ++p) {
                        const int e = 8 * h + p;
                        const uint32_t a = xi[e], b = xi[e + 2], c = xi[e + 4], d = xi[e + 6];
                        const uint32_t t01 = __byte_perm(a, b, 0x5140), t23 = __byte_perm(c, d, 0x5140);
                        const uint32_t v01 = __byte_perm(a, b, 0x7362), v23 = __byte_perm(c, d, 0x7362);
                        digit[u][h][p][0] = __byte_perm(t01, t23, 0x5410);
                        digit[u][h][p][1] = __byte_perm(t01, t23, 0x7632);
                        digit[u][h][p][2] = __byte_perm(v01, v23, 0x5410);
                    }
                }
            }
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                float a = 0.0f;
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    unsigned s0 = 0u, s1 = 0u;
                    int s2 = 0;
                    const uint32_t words[2] = {w[r][u].x, w[r][u].y};
                    #pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t lo = words[h] & 0x0F0F0F0Fu;
                        const uint32_t hi = (words[h] >> 4) & 0x0F0F0F0Fu;
                        s0 = __dp4a(digit[u][h][0][0], lo, s0);
                        s0 = __dp4a(digit[u][h][1][0], hi, s0);
                        s1 = __dp4a(digit[u][h][0][1], lo, s1);
                        s1 = __dp4a(digit[u][h][1][1], hi, s1);
                        s2 = __dp4a(static_cast<int>(digit[u][h][0][2]), static_cast<int>(lo), s2);
                        s2 = __dp4a(static_cast<int>(digit[u][h][1][2]), static_cast<int>(hi), s2);
                    }
                    const int t = s2 * 65536 + static_cast<int>(s1 * 256u + s0) - 8 * xs[u];
                    const float d = fmaf(-zc[r][u], static_cast<float>(xs[u]), static_cast<float>(t));
                    a = fmaf(sc[r][u], d, a);
                }
                acc[r] = a * down;
            }
        } else {
            dot_float();
        }
    } else {
        dot_float();
    }

    constexpr int V = R * MT;
    const float total = i4_reduce_scatter<V>(acc, lane);
    constexpr int span = 32 / V;
    if ((lane % span) == 0) part[lane / span][warp] = total;
    __syncthreads();
    if (tid < V) {
        const int r = tid / MT;
        const int m = tid % MT;
        float s = 0.0f;
        #pragma unroll
        for (int wv = 0; wv < kI4Warps; ++wv) s += part[tid][wv];
        if (r0 + r < N && m0 + m < M) out[(m0 + m) * N + r0 + r] = s;
    }
}

// Decode (M = 1) with the weights staged in shared memory before the
// previous kernel of the stream has finished: the int4 counterpart of the
// per-channel gemv_stage_kernel. One 512-thread CTA per SM owns a contiguous
// range of rows; right after it starts, each row's packed codes, group scales
// and group zero points go to the TMA engine as three 1-D bulk copies (one
// mbarrier for all), and only then does the CTA wait for the previous kernel
// and read x. At K = 4096, group 128, a CTA holds 28 rows in 64.5 KB, so the
// next call's CTA fits on the same SM and streams its weights while this one
// computes. Two groups of 256 threads take alternate rows; thread t of a
// group owns the 16-element slice t (as in i4_xs_kernel<1, 1, 8>), and the
// per-row arithmetic, the butterfly reduce-scatter (whose pairings do not
// depend on a row's place in it) and the fixed-order sum across warps are
// i4_xs_kernel's, so the two kernels return the same bits. Only weight-side
// data is read before the wait (the matmul kernels that release this one
// early never write codes, scales or zero points).
constexpr int kI4StageGroups = 2;
constexpr int kI4StageThreads = kI4StageGroups * kI4Threads;
constexpr int kI4StageSR = 8;              // rows per group per iteration
constexpr int kI4StageMaxRows = 64;
constexpr int kI4StageBytes = 100 * 1024;  // room for a second CTA on the SM

__global__ void __launch_bounds__(kI4StageThreads, 2)
i4_stage_kernel(float* __restrict__ out, const float* __restrict__ x, const uint8_t* __restrict__ q,
                const float* __restrict__ scale, const float* __restrict__ zero, int64_t N, int64_t K, int64_t gs) {
    extern __shared__ __align__(16) uint8_t st[];
    __shared__ __align__(8) uint64_t s_full;
    const int grp = threadIdx.x / kI4Threads;
    const int tid = threadIdx.x % kI4Threads;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t G = gridDim.x;
    const int64_t r0 = N * blockIdx.x / G;
    const int rows = static_cast<int>(N * (blockIdx.x + 1) / G - r0);
    const int rows_max = static_cast<int>((N + G - 1) / G);
    const int64_t units = K >> 4;
    const int groups = static_cast<int>(K / gs);
    const int row_bytes = static_cast<int>(K >> 1);
    uint8_t* codes = st;                                                            // [rows_max][K/2]
    float* sc_s = reinterpret_cast<float*>(st + rows_max * row_bytes);              // [rows_max][groups]
    float* zp_s = sc_s + rows_max * groups;                                         // [rows_max][groups]
    float* part = zp_s + rows_max * groups;                                         // [rows_max][8 warps]
    const uint32_t full = sm100::smem_addr(&s_full);

    if (threadIdx.x == 0) {
        sm100::mbar_init(full, 1);
        sm100::fence_barrier_init();
        sm100::mbar_arrive_expect_tx(full, static_cast<uint32_t>(rows * (row_bytes + 8 * groups)));
    }
    pdl_launch_dependents();
    __syncthreads();
    if (threadIdx.x < rows) {
        const int r = threadIdx.x;
        sm100::bulk_load_1d(sm100::smem_addr(codes + r * row_bytes), q + (r0 + r) * row_bytes,
                            static_cast<uint32_t>(row_bytes), full);
    } else if (threadIdx.x >= 128 && threadIdx.x < 128 + rows) {
        const int r = threadIdx.x - 128;
        sm100::bulk_load_1d(sm100::smem_addr(sc_s + r * groups), scale + (r0 + r) * groups,
                            static_cast<uint32_t>(4 * groups), full);
    } else if (threadIdx.x >= 256 && threadIdx.x < 256 + rows) {
        const int r = threadIdx.x - 256;
        sm100::bulk_load_1d(sm100::smem_addr(zp_s + r * groups), zero + (r0 + r) * groups,
                            static_cast<uint32_t>(4 * groups), full);
    } else if (threadIdx.x == kI4StageThreads - 1) {
        prefetch_l2_range(x, K * static_cast<int64_t>(sizeof(float)), 0, 1);
    }
    pdl_wait();

    // This thread's 16 activations (zero beyond K), as i4_xs_kernel loads them.
    const bool in_k = tid < units;
    float4 xr[4];
    #pragma unroll
    for (int c = 0; c < 4; ++c) {
        xr[c] = in_k ? __ldg(reinterpret_cast<const float4*>(x + tid * 16) + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    const int g = in_k ? static_cast<int>(tid / (gs >> 4)) : 0;
    if (!sm100::mbar_wait(full, 0, &g_i4_error, kI4StageTimeoutBit)) {
        sm100::mbar_wait(full, 0, &g_i4_error, kI4StageTimeoutBit);
    }

    // The row loop: this group's rows rg, rg + 2, ..., SR at a time; `dot`
    // returns this thread's partial of one row from its staged bytes.
    auto run = [&](auto&& dot) {
        for (int rg = grp; rg < rows; rg += kI4StageSR * kI4StageGroups) {
            float acc[kI4StageSR];
            #pragma unroll
            for (int r = 0; r < kI4StageSR; ++r) {
                const int row = rg + r * kI4StageGroups;
                acc[r] = 0.0f;
                if (row < rows && in_k) {
                    const uint2 w = *reinterpret_cast<const uint2*>(codes + row * row_bytes + tid * 8);
                    acc[r] = dot(w, sc_s[row * groups + g], zp_s[row * groups + g]);
                }
            }
            const float total = i4_reduce_scatter<kI4StageSR>(acc, lane);
            constexpr int span = 32 / kI4StageSR;
            if ((lane % span) == 0) {
                const int row = rg + (lane / span) * kI4StageGroups;
                if (row < rows) part[row * kI4Warps + warp] = total;
            }
        }
    };

    // Fixed point unless the warp holds a non-finite x or a slice max
    // outside [2^-90, 2^100] (i4_xs_kernel's rule and scaling).
    uint32_t mb = 0;
    #pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float4 v = xr[c];
        mb = max(mb, max(max(__float_as_uint(v.x) & 0x7FFFFFFFu, __float_as_uint(v.y) & 0x7FFFFFFFu),
                         max(__float_as_uint(v.z) & 0x7FFFFFFFu, __float_as_uint(v.w) & 0x7FFFFFFFu)));
    }
    const bool bad = mb != 0u && (mb < 0x12800000u || mb > 0x71800000u);
    if (!__any_sync(0xffffffffu, bad)) {
        float up = 1.0f, down = 1.0f;
        if (mb != 0u) {
            const int ex = 148 - static_cast<int>(mb >> 23);  // max |x| * 2^ex < 2^22
            up = __int_as_float((ex + 127) << 23);
            down = __int_as_float((127 - ex) << 23);
        }
        int xi[16];
        #pragma unroll
        for (int c = 0; c < 4; ++c) {
            xi[4 * c] = __float2int_rn(xr[c].x * up);
            xi[4 * c + 1] = __float2int_rn(xr[c].y * up);
            xi[4 * c + 2] = __float2int_rn(xr[c].z * up);
            xi[4 * c + 3] = __float2int_rn(xr[c].w * up);
        }
        int xs = 0;
        #pragma unroll
        for (int e = 0; e < 16; ++e) xs += xi[e];
        uint32_t digit[2][2][3];
        #pragma unroll
        for (int h = 0; h < 2; ++h) {
            #pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int e = 8 * h + p;
                const uint32_t a = xi[e], b = xi[e + 2], c = xi[e + 4], d = xi[e + 6];
                const uint32_t t01 = __byte_perm(a, b, 0x5140), t23 = __byte_perm(c, d, 0x5140);
                const uint32_t v01 = __byte_perm(a, b, 0x7362), v23 = __byte_perm(c, d, 0x7362);
                digit[h][p][0] = __byte_perm(t01, t23, 0x5410);
                digit[h][p][1] = __byte_perm(t01, t23, 0x7632);
                digit[h][p][2] = __byte_perm(v01, v23, 0x5410);
            }
        }
        run([&](uint2 w, float sc, float zp) {
            const float zc = zp - 8.0f;
            unsigned s0 = 0u, s1 = 0u;
            int s2 = 0;
            const uint32_t words[2] = {w.x, w.y};
            #pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t lo = words[h] & 0x0F0F0F0Fu;
                const uint32_t hi = (words[h] >> 4) & 0x0F0F0F0Fu;
                s0 = __dp4a(digit[h][0][0], lo, s0);
                s0 = __dp4a(digit[h][1][0], hi, s0);
                s1 = __dp4a(digit[h][0][1], lo, s1);
                s1 = __dp4a(digit[h][1][1], hi, s1);
                s2 = __dp4a(static_cast<int>(digit[h][0][2]), static_cast<int>(lo), s2);
                s2 = __dp4a(static_cast<int>(digit[h][1][2]), static_cast<int>(hi), s2);
            }
            const int t = s2 * 65536 + static_cast<int>(s1 * 256u + s0) - 8 * xs;
            const float d = fmaf(-zc, static_cast<float>(xs), static_cast<float>(t));
            return fmaf(sc, d, 0.0f) * down;
        });
    } else {
        float2 xv[8];
        float s = 0.0f;
        #pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4 v = xr[c];
            s += (v.x + v.y) + (v.z + v.w);
            xv[2 * c] = make_float2(v.x, v.y * 0.0625f);
            xv[2 * c + 1] = make_float2(v.z, v.w * 0.0625f);
        }
        const float xsum = s;
        const bool fin = slice_finite(xr);
        run([&](uint2 w, float sc, float zp) {
            if (!fin) return i4_direct_slice(w, xr, sc, zp);
            const float zc = zp - 8.0f;
            float2 a = make_float2(0.0f, 0.0f);
            const uint32_t words[2] = {w.x, w.y};
            #pragma unroll
            for (int h = 0; h < 2; ++h) {
                float2 c[4];
                widen8(words[h], c);
                #pragma unroll
                for (int j = 0; j < 4; ++j) a = __ffma2_rn(xv[4 * h + j], c[j], a);
            }
            const float d = fmaf(-zc, xsum, a.x + a.y);
            return fmaf(sc, d, 0.0f);
        });
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rows; i += kI4StageThreads) {
        float sum = 0.0f;
        #pragma unroll
        for (int wv = 0; wv < kI4Warps; ++wv) sum += part[i * kI4Warps + wv];
        out[r0 + i] = sum;
    }
}

// Position of element i of a group in the order in which popcorn's min/max
// block (256 threads, thread t scanning t, t + 256, ...; a halving tree that
// keeps the lower partner on a tie) lets it win a tie: threads rank by their
// bit-reversed index, then by their scan order. Smaller wins.
__device__ __forceinline__ uint64_t i4_tie_rank(int64_t i) {
    const uint64_t rev = __brev(static_cast<uint32_t>(i & 255)) >> 24;
    return (rev << 56) | static_cast<uint64_t>(i >> 8);
}

__device__ __forceinline__ uint32_t i4_code(float v, float sc, float zp) {
    float qv = rintf(__fadd_rn(__fdiv_rn(v, sc), zp));
    if (qv < 0.0f) qv = 0.0f;
    if (qv > 15.0f) qv = 15.0f;
    return (qv != qv) ? 0u : static_cast<uint32_t>(qv);  // a NaN code packs as 0
}

// One warp per (row, group); grid-stride over all groups. With PACK (even
// group sizes) the warp also writes the group's gs / 2 packed bytes.
template <bool PACK>
__global__ void __launch_bounds__(256)
i4_quantize_kernel(uint8_t* __restrict__ out, float* __restrict__ scale, float* __restrict__ zero,
                   const float* __restrict__ in, int64_t N, int64_t K, int64_t gs) {
    const int lane = threadIdx.x & 31;
    const int64_t groups = K / gs;
    const int64_t total = N * groups;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < total;
         item += nwarps) {
        const int64_t row = item / groups;
        const int64_t g = item - row * groups;
        const float* r = in + row * K + g * gs;
        // (value, tie rank) minimum and maximum; NaN fails every compare.
        float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
        uint64_t mnk = ~uint64_t{0}, mxk = ~uint64_t{0};
        for (int64_t i = lane; i < gs; i += 32) {
            const float v = __ldg(r + i);
            const uint64_t key = i4_tie_rank(i);
            if (v < mn || (v == mn && key < mnk)) { mn = v; mnk = key; }
            if (v > mx || (v == mx && key < mxk)) { mx = v; mxk = key; }
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float omn = __shfl_xor_sync(0xffffffffu, mn, off);
            const uint64_t omnk = __shfl_xor_sync(0xffffffffu, mnk, off);
            const float omx = __shfl_xor_sync(0xffffffffu, mx, off);
            const uint64_t omxk = __shfl_xor_sync(0xffffffffu, mxk, off);
            if (omn < mn || (omn == mn && omnk < mnk)) { mn = omn; mnk = omnk; }
            if (omx > mx || (omx == mx && omxk < mxk)) { mx = omx; mxk = omxk; }
        }
        float sc = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
        if (sc == 0.0f) sc = 1.0f;
        const float zp = __fdiv_rn(-mn, sc);
        if (lane == 0) {
            scale[item] = sc;
            zero[item] = zp;
        }
        if (PACK) {
            uint8_t* o = out + row * (K >> 1) + ((g * gs) >> 1);
            for (int64_t b = lane; b < (gs >> 1); b += 32) {
                const uint32_t lo = i4_code(__ldg(r + 2 * b), sc, zp);
                const uint32_t hi = i4_code(__ldg(r + 2 * b + 1), sc, zp);
                o[b] = static_cast<uint8_t>((hi << 4) | lo);
            }
        }
    }
}

// Odd group sizes: one thread per packed byte, each nibble with the
// parameters of its own group (stored by i4_quantize_kernel<false>).
__global__ void __launch_bounds__(256)
i4_pack_kernel(uint8_t* __restrict__ out, const float* __restrict__ scale, const float* __restrict__ zero,
               const float* __restrict__ in, int64_t N, int64_t K, int64_t gs) {
    const int64_t row_bytes = K >> 1;
    const int64_t groups = K / gs;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < N * row_bytes; t += stride) {
        const int64_t row = t / row_bytes;
        const int64_t k = 2 * (t - row * row_bytes);
        const int64_t glo = row * groups + k / gs;
        const int64_t ghi = row * groups + (k + 1) / gs;
        const uint32_t lo = i4_code(__ldg(in + row * K + k), scale[glo], zero[glo]);
        const uint32_t hi = i4_code(__ldg(in + row * K + k + 1), scale[ghi], zero[ghi]);
        out[t] = static_cast<uint8_t>((hi << 4) | lo);
    }
}

// The staged decode kernel when its conditions hold (M = 1, K <= 4096 with
// 16-byte rows, group scales and zero points in 16-byte rows, every CTA's
// rows within kI4StageBytes); returns false (nothing launched) otherwise.
bool launch_i4_stage(popcornStatus_t* stp, float* out, const float* x, const uint8_t* q, const float* scale,
                     const float* zero, int64_t N, int64_t K, int64_t gs, cudaStream_t stream) {
    const int64_t groups = K / gs;
    if (K > 16 * kI4Threads || K % 32 != 0 || gs % 16 != 0 || groups % 4 != 0) return false;
    if (!aligned16(x) || !aligned16(q) || !aligned16(scale) || !aligned16(zero)) return false;
    const int64_t G = device_sm_count() < N ? device_sm_count() : N;
    const int64_t rows_max = ceil_div(N, G);
    const int64_t smem = rows_max * (K / 2 + 8 * groups) + rows_max * kI4Warps * 4;
    if (rows_max > kI4StageMaxRows || smem > kI4StageBytes) return false;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool known = dev >= 0 && dev < 64;
    if (!known || !attr_set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(i4_stage_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kI4StageBytes);
        if (e != cudaSuccess) {
            *stp = record_cuda(e);
            return true;
        }
        if (known) attr_set[dev] = true;
    }
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(G)), dim3(kI4StageThreads),
                                              static_cast<size_t>(smem), stream, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, i4_stage_kernel, out, x, q, scale, zero, N, K, gs);
    *stp = (e != cudaSuccess) ? record_cuda(e) : check_launch();
    return true;
}

// Decode (M = 1, K = 1024, 2048 or 4096) on the warp-level tensor path: the
// staging of i4_stage_kernel (each row's packed codes, group scales and zero
// points as 1-D bulk copies before griddepcontrol.wait, two CTAs per SM),
// codes at a pitch of K / 2 + 16 bytes (an odd multiple of 16, so the
// ldmatrix phases are free of bank conflicts), and the arithmetic of the
// per-channel gemv_mma_kernel: warp w owns the k-steps [w KSMAX,
// (w + 1) KSMAX) of 32 codes, its activations become 30-bit fixed point
// X = rint(x 2^s) held as four signed base-256 digits, and
// mma.sync m16n8k32 (u8 codes x s8 digits -> s32) sums them exactly.
//
// One ldmatrix.x4 brings a lane the 4 bytes (8 codes, k = 8t .. 8t + 7) of
// rows g and g + 8 for two k-steps; the low nibbles (even k) form A's first
// k-half and the high nibbles (odd k) its second, and B is built in the
// same order (digits of x at 8t, 8t + 2, ... in b0, at 8t + 1, 8t + 3, ...
// in b1) from the warp's activations, converted once (one value per lane
// and step) into shared memory; sum_k X_k comes from the digit sums. After each group of GSTEPS steps the exact sums give
//     sum_k (c_k - z) x_k = 2^-s (sum_k c_k X_k - z sum_k X_k)
// in double (sum_k X_k exact), times the group scale; the 16 warp partials
// are added in warp order and rounded once. Warps holding a non-finite or
// extreme activation use popcorn's per-element form (w = (c - z) s, fma).
constexpr int kI4MmaStageBytes = (228 * 1024 - 2 * 1024) / 2 - 64;
constexpr int kI4MmaMaxRows = 64;

// B fragment of a k-step in the int4 k-order from the warp's converted
// activations y (Y = X + 0x80808080 per value, 32 per step): lane (g, t)
// takes the eight values 8t .. 8t + 7 of the step, digit g % 4 of the even
// ones in b0 and of the odd ones in b1 (lanes g >= 4: zero); *dsum gains
// the sum of those eight digits.
__device__ __forceinline__ void i4_b_fragment(const uint32_t* y, int lane, uint32_t& b0, uint32_t& b1, int& dsum) {
    const int g = lane >> 2;
    const uint4 p = *reinterpret_cast<const uint4*>(y + 8 * (lane & 3));
    const uint4 r = *reinterpret_cast<const uint4*>(y + 8 * (lane & 3) + 4);
    const uint32_t sel = static_cast<uint32_t>((g & 3) | (((g & 3) + 4) << 4));
    const uint32_t o = 0x80808080u;
    const uint32_t ev = __byte_perm(__byte_perm(p.x, p.z, sel), __byte_perm(r.x, r.z, sel), 0x5410) ^ o;
    const uint32_t od = __byte_perm(__byte_perm(p.y, p.w, sel), __byte_perm(r.y, r.w, sel), 0x5410) ^ o;
    b0 = g < 4 ? ev : 0u;
    b1 = g < 4 ? od : 0u;
    dsum = __dp4a(static_cast<int>(b0), 0x01010101, __dp4a(static_cast<int>(b1), 0x01010101, dsum));
}

template <int KSMAX, int GSTEPS, int GROUPS, int SETS>
__global__ void __launch_bounds__(kMmaThreads, 2)
i4_mma_kernel(float* __restrict__ out, const float* __restrict__ x, const uint8_t* __restrict__ q,
              const float* __restrict__ scale, const float* __restrict__ zero, int64_t N, int64_t K, int64_t gs) {
    constexpr int NG = KSMAX / GSTEPS;  // groups of one warp
    // codes [rows][K/2 + 16], scales and zeros [rows][groups + 4] (the pad
    // spreads the rows of one scale read over the banks), then Y
    extern __shared__ __align__(16) uint8_t st[];
    __shared__ __align__(8) uint64_t s_full;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t G = gridDim.x;
    const int64_t r0 = N * blockIdx.x / G;
    const int rows = static_cast<int>(N * (blockIdx.x + 1) / G - r0);
    const int rows_max = static_cast<int>((N + G - 1) / G);
    const int row_bytes = static_cast<int>(K >> 1);
    const int pitch = row_bytes + 16;
    const int groups = static_cast<int>(K / gs);
    float* sc_s = reinterpret_cast<float*>(st + rows_max * pitch);
    const int gstride = groups + 4;
    float* zp_s = sc_s + rows_max * gstride;
    uint32_t* ybuf = reinterpret_cast<uint32_t*>(zp_s + rows_max * gstride) + warp * (32 * KSMAX);  // this warp's Y
    const uint32_t full = sm100::smem_addr(&s_full);
    const uint32_t base = sm100::smem_addr(st);

    if (threadIdx.x == 0) {
        sm100::mbar_init(full, 1);
        sm100::fence_barrier_init();
        sm100::mbar_arrive_expect_tx(full, static_cast<uint32_t>(rows * (row_bytes + 8 * groups)));
    }
    pdl_launch_dependents();
    __syncthreads();
    if (threadIdx.x < rows) {
        const int r = threadIdx.x;
        sm100::bulk_load_1d(base + r * pitch, q + (r0 + r) * row_bytes, static_cast<uint32_t>(row_bytes), full);
    } else if (threadIdx.x >= 128 && threadIdx.x < 128 + rows) {
        const int r = threadIdx.x - 128;
        sm100::bulk_load_1d(sm100::smem_addr(sc_s + r * gstride), scale + (r0 + r) * groups,
                            static_cast<uint32_t>(4 * groups), full);
    } else if (threadIdx.x >= 256 && threadIdx.x < 256 + rows) {
        const int r = threadIdx.x - 256;
        sm100::bulk_load_1d(sm100::smem_addr(zp_s + r * gstride), zero + (r0 + r) * groups,
                            static_cast<uint32_t>(4 * groups), full);
    } else if (threadIdx.x == kMmaThreads - 1) {
        prefetch_l2_range(x, K * static_cast<int64_t>(sizeof(float)), 0, 1);
    }
    pdl_wait();
    const int c0 = warp * KSMAX;
    // This warp's 32 * KSMAX activations, one per lane and step (coalesced),
    // their max |x| (the rule of warp_scale), then Y = X + 0x80808080 into
    // shared memory once, where every step's B fragments are built from.
    float xv[KSMAX];
    uint32_t mb = 0;
    #pragma unroll
    for (int i = 0; i < KSMAX; ++i) {
        xv[i] = __ldg(x + 32 * (c0 + i) + lane);
        mb = max(mb, __float_as_uint(xv[i]) & 0x7FFFFFFFu);
    }
    mb = __reduce_max_sync(0xffffffffu, mb);
    WarpScale ws;
    ws.fixed = mb == 0u || (mb >= 0x12800000u && mb <= 0x71800000u);
    ws.s = mb == 0u ? 0 : 29 - (static_cast<int>(mb >> 23) - 127);
    ws.up = mb == 0u ? 1.0f : __int_as_float((ws.s + 127) << 23);
    if (ws.fixed) {
        #pragma unroll
        for (int i = 0; i < KSMAX; ++i) {
            ybuf[32 * i + lane] = static_cast<uint32_t>(__float2int_rn(xv[i] * ws.up)) + 0x80808080u;
        }
    }
    __syncwarp();
    const int64_t grp0 = static_cast<int64_t>(32) * c0 / gs;

    if (!sm100::mbar_wait(full, 0, &g_i4_error, kI4StageTimeoutBit)) {
        sm100::mbar_wait(full, 0, &g_i4_error, kI4StageTimeoutBit);
    }

    const int g = lane >> 2;
    const int rgroups = (rows + 15) >> 4;
    double part_lo[GROUPS], part_hi[GROUPS];
    #pragma unroll
    for (int j = 0; j < GROUPS; ++j) part_lo[j] = part_hi[j] = 0.0;
    if (ws.fixed) {
        const double down = __longlong_as_double(static_cast<long long>(1023 - ws.s) << 52);
        const int mi = lane >> 3;
        const int mrow = (lane & 7) + 8 * (mi & 1);
        const int mk = 16 * (mi >> 1);
        #pragma unroll
        for (int n = 0; n < NG; ++n) {
            int d[GROUPS][SETS][4];
            #pragma unroll
            for (int j = 0; j < GROUPS; ++j) {
                #pragma unroll
                for (int e2 = 0; e2 < SETS; ++e2) d[j][e2][0] = d[j][e2][1] = d[j][e2][2] = d[j][e2][3] = 0;
            }
            int dsum = 0;  // this lane's digit-g sum over the group's steps (lanes g < 4)
            #pragma unroll
            for (int i2 = 0; i2 < GSTEPS; i2 += 2) {
                const int c = c0 + n * GSTEPS + i2;  // steps c and c + 1
                uint32_t b[2][2];
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    i4_b_fragment(ybuf + 32 * (n * GSTEPS + i2 + h), lane, b[h][0], b[h][1], dsum);
                }
                #pragma unroll
                for (int j = 0; j < GROUPS; ++j) {
                    if (j < rgroups) {
                        int r = 16 * j + mrow;
                        r = r < rows ? r : rows - 1;  // past the last row: read it again, never stored
                        uint32_t m[4];
                        ldmatrix_x4(m, base + r * pitch + 16 * c + mk);
                        #pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const uint32_t a[4] = {m[2 * h] & 0x0F0F0F0Fu, m[2 * h + 1] & 0x0F0F0F0Fu,
                                                   (m[2 * h] >> 4) & 0x0F0F0F0Fu, (m[2 * h + 1] >> 4) & 0x0F0F0F0Fu};
                            mma_u8s8_16832(d[j][(i2 + h) % SETS], a, b[h][0], b[h][1]);
                        }
                    }
                }
            }
            // The group's sum of X = sum_d 256^d (sum of digit d): digit sums
            // over t, then from lanes 0, 4, 8, 12 (exact in double).
            dsum += __shfl_xor_sync(0xffffffffu, dsum, 1);
            dsum += __shfl_xor_sync(0xffffffffu, dsum, 2);
            const int s0 = __shfl_sync(0xffffffffu, dsum, 0);
            const int s1 = __shfl_sync(0xffffffffu, dsum, 4);
            const int s2 = __shfl_sync(0xffffffffu, dsum, 8);
            const int s3 = __shfl_sync(0xffffffffu, dsum, 12);
            const double xs = static_cast<double>(s0) + 256.0 * static_cast<double>(s1) +
                              65536.0 * static_cast<double>(s2) + 16777216.0 * static_cast<double>(s3);
            const double sxs = xs * down;
            const int64_t grp = grp0 + n;
            #pragma unroll
            for (int j = 0; j < GROUPS; ++j) {
                #pragma unroll
                for (int e2 = 1; e2 < SETS; ++e2) {  // exact: |column sum| < 2^22
                    #pragma unroll
                    for (int v = 0; v < 4; ++v) d[j][0][v] += d[j][e2][v];
                }
                double lo, hi;
                combine_digits(d[j][0], ws.s, lo, hi);
                const int ra = min(16 * j + g, rows - 1);
                const int rb = min(16 * j + g + 8, rows - 1);
                part_lo[j] += (lo - static_cast<double>(zp_s[ra * gstride + grp]) * sxs) *
                              static_cast<double>(sc_s[ra * gstride + grp]);
                part_hi[j] += (hi - static_cast<double>(zp_s[rb * gstride + grp]) * sxs) *
                              static_cast<double>(sc_s[rb * gstride + grp]);
            }
        }
    } else {
        // popcorn's per-element form (rare); lane r % 32 keeps row r's sum.
        float fb0 = 0.0f, fb1 = 0.0f;
        for (int r = 0; r < rows; ++r) {
            const uint8_t* codes = st + r * pitch;
            float a = 0.0f;
            for (int c = c0; c < c0 + KSMAX; ++c) {
                const int k = 32 * c + lane;
                const int code = (codes[k >> 1] >> ((k & 1) * 4)) & 0xF;
                const int gi = static_cast<int>(k / gs);
                const float w = (static_cast<float>(code) - zp_s[r * gstride + gi]) * sc_s[r * gstride + gi];
                a = fmaf(__ldg(x + k), w, a);
            }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (lane == (r & 31)) {
                if (r < 32) fb0 = a;
                else fb1 = a;
            }
        }
        part_lo[0] = static_cast<double>(fb0);
        part_hi[0] = static_cast<double>(fb1);
    }
    __syncthreads();  // every read of the staged codes is done: reuse them as [16][rows] doubles
    double* part = reinterpret_cast<double*>(st);
    if (ws.fixed) {
        if ((lane & 3) == 0) {
            #pragma unroll
            for (int j = 0; j < GROUPS; ++j) {
                if (16 * j + g < rows) part[warp * rows + 16 * j + g] = part_lo[j];
                if (16 * j + g + 8 < rows) part[warp * rows + 16 * j + g + 8] = part_hi[j];
            }
        }
    } else {
        if (lane < rows) part[warp * rows + lane] = part_lo[0];
        if (lane + 32 < rows) part[warp * rows + lane + 32] = part_hi[0];
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < rows) {
        const int i = threadIdx.x;
        double sum = 0.0;
        #pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) sum += part[w * rows + i];
        out[r0 + i] = static_cast<float>(sum);
    }
}

template <int KSMAX, int GSTEPS, int GROUPS, int SETS>
popcornStatus_t launch_i4_mma_t(float* out, const float* x, const uint8_t* q, const float* scale, const float* zero,
                                int64_t N, int64_t K, int64_t gs, int64_t G, int64_t smem, cudaStream_t stream) {
    auto kern = i4_mma_kernel<KSMAX, GSTEPS, GROUPS, SETS>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool known = dev >= 0 && dev < 64;
    if (!known || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kI4MmaStageBytes);
        if (e == cudaSuccess) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
        }
        if (e != cudaSuccess) return record_cuda(e);
        if (known) attr_set[dev] = true;
    }
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(G)), dim3(kMmaThreads),
                                              static_cast<size_t>(smem), stream, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, out, x, q, scale, zero, N, K, gs);
    return (e != cudaSuccess) ? record_cuda(e) : check_launch();
}

// Tensor-path int4 decode: M = 1, K of 1024, 2048 or 4096, group_size a
// multiple of 64 (of 128 at K = 4096) with a warp's K / 16 columns holding
// whole groups (or lying in one), K / group_size % 4 == 0 (16-byte scale
// rows), 16-byte aligned operands, each CTA's rows within kI4MmaStageBytes
// and at most 20 MMAs per warp. Returns false (nothing launched) otherwise.
bool launch_i4_mma(popcornStatus_t* stp, float* out, const float* x, const uint8_t* q, const float* scale,
                   const float* zero, int64_t N, int64_t K, int64_t gs, cudaStream_t stream) {
    if (K != 1024 && K != 2048 && K != 4096) return false;
    const int64_t groups = K / gs;
    if (gs % 64 != 0 || groups % 4 != 0) return false;
    if (!aligned16(x) || !aligned16(q) || !aligned16(scale) || !aligned16(zero)) return false;
    const int64_t ksmax = K / 512;
    const int64_t span = 32 * ksmax;
    if (!(span % gs == 0 || gs % span == 0)) return false;
    const int64_t gsteps = gs >= span ? ksmax : gs / 32;
    const int64_t G = device_sm_count() < N ? device_sm_count() : N;
    const int64_t rows_max = ceil_div(N, G);
    const int64_t pitch = K / 2 + 16;
    const int64_t smem = rows_max * (pitch + 8 * (groups + 4)) + 4 * K;  // + 16 warps x (K / 16) Y words
    if (rows_max > kI4MmaMaxRows || smem > kI4MmaStageBytes) return false;
    if (ceil_div(rows_max, 16) * ksmax > 20) return false;
    popcornStatus_t r = POPCORN_SUCCESS;
    if (ksmax == 2) {
        r = launch_i4_mma_t<2, 2, 4, 2>(out, x, q, scale, zero, N, K, gs, G, smem, stream);
    } else if (ksmax == 4) {
        if (gsteps == 2) return false;  // group 64 at K = 2048: spills at 64 registers; the staged dp4a kernel
        r = launch_i4_mma_t<4, 4, 4, 2>(out, x, q, scale, zero, N, K, gs, G, smem, stream);
    } else {
        // Group 64 at K = 4096 (four flushes per warp) measured slower than
        // i4_stage_kernel: 5.28 against 4.34 us at N = 4096.
        if (rows_max > 32 || gsteps == 2) return false;
        if (gsteps == 4) r = launch_i4_mma_t<8, 4, 2, 4>(out, x, q, scale, zero, N, K, gs, G, smem, stream);
        else r = launch_i4_mma_t<8, 8, 2, 2>(out, x, q, scale, zero, N, K, gs, G, smem, stream);
    }
    *stp = r;
    return true;
}

template <int MT, int U, int R>
popcornStatus_t launch_i4_xs(float* out, const float* x, const uint8_t* q, const float* scale, const float* zero,
                             int64_t M, int64_t N, int64_t K, int64_t gs, cudaStream_t stream) {
    const int64_t gx = ceil_div(N, R);
    const int64_t gy = ceil_div(M, MT);
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)),
                                              dim3(kI4Threads), 0, stream, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, i4_xs_kernel<MT, U, R>, out, x, q, scale, zero, M, N, K, gs);
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

}  // namespace

cudaError_t i4_take_errors(unsigned int* bits) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(bits, g_i4_error, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_i4_error, &zero, sizeof(unsigned int));
    return e;
}

}  // namespace pcb

extern "C" popcornStatus_t popcornDequantizeMatmulGrouped_i4f32(float* out, const float* x, const uint8_t* qweight,
                                                               const float* scale, const float* zero, int64_t M,
                                                               int64_t N, int64_t K, int64_t group_size,
                                                               cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || x == nullptr || qweight == nullptr || scale == nullptr || zero == nullptr) {
        return POPCORN_ERROR_INVALID_VALUE;
    }
    if (M <= 0 || N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (group_size <= 0 || K % group_size != 0) return POPCORN_ERROR_INVALID_VALUE;
    if (K % 2 != 0) return POPCORN_ERROR_INVALID_VALUE;
    // More than four activation rows and >= 2^27 multiply-adds: tensor cores,
    // the group factors applied by the converters.
    if (M > 4 && static_cast<double>(M) * static_cast<double>(N) * static_cast<double>(K) >= 134217728.0 &&
        tc_grouped_supported(qweight, M, N, K, group_size)) {
        return tc_dequant_matmul_grouped(kFmtGroup4, out, x, qweight, scale, zero, M, N, K, group_size, stream);
    }
    const bool aligned = aligned16(x) && (reinterpret_cast<uintptr_t>(qweight) & 7u) == 0 && K % 16 == 0;
    const int64_t slices = ceil_div(K / 16, kI4Threads);
    const bool tiny = M * N * K <= (int64_t{1} << 22);
    const bool grid_ok = ceil_div(M, 4) <= 65535 && ceil_div(N, 2) <= 0x7FFFFFFF;
    if (!tiny && aligned && group_size % 16 == 0 && slices <= 4 && grid_ok) {
        if (M == 1) {
            popcornStatus_t st = POPCORN_SUCCESS;
            if (launch_i4_mma(&st, out, x, qweight, scale, zero, N, K, group_size, stream)) return st;
            if (launch_i4_stage(&st, out, x, qweight, scale, zero, N, K, group_size, stream)) return st;
            if (slices == 1) return launch_i4_xs<1, 1, 8>(out, x, qweight, scale, zero, M, N, K, group_size, stream);
            if (slices == 2) return launch_i4_xs<1, 2, 4>(out, x, qweight, scale, zero, M, N, K, group_size, stream);
            return launch_i4_xs<1, 4, 2>(out, x, qweight, scale, zero, M, N, K, group_size, stream);
        }
        if (M == 2 && slices <= 2) {
            if (slices == 1) return launch_i4_xs<2, 1, 8>(out, x, qweight, scale, zero, M, N, K, group_size, stream);
            return launch_i4_xs<2, 2, 4>(out, x, qweight, scale, zero, M, N, K, group_size, stream);
        }
        if (slices == 1) return launch_i4_xs<4, 1, 4>(out, x, qweight, scale, zero, M, N, K, group_size, stream);
    }
    int64_t blocks = ceil_div(M * N, 256);
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 32;
    if (blocks > cap) blocks = cap;
    i4_seq_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(out, x, qweight, scale, zero, M, N, K,
                                                                     group_size);
    return check_launch();
}

extern "C" popcornStatus_t popcornQuantizeGrouped_f32i4(uint8_t* out, float* scale, float* zero, const float* input,
                                                       int64_t N, int64_t K, int64_t group_size,
                                                       cudaStream_t stream) {
    using namespace pcb;
    if (out == nullptr || scale == nullptr || zero == nullptr || input == nullptr) return POPCORN_ERROR_INVALID_VALUE;
    if (N <= 0 || K <= 0) return POPCORN_SUCCESS;
    if (group_size <= 0 || K % group_size != 0) return POPCORN_ERROR_INVALID_VALUE;
    if (K % 2 != 0) return POPCORN_ERROR_INVALID_VALUE;
    const int64_t items = N * (K / group_size);
    int64_t blocks = ceil_div(items, kI4Warps);
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    if (group_size % 2 == 0) {
        i4_quantize_kernel<true><<<static_cast<unsigned>(blocks), kI4Threads, 0, stream>>>(out, scale, zero, input, N,
                                                                                          K, group_size);
        return check_launch();
    }
    i4_quantize_kernel<false><<<static_cast<unsigned>(blocks), kI4Threads, 0, stream>>>(out, scale, zero, input, N, K,
                                                                                       group_size);
    const popcornStatus_t st = check_launch();
    if (st != POPCORN_SUCCESS) return st;
    int64_t pblocks = ceil_div(N * (K / 2), 256);
    const int64_t pcap = static_cast<int64_t>(device_sm_count()) * 32;
    if (pblocks > pcap) pblocks = pcap;
    i4_pack_kernel<<<static_cast<unsigned>(pblocks), 256, 0, stream>>>(out, scale, zero, input, N, K, group_size);
    return check_launch();
}
