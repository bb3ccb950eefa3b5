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
//  * grouped_mma_kernel -- decode (M = 1, K = 1024, 2048, 4096, group size a
//    multiple of 32): the staged tensor-path layout of gemv_mma_kernel, each
//    group's exact integer sum scaled in double.
//  * grouped_quantize_kernel -- one warp per (row, group): the group max by
//    shuffles with popcorn's NaN-skipping compare, then the codes; bit-
//    identical to popcorn's two kernels, with no temporary buffer.
#include "common.cuh"
#include "mma_frag.cuh"
#include "sm100.cuh"

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

// ------------------------------------------------------- grouped_mma_kernel
// Per-group decode (M = 1, K = 1024, 2048 or 4096, group_size % 32 == 0) on
// the warp-level tensor path: gemv_mma_kernel's staging (each CTA's rows
// copied into shared memory at a pitch of K + 16 by 1-D bulk copies before
// griddepcontrol.wait, two CTAs per SM) and arithmetic (per-warp 30-bit
// fixed-point activations as four base-256 digits, mma.sync s8 column sums),
// with one change: a warp's KSMAX k-steps hold NG = KSMAX / GSTEPS whole
// groups, and the exact integer sum of each group (per row) is multiplied by
// that group's scale in double before it joins the warp's partial. The 16
// warp partials are added in warp order in double and rounded once. Group
// scales are loaded into registers before the wait (weight-side data, like
// the codes). Warps with a non-finite or extreme activation use popcorn's
// per-element form (w = code * scale, fma), lane-strided.
constexpr int kGMmaStageBytes = (228 * 1024 - 2 * 1024) / 2 - 64;
constexpr int kGMaxDevices = 64;  // per-device caches of the launch attributes
constexpr int kGMmaMaxRows = 64;
constexpr unsigned int kGroupedStageTimeoutBit = 0x1000u;

__device__ unsigned int g_grouped_error;

template <int KSMAX, int GSTEPS, int GROUPS, int SETS>
__global__ void __launch_bounds__(kMmaThreads, 2)
grouped_mma_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
                   const float* __restrict__ scale, int64_t N, int64_t K, int64_t gs) {
    constexpr int NG = KSMAX / GSTEPS;  // groups of one warp
    extern __shared__ __align__(16) uint8_t stage[];  // [rows][K + 16]
    __shared__ __align__(8) uint64_t s_full;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t G = gridDim.x;
    const int64_t r0 = N * blockIdx.x / G;
    const int rows = static_cast<int>(N * (blockIdx.x + 1) / G - r0);
    const int k32 = static_cast<int>(K);
    const int pitch = k32 + 16;
    const int steps = k32 >> 5;
    const int64_t ng_row = K / gs;  // groups per row
    const uint32_t full = sm100::smem_addr(&s_full);
    const uint32_t base = sm100::smem_addr(stage);

    if (threadIdx.x == 0) {
        sm100::mbar_init(full, 1);
        sm100::fence_barrier_init();
        sm100::mbar_arrive_expect_tx(full, static_cast<uint32_t>(rows * K));  // < 2^20 - 1
    }
    pdl_launch_dependents();
    __syncthreads();
    if (threadIdx.x < rows) {
        sm100::bulk_load_1d(base + threadIdx.x * pitch, q + (r0 + threadIdx.x) * K, static_cast<uint32_t>(k32), full);
    } else if (threadIdx.x == kMmaThreads - 1) {
        prefetch_l2_range(x, K * static_cast<int64_t>(sizeof(float)), 0, 1);
    }
    // Scales of the groups this lane finishes: rows 16 j + g and 16 j + g + 8,
    // groups grp0 .. grp0 + NG - 1 (rows past the last read the last row's).
    const int g = lane >> 2;
    const int c0 = warp * KSMAX;
    const int64_t grp0 = static_cast<int64_t>(32) * c0 / gs;
    float sc[GROUPS][2][NG];
    #pragma unroll
    for (int j = 0; j < GROUPS; ++j) {
        #pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = min(16 * j + g + 8 * h, rows - 1);
            #pragma unroll
            for (int n = 0; n < NG; ++n) sc[j][h][n] = __ldg(scale + (r0 + row) * ng_row + grp0 + n);
        }
    }
    pdl_wait();
    const WarpScale ws = warp_scale<KSMAX, true>(x, steps, c0, KSMAX, lane);

    if (!sm100::mbar_wait(full, 0, &g_grouped_error, kGroupedStageTimeoutBit)) {
        sm100::mbar_wait(full, 0, &g_grouped_error, kGroupedStageTimeoutBit);
    }

    const int groups = (rows + 15) >> 4;
    double part_lo[GROUPS], part_hi[GROUPS];
    #pragma unroll
    for (int j = 0; j < GROUPS; ++j) part_lo[j] = part_hi[j] = 0.0;
    if (ws.fixed) {
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
            #pragma unroll
            for (int i2 = 0; i2 < GSTEPS; ++i2) {
                const int c = c0 + n * GSTEPS + i2;
                uint32_t b0, b1;
                b_fragment(x, c, ws.up, lane, b0, b1);
                #pragma unroll
                for (int j = 0; j < GROUPS; ++j) {
                    if (j < groups) {
                        int r = 16 * j + mrow;
                        r = r < rows ? r : rows - 1;  // past the last row: read it again, never stored
                        uint32_t a[4];
                        ldmatrix_x4(a, base + r * pitch + 32 * c + mk);
                        mma_s8_16832(d[j][i2 % SETS], a, b0, b1);
                    }
                }
            }
            #pragma unroll
            for (int j = 0; j < GROUPS; ++j) {
                #pragma unroll
                for (int e2 = 1; e2 < SETS; ++e2) {  // exact: |column sum| < 2^22
                    #pragma unroll
                    for (int v = 0; v < 4; ++v) d[j][0][v] += d[j][e2][v];
                }
                double lo, hi;
                combine_digits(d[j][0], ws.s, lo, hi);
                part_lo[j] += lo * static_cast<double>(sc[j][0][n]);
                part_hi[j] += hi * static_cast<double>(sc[j][1][n]);
            }
        }
    } else {
        // popcorn's per-element form (rare); lane r % 32 keeps row r's sum.
        float fb0 = 0.0f, fb1 = 0.0f;
        for (int r = 0; r < rows; ++r) {
            const int8_t* codes = reinterpret_cast<const int8_t*>(stage + r * pitch);
            const float* srow = scale + (r0 + r) * ng_row;
            float a = 0.0f;
            for (int c = c0; c < c0 + KSMAX; ++c) {
                const int k = 32 * c + lane;
                a = fmaf(__ldg(x + k), static_cast<float>(codes[k]) * __ldg(srow + k / gs), a);
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
    __syncthreads();  // every read of the staged rows is done: reuse them as [16][rows] doubles
    double* part = reinterpret_cast<double*>(stage);
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
popcornStatus_t launch_grouped_mma_t(float* out, const float* x, const int8_t* q, const float* scale, int64_t N,
                                     int64_t K, int64_t gs, int64_t G, int64_t smem, cudaStream_t stream) {
    auto kern = grouped_mma_kernel<KSMAX, GSTEPS, GROUPS, SETS>;
    static bool attr_set[kGMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool cached = dev >= 0 && dev < kGMaxDevices;
    if (!cached || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGMmaStageBytes);
        if (e == cudaSuccess) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
        }
        if (e != cudaSuccess) return record_cuda(e);
        if (cached) attr_set[dev] = true;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(G)), dim3(kMmaThreads),
                                        static_cast<size_t>(smem), stream, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, out, x, q, scale, N, K, gs);
    return (e != cudaSuccess) ? record_cuda(e) : check_launch();
}

// Staged per-group decode: M = 1, K of 1024, 2048 or 4096, group_size % 32
// == 0 with a warp's 32 * K / 512 columns holding whole groups (or lying in
// one; at K = 4096 groups of at least 128), each CTA's rows within
// kGMmaStageBytes, at most 16 group scales per lane and 20 MMAs per warp; x
// and the codes 16-byte aligned. Returns false (nothing launched) otherwise.
bool launch_grouped_mma(popcornStatus_t* st, float* out, const float* x, const int8_t* q, const float* scale,
                        int64_t N, int64_t K, int64_t gs, cudaStream_t stream) {
    if (K != 1024 && K != 2048 && K != 4096) return false;
    if (gs % 32 != 0) return false;
    const int64_t ksmax = K / 512;       // k-steps of one warp
    const int64_t span = 32 * ksmax;     // columns of one warp
    if (!(span % gs == 0 || gs % span == 0)) return false;
    const int64_t gsteps = gs >= span ? ksmax : gs / 32;
    const int64_t G = device_sm_count() < N ? device_sm_count() : N;
    const int64_t rows = ceil_div(N, G);
    const int64_t smem = rows * (K + 16);
    if (rows > kGMmaMaxRows || smem > kGMmaStageBytes) return false;
    const int64_t rgroups = ceil_div(rows, 16);
    if (rgroups * ksmax > 20) return false;
    popcornStatus_t r = POPCORN_ERROR_INVALID_VALUE;
    bool done = true;
    if (ksmax == 2) {
        if (gsteps == 1) r = launch_grouped_mma_t<2, 1, 4, 1>(out, x, q, scale, N, K, gs, G, smem, stream);
        else r = launch_grouped_mma_t<2, 2, 4, 1>(out, x, q, scale, N, K, gs, G, smem, stream);
    } else if (ksmax == 4) {
        if (gsteps == 2) r = launch_grouped_mma_t<4, 2, 4, 1>(out, x, q, scale, N, K, gs, G, smem, stream);
        else if (gsteps == 4) r = launch_grouped_mma_t<4, 4, 4, 2>(out, x, q, scale, N, K, gs, G, smem, stream);
        else done = false;  // group_size 32: 32 scales per lane
    } else {
        // K = 4096 holds at most 28 rows. Group size 64 (four scale flushes
        // per warp) measured slower than grouped_xs_kernel: 6.2-6.7 us
        // against 5.4 us at N = 4096.
        if (rows > 32) done = false;
        else if (gsteps == 4) r = launch_grouped_mma_t<8, 4, 2, 2>(out, x, q, scale, N, K, gs, G, smem, stream);
        else if (gsteps == 8) r = launch_grouped_mma_t<8, 8, 2, 4>(out, x, q, scale, N, K, gs, G, smem, stream);
        else done = false;
    }
    if (done) *st = r;
    return done;
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

cudaError_t grouped_take_errors(unsigned int* bits) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(bits, g_grouped_error, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_grouped_error, &zero, sizeof(unsigned int));
    return e;
}

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
        popcornStatus_t st = POPCORN_SUCCESS;
        if (M == 1 && launch_grouped_mma(&st, out, x, qweight, scale, N, K, group_size, stream)) return st;
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
