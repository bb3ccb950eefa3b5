// f32 CUDA-core dequant-matmul path: out[m, n] = scale[n] * sum_k x[m, k] * q[n, k].
//
// Arithmetic follows popcorn's dequantizeMatmulKernel_i8f32
// (src/quantize.cu:18-84): int8 codes widened exactly to f32, products
// accumulated in f32. Kernels:
//
//  * seq_kernel -- tiny problems (launch-bound anyway): one thread per output
//    walks k upward with w = code * scale and acc = fma(x, w, acc), the exact
//    operation sequence of popcorn's kernel, so results are bit-identical to
//    it (and to the oracle's fused variant).
//  * gemv_xs_kernel -- decode (M <= 4): "x-stationary" streaming GEMV. Each
//    thread owns U 16-element slices of K and keeps those activations in
//    registers; every weight row is read with one 16-byte load per thread
//    (256 threads cover 4 KB of a row, fully coalesced), R rows at a time, so
//    a block has R*U*4 KB of weights in flight with no shared-memory staging.
//    The per-channel scale is applied once to the finished sum (it factors
//    out of the k-sum). Per-lane partial sums are combined by a fixed
//    butterfly reduce-scatter across the warp and a fixed-order sum across
//    warps, so results are deterministic; they differ from popcorn's
//    sequential order by f32 rounding only.
//  * gemv_stage_kernel -- decode (M = 1) when every SM's share of the rows
//    fits in 112 KB: the weights are copied into shared memory with cp.async
//    as soon as the kernel starts, before it waits for the previous kernel of
//    the stream, so under programmatic dependent launch the next call's
//    weight stream overlaps this call; same arithmetic and bits as
//    gemv_xs_kernel. Also behind the fused all-gather / all-reduce.
//  * gemv_mma_kernel -- the staged decode for K % 32 == 0, K <= 8192, with
//    the dot products on the warp-level tensor path (mma.sync m16n8k32,
//    s8 x s8 -> s32): activations as four signed base-256 digits of a
//    30-bit fixed point value per warp, exact integer column sums, partials
//    combined in double and rounded once. Takes the place of
//    gemv_stage_kernel (and behind the fused collectives) wherever its rows
//    fit and each warp has at most 20 MMAs.
//  * gemv_kernel -- other aligned shapes (larger K or M): activations staged
//    in shared memory with cp.async, weights streamed per warp.
//  * generic_kernel -- any shape / alignment.
//
// Codes are widened with the exponent trick: byte (code ^ 0x80) in the low
// mantissa byte of 2^23 is the float 2^23 + 128 + code; subtracting
// 2^23 + 128 is exact.
//
// Roofline: HBM. Algorithmic bytes per launch = N*K (int8 weights).
#include "common.cuh"
#include "mma_frag.cuh"
#include "sm100.cuh"

namespace pcb {

// Error bits of bounded waits in this file's kernels (read by
// popcornB200DeviceErrors): kPeerTimeoutBit, kStageTimeoutBit.
__device__ unsigned int g_gemv_error = 0;

namespace {

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

// ---------------------------------------------------------------- seq_kernel
__global__ void __launch_bounds__(256)
seq_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
           const float* __restrict__ scale, int64_t M, int64_t N, int64_t K) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < M * N; t += stride) {
        const int64_t n = t % N;
        const int64_t m = t / N;
        const float* xr = x + m * K;
        const int8_t* qr = q + n * K;
        const float sc = __ldg(scale + n);
        float acc = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float w = static_cast<float>(__ldg(qr + k)) * sc;
            acc = __fmaf_rn(__ldg(xr + k), w, acc);
        }
        out[t] = acc;
    }
}

constexpr int kMaxDevices = 64;
constexpr int kXsSlots = 8;  // decode kernel variants (launch_xs slot numbers)

// ------------------------------------------------------------ gemv_xs_kernel
// Fused collectives (tensor-parallel decode). A call with sequence number e
// (this rank's call count + 1, the same on every rank) sends each output
// value as one 8-byte word {e, f32 bits} into half (e & 1) of the receiving
// rank's area: an aligned 64-bit store is single-copy atomic, so a reader
// that sees the tag e also sees the value, and no flag or fence has to
// follow the data. All-gather: the value of output (m, n) goes to slot
// m * N + n of every other rank. All-reduce: rank r's partial of (m, n) goes
// to slot r * M * N + m * N + n of every rank, its own included. After its
// own outputs, every block polls its share of this rank's slots until they
// carry tag e (bounded), then writes them (all-gather) or their sum in rank
// order (all-reduce) to `out`. A rank is at most one call ahead of another
// (a call ends only when all of its inputs from every rank have arrived), so
// alternating halves keep a faster rank from overwriting slots that a slower
// one has not read yet.
constexpr uint64_t kPeerWaitNs = 1000ull * 1000ull * 1000ull;  // 1 s
constexpr unsigned int kPeerTimeoutBit = 0x100u;
constexpr unsigned int kStageTimeoutBit = 0x200u;  // staged decode weights did not land within 1 s

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned long long tagged(unsigned int e, float v) {
    return (static_cast<unsigned long long>(e) << 32) | __float_as_uint(v);
}

// Waits (until deadline) for slot p to carry tag e; returns false on timeout.
__device__ __forceinline__ bool wait_tag(const unsigned long long* p, unsigned int e, uint64_t deadline, float& v) {
    for (;;) {
        const unsigned long long w = ld_relaxed_sys_u64(p);
        if (static_cast<unsigned int>(w >> 32) == e) {
            v = __uint_as_float(static_cast<unsigned int>(w));
            return true;
        }
        if (global_ns() > deadline) {
            atomicOr(&g_gemv_error, kPeerTimeoutBit);
            return false;
        }
    }
}

// dp2a with unsigned 16-bit halves in a and signed bytes in b.
__device__ __forceinline__ int dp2a_lo_us(uint32_t a, int b, int c) {
    int d;
    asm("dp2a.lo.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_us(uint32_t a, int b, int c) {
    int d;
    asm("dp2a.hi.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Second half of a fused call, run by every block after its own outputs:
// collect this block's share of the values other ranks send, then count the
// block done; the last block advances the call count for the next call.
template <int MODE>
__device__ void peer_finish(const PeerArgs& pa, float* __restrict__ out, int64_t M, int64_t rows, unsigned int e) {
    const int64_t blocks = static_cast<int64_t>(gridDim.x) * gridDim.y;
    const int64_t b = static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x;
    const unsigned long long* mine = pa.recv[pa.rank] + (e & 1u) * pa.half_words;
    const int64_t others = pa.n_total - rows;  // all-gather: columns owned by other ranks
    const int64_t total = (MODE == kPeerGather) ? M * others : M * rows;
    const int64_t j0 = total * b / blocks;
    const int64_t j1 = total * (b + 1) / blocks;
    const uint64_t deadline = global_ns() + kPeerWaitNs;
    for (int64_t j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
        if constexpr (MODE == kPeerGather) {
            const int64_t m = j / others;
            const int64_t c = j - m * others;
            const int64_t idx = m * pa.n_total + (c < pa.n_offset ? c : c + rows);
            float v;
            if (!wait_tag(mine + idx, e, deadline, v)) break;
            out[idx] = v;
        } else {
            float sum = 0.0f;
            bool ok = true;
            for (int p = 0; p < pa.world; ++p) {
                float v;
                if (!wait_tag(mine + static_cast<int64_t>(p) * total + j, e, deadline, v)) {
                    ok = false;
                    break;
                }
                sum = (p == 0) ? v : sum + v;
            }
            if (!ok) break;
            out[j] = sum;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atom_add_acq_rel_gpu(pa.state + 1, 1u) == static_cast<unsigned int>(blocks - 1)) {
        volatile unsigned int* st = pa.state;
        st[1] = 0u;  // ready for the next call
        st[0] = e;
    }
}

constexpr int kXsThreads = 256;
constexpr int kXsWarps = kXsThreads / 32;

// Butterfly reduce-scatter of V values across the warp: afterwards the lanes
// with (lane % (32 / V)) == 0 hold the warp total of value index lane / (32 / V).
template <int V>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[V], int lane) {
    int cnt = V;
    #pragma unroll
    for (int step = 16; step >= 1; step >>= 1) {
        if (cnt > 1) {
            const int half = cnt >> 1;
            const bool upper = (lane & step) != 0;
            #pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < half) {
                    const float send = upper ? v[i] : v[i + half];
                    const float keep = upper ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, step);
                }
            }
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], step);
        }
    }
    return v[0];
}

// MT activation rows (<= 4), U 16-element K slices per thread, R weight rows
// per iteration. Block b owns weight rows [b*rpc, min(N, (b+1)*rpc)).
// PIPE: blocks own several row groups and overlap the next group's loads with
// the current group's math (more registers, two blocks per SM); without it a
// block owns one row group and four blocks fit per SM.
template <int MT, int U, int R, bool PIPE, int MODE = kPeerNone>
__global__ void __launch_bounds__(kXsThreads, (MT * U <= 1 && !PIPE) ? 4 : 2)
gemv_xs_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
               const float* __restrict__ scale, int64_t M, int64_t N, int64_t K, int rpc, const PeerArgs pa) {
    extern __shared__ float part[];  // [rpc][MT][kXsWarps]
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t units = K >> 4;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
    const int64_t r1 = (r0 + rpc < N) ? r0 + rpc : N;
    // Programmatic dependent launch: let the next kernel in the stream start
    // as soon as SM resources free up, and, before waiting for the previous
    // kernel, pull this block's weight rows into L2. A prefetch is only a
    // hint (L2 is the coherence point), so it is safe even if the previous
    // kernel writes these rows; every real read happens after the wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid < kXsWarps && blockIdx.y == 0) {
        // The first two row groups: enough to cover the previous kernel's tail.
        const int64_t bytes = ((r1 - r0) < 2 * R ? (r1 - r0) : 2 * R) * K;
        const int64_t chunk = (bytes + kXsWarps - 1) / kXsWarps;
        const int64_t c0 = (static_cast<int64_t>(tid) * chunk) & ~int64_t(15);
        int64_t c1 = (static_cast<int64_t>(tid + 1) * chunk) & ~int64_t(15);
        if (tid == kXsWarps - 1 || c1 > bytes) c1 = bytes;
        if (c1 > c0) {
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q + r0 * K + c0),
                         "r"(static_cast<uint32_t>(c1 - c0))
                         : "memory");
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // Fused collective: this call's sequence number (the count is advanced
    // by the previous call's last block, so it is stable for this whole grid).
    unsigned int e = 0;
    if constexpr (MODE != kPeerNone) {
        __shared__ unsigned int s_e;
        if (tid == 0) s_e = *reinterpret_cast<volatile unsigned int*>(pa.state) + 1u;
        __syncthreads();
        e = s_e;
    }

    for (int64_t m0 = static_cast<int64_t>(blockIdx.y) * MT; m0 < M; m0 += static_cast<int64_t>(gridDim.y) * MT) {
        // Activations of this thread's K slices, kept in registers.
        float2 xv[MT][U][8];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t unit = tid + static_cast<int64_t>(u) * kXsThreads;
            #pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (unit < units && m0 + m < M) {
                    const float4* p = reinterpret_cast<const float4*>(x + (m0 + m) * K + unit * 16);
                    #pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float4 v = __ldg(p + c);
                        xv[m][u][2 * c] = make_float2(v.x, v.y);
                        xv[m][u][2 * c + 1] = make_float2(v.z, v.w);
                    }
                } else {
                    #pragma unroll
                    for (int c = 0; c < 8; ++c) xv[m][u][c] = make_float2(0.0f, 0.0f);
                }
            }
        }

        // With PIPE, row groups of R are software-pipelined: the next group's
        // loads are in flight while the current group is multiplied and
        // reduced. Without it each group is loaded at the top of its iteration.
        uint4 wn[R][U];
        auto load_group = [&](int64_t rb, uint4 (&dst)[R][U]) {
            if (U == 1 && rb + R <= r1 && units == kXsThreads) {
                // Whole group, every slice in range: no predicates, no zero fill.
                const uint4* p = reinterpret_cast<const uint4*>(q + rb * K) + tid;
                const int64_t row16 = K >> 4;
                #pragma unroll
                for (int r = 0; r < R; ++r)
                    #pragma unroll
                    for (int u = 0; u < U; ++u) dst[r][u] = __ldg(p + r * row16 + u * kXsThreads);
                return;
            }
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t unit = tid + static_cast<int64_t>(u) * kXsThreads;
                    if (rb + r < r1 && unit < units) {
                        dst[r][u] = __ldg(reinterpret_cast<const uint4*>(q + (rb + r) * K) + unit);
                    } else {
                        dst[r][u] = make_uint4(0u, 0u, 0u, 0u);  // code 0
                    }
                }
            }
        };
        // The first row group is requested before anything else is computed
        // (this launch is latency-bound), then the row-group loop runs with
        // the per-group arithmetic as a parameter, so the fixed-point and the
        // float path each keep only their own copy of x live.
        load_group(r0, wn);
        // Without PIPE a block owns exactly one row group (rpc == R).
        auto run_groups = [&](auto&& dot) {
            for (int64_t rb = r0; rb < r1; rb += R) {
                float acc[R * MT];
                if constexpr (PIPE) {
                    uint4 w[R][U];
                    #pragma unroll
                    for (int r = 0; r < R; ++r)
                        #pragma unroll
                        for (int u = 0; u < U; ++u) w[r][u] = wn[r][u];
                    if (rb + R < r1) load_group(rb + R, wn);
                    // The group after next into L2 (its R rows are contiguous):
                    // more bytes in flight than the registers hold. A same-box
                    // A/B, us per call: K = 11008, N = 4096 11.52 -> 10.24;
                    // N = 12288 10.50 -> 10.32; N = 32000 21.9 -> 21.3 (a
                    // distance of three or four groups was slower).
                    if (tid == 0 && rb + 2 * R < r1) {
                        const int64_t nb = ((r1 - rb - 2 * R) < R ? (r1 - rb - 2 * R) : R) * K;
                        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q + (rb + 2 * R) * K),
                                     "r"(static_cast<uint32_t>(nb))
                                     : "memory");
                    }
                    dot(w, acc);
                } else {
                    if (rb != r0) load_group(rb, wn);
                    dot(wn, acc);
                }
                constexpr int V = R * MT;
                const float total = warp_reduce_scatter<V>(acc, lane);
                constexpr int span = 32 / V;
                if ((lane % span) == 0) {
                    const int idx = lane / span;  // = r * MT + m
                    const int r = idx / MT;
                    const int m = idx % MT;
                    if (rb + r < r1) part[((rb + r - r0) * MT + m) * kXsWarps + warp] = total;
                }
            }
        };
        auto dot_float = [&](const uint4 (&w)[R][U], float (&acc)[R * MT]) {
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                float2 a[MT];
                #pragma unroll
                for (int m = 0; m < MT; ++m) a[m] = make_float2(0.0f, 0.0f);
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const uint32_t words[4] = {w[r][u].x, w[r][u].y, w[r][u].z, w[r][u].w};
                    #pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float2 lo, hi;
                        widen4(words[c], lo, hi);
                        #pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            a[m] = __ffma2_rn(xv[m][u][2 * c], lo, a[m]);
                            a[m] = __ffma2_rn(xv[m][u][2 * c + 1], hi, a[m]);
                        }
                    }
                }
                #pragma unroll
                for (int m = 0; m < MT; ++m) acc[r * MT + m] = a[m].x + a[m].y;
            }
        };

        // M = 1: each thread turns its slice of x into 30-bit fixed point
        // X (scaled by a power of two from the slice's max |x|), written as
        // X = hi * 2^16 + lo with hi signed and lo unsigned 16-bit, so one
        // dp2a multiplies two codes by two halves exactly and four dp2a
        // finish a 4-byte weight word: no widening, no float multiply-adds.
        // The thread's int32 sums over its <= 64 columns cannot overflow
        // (|hi| <= 2^14, lo < 2^16, |code| <= 128); they are combined in f32
        // as hi_sum * 2^16 + lo_sum (one rounding) and scaled back by the
        // power of two (exact) before the float reduction across threads. A
        // warp that holds a non-finite x or a slice max outside
        // [2^-90, 2^100] keeps the float path (same NaN/inf behaviour as
        // popcorn's f32 kernel).
        bool fixed = false;
        float up = 1.0f, down = 1.0f;
        if constexpr (MT == 1) {
            // Max of the |x| bit patterns: NaN and inf have the largest.
            uint32_t mb = 0;
            #pragma unroll
            for (int u = 0; u < U; ++u) {
                #pragma unroll
                for (int c = 0; c < 8; ++c) {
                    mb = max(mb, __float_as_uint(xv[0][u][c].x) & 0x7FFFFFFFu);
                    mb = max(mb, __float_as_uint(xv[0][u][c].y) & 0x7FFFFFFFu);
                }
            }
            const bool bad = mb != 0u && (mb < 0x12800000u || mb > 0x71800000u);  // outside [2^-90, 2^100]
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
                for (int c = 0; c < 8; ++c) {
                    const uint32_t a = static_cast<uint32_t>(__float2int_rn(xv[0][u][c].x * up));
                    const uint32_t b = static_cast<uint32_t>(__float2int_rn(xv[0][u][c].y * up));
                    xl[u][c] = __byte_perm(a, b, 0x5410);  // low halves (unsigned)
                    xh[u][c] = __byte_perm(a, b, 0x7632);  // high halves (signed)
                }
            }
            run_groups([&](const uint4 (&w)[R][U], float (&acc)[R * MT]) {
                #pragma unroll
                for (int r = 0; r < R; ++r) {
                    int sh = 0, sl = 0;
                    #pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int words[4] = {static_cast<int>(w[r][u].x), static_cast<int>(w[r][u].y),
                                              static_cast<int>(w[r][u].z), static_cast<int>(w[r][u].w)};
                        #pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            sh = __dp2a_lo(static_cast<int>(xh[u][2 * c]), words[c], sh);
                            sh = __dp2a_hi(static_cast<int>(xh[u][2 * c + 1]), words[c], sh);
                            sl = dp2a_lo_us(xl[u][2 * c], words[c], sl);
                            sl = dp2a_hi_us(xl[u][2 * c + 1], words[c], sl);
                        }
                    }
                    acc[r] = fmaf(static_cast<float>(sh), 65536.0f, static_cast<float>(sl)) * down;
                }
            });
        } else {
            run_groups(dot_float);
        }
        __syncthreads();
        const int nvals = static_cast<int>(r1 - r0) * MT;
        for (int i = tid; i < nvals; i += kXsThreads) {
            const int r = i / MT;
            const int m = i % MT;
            float s = 0.0f;
            #pragma unroll
            for (int wv = 0; wv < kXsWarps; ++wv) s += part[i * kXsWarps + wv];
            if (m0 + m < M) {
                const float val = s * __ldg(scale + r0 + r);
                if constexpr (MODE == kPeerGather) {
                    const int64_t idx = (m0 + m) * pa.n_total + pa.n_offset + r0 + r;
                    out[idx] = val;
                    const int64_t slot = (e & 1u) * pa.half_words + idx;
                    for (int p = 0; p < pa.world; ++p) {
                        if (p != pa.rank) st_relaxed_sys_u64(pa.recv[p] + slot, tagged(e, val));
                    }
                } else if constexpr (MODE == kPeerReduce) {
                    const int64_t slot = (e & 1u) * pa.half_words + pa.rank * M * N + (m0 + m) * N + r0 + r;
                    for (int p = 0; p < pa.world; ++p) st_relaxed_sys_u64(pa.recv[p] + slot, tagged(e, val));
                } else {
                    out[(m0 + m) * N + r0 + r] = val;
                }
            }
        }
        __syncthreads();
    }
    if constexpr (MODE != kPeerNone) peer_finish<MODE>(pa, out, M, N, e);
}

// --------------------------------------------------------------- gemv_kernel
constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kChunk = 4096;               // activations staged per pass (elements)
constexpr int kSeg = 512;                  // weight bytes one warp load covers
constexpr int kSegsPerChunk = kChunk / kSeg;
constexpr int kUnitsPerChunk = kChunk / 4; // 16-byte units per staged row

__device__ __forceinline__ int swz(int u) { return u ^ ((u >> 3) & 7); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
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
                    float4* dst = &xs[m * kUnitsPerChunk + swz(u)];
                    if (row_ok && u * 4 < kn) {
                        cp_async16(dst, xr + u);  // all copies in flight at once
                    } else {
                        *dst = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    }
                }
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
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

// --------------------------------------------------------- gemv_stage_kernel
// Decode GEMV (M = 1) whose weights are copied into shared memory before the
// previous kernel of the stream has finished. One CTA per SM owns a
// contiguous range of at most kStageMaxRows weight rows whose bytes fit in
// kStageBytes of shared memory, so a second CTA -- the next call's, under
// programmatic dependent launch -- fits on the same SM. Right after it starts,
// the CTA hands its rows to the TMA engine as one 1-D bulk copy per row
// (cp.async.bulk, completing on one mbarrier) and asks for x to be pulled
// into L2, then waits for the previous kernel (griddepcontrol.wait), loads x
// and turns it into the same fixed-point (or float) form as gemv_xs_kernel.
// By then the weights have been streaming from HBM while the previous call
// ran. Bulk copies bypass the load/store units, so the next call's weight
// stream does not queue in front of this call's reads of x (per-thread
// 16-byte cp.async copies measured ~12 % slower per call on a B200).
//
// Only the weights (and nothing else) are read before the wait. Kernels that
// let this one start early are this library's matmul kernels, which write
// their outputs and their own scratch but never int8 weight codes or scales;
// the quantizers, which do write them, do not release dependents early.
//
// The per-thread slices, the butterfly reduce-scatter and the fixed-order sum
// across warps are those of gemv_xs_kernel, so the two kernels return the
// same bits.
constexpr int kStageBytes = 112 * 1024;  // weight bytes one CTA stages
constexpr int kStageMaxRows = 64;
constexpr int kStageGroups = 2;
constexpr int kStageThreads = kStageGroups * kXsThreads;

template <int U, int SR, int MODE>
__global__ void __launch_bounds__(kStageThreads, 2)
gemv_stage_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
                  const float* __restrict__ scale, int64_t N, int64_t K, const PeerArgs pa) {
    // [rows_max][K] weight codes, then [rows_max][warps] partial sums, with
    // rows_max = ceil(N / gridDim.x): nothing else in shared memory, so two
    // CTAs of a 4096-wide layer (28 rows x 4 KB) fit on one SM.
    extern __shared__ __align__(16) uint8_t stage[];
    __shared__ unsigned int s_e;
    __shared__ __align__(8) uint64_t s_full;  // completes when every staged row has landed
    // Two groups of 256 threads take alternate rows; within a group thread t
    // owns the K slices t + 256u, as in gemv_xs_kernel.
    const int grp = threadIdx.x / kXsThreads;
    const int tid = threadIdx.x % kXsThreads;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t G = gridDim.x;
    const int64_t r0 = N * blockIdx.x / G;
    const int rows = static_cast<int>(N * (blockIdx.x + 1) / G - r0);
    const int64_t units = K >> 4;
    float* part = reinterpret_cast<float*>(stage + ((N + G - 1) / G) * K);
    const uint32_t full = sm100::smem_addr(&s_full);

    if (threadIdx.x == 0) {
        sm100::mbar_init(full, 1);
        sm100::fence_barrier_init();
        // rows * K <= kStageBytes, far below the 2^20 - 1 limit of a transaction count.
        sm100::mbar_arrive_expect_tx(full, static_cast<uint32_t>(rows * K));
    }
    pdl_launch_dependents();
    __syncthreads();
    if (threadIdx.x < rows) {
        // One contiguous row of K bytes (K % 16 == 0, q 16-byte aligned).
        sm100::bulk_load_1d(sm100::smem_addr(stage + threadIdx.x * K), q + (r0 + threadIdx.x) * K,
                            static_cast<uint32_t>(K), full);
    } else if (threadIdx.x == kStageThreads - 1) {
        prefetch_l2_range(x, K * static_cast<int64_t>(sizeof(float)), 0, 1);
    }
    pdl_wait();

    unsigned int e = 0;
    if constexpr (MODE != kPeerNone) {
        if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile unsigned int*>(pa.state) + 1u;
    }

    // Activations of this thread's K slices (zero beyond K).
    float2 xv[U][8];
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t unit = tid + static_cast<int64_t>(u) * kXsThreads;
        if (unit < units) {
            const float4* p = reinterpret_cast<const float4*>(x + unit * 16);
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 v = __ldg(p + c);
                xv[u][2 * c] = make_float2(v.x, v.y);
                xv[u][2 * c + 1] = make_float2(v.z, v.w);
            }
        } else {
            #pragma unroll
            for (int c = 0; c < 8; ++c) xv[u][c] = make_float2(0.0f, 0.0f);
        }
    }
    // Fixed point unless the warp holds a non-finite x or a slice max outside
    // [2^-90, 2^100] (the rule and scaling of gemv_xs_kernel).
    uint32_t mb = 0;
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        #pragma unroll
        for (int c = 0; c < 8; ++c) {
            mb = max(mb, __float_as_uint(xv[u][c].x) & 0x7FFFFFFFu);
            mb = max(mb, __float_as_uint(xv[u][c].y) & 0x7FFFFFFFu);
        }
    }
    const bool bad = mb != 0u && (mb < 0x12800000u || mb > 0x71800000u);
    const bool fixed = !__any_sync(0xffffffffu, bad);
    float up = 1.0f, down = 1.0f;
    if (fixed && mb != 0u) {
        const int ex = 156 - static_cast<int>(mb >> 23);
        up = __int_as_float((ex + 127) << 23);
        down = __int_as_float((127 - ex) << 23);
    }
    // Bounded wait for the staged rows. A timeout sets kStageTimeoutBit (the
    // launch's results are then invalid) and waits once more, so the CTA does
    // not leave while a copy may still be writing its shared memory.
    if (!sm100::mbar_wait(full, 0, &g_gemv_error, kStageTimeoutBit)) {
        sm100::mbar_wait(full, 0, &g_gemv_error, kStageTimeoutBit);
    }

    // This group's rows (grp, grp + 2, ...) SR at a time; `dot` fills acc[j]
    // with this thread's partial of row row(j) from its own staged chunks.
    auto row = [&](int rg, int j) { return rg + j * kStageGroups; };
    auto run = [&](auto&& dot) {
        for (int rg = grp; rg < rows; rg += SR * kStageGroups) {
            float acc[SR];
            dot(rg, acc);
            const float total = warp_reduce_scatter<SR>(acc, lane);
            constexpr int span = 32 / SR;
            if ((lane % span) == 0) {
                const int r = row(rg, lane / span);
                if (r < rows) part[r * kXsWarps + warp] = total;
            }
        }
    };
    if (fixed) {
        uint32_t xh[U][8], xl[U][8];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            #pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t a = static_cast<uint32_t>(__float2int_rn(xv[u][c].x * up));
                const uint32_t b = static_cast<uint32_t>(__float2int_rn(xv[u][c].y * up));
                xl[u][c] = __byte_perm(a, b, 0x5410);
                xh[u][c] = __byte_perm(a, b, 0x7632);
            }
        }
        run([&](int rg, float (&acc)[SR]) {
            #pragma unroll
            for (int r = 0; r < SR; ++r) {
                int sh = 0, sl = 0;
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t unit = tid + static_cast<int64_t>(u) * kXsThreads;
                    if (row(rg, r) < rows && unit < units) {
                        const uint4 w = *reinterpret_cast<const uint4*>(stage + row(rg, r) * K + unit * 16);
                        const int words[4] = {static_cast<int>(w.x), static_cast<int>(w.y), static_cast<int>(w.z),
                                              static_cast<int>(w.w)};
                        #pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            sh = __dp2a_lo(static_cast<int>(xh[u][2 * c]), words[c], sh);
                            sh = __dp2a_hi(static_cast<int>(xh[u][2 * c + 1]), words[c], sh);
                            sl = dp2a_lo_us(xl[u][2 * c], words[c], sl);
                            sl = dp2a_hi_us(xl[u][2 * c + 1], words[c], sl);
                        }
                    }
                }
                acc[r] = fmaf(static_cast<float>(sh), 65536.0f, static_cast<float>(sl)) * down;
            }
        });
    } else {
        run([&](int rg, float (&acc)[SR]) {
            #pragma unroll
            for (int r = 0; r < SR; ++r) {
                float2 a = make_float2(0.0f, 0.0f);
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t unit = tid + static_cast<int64_t>(u) * kXsThreads;
                    if (row(rg, r) < rows && unit < units) {
                        const uint4 w = *reinterpret_cast<const uint4*>(stage + row(rg, r) * K + unit * 16);
                        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
                        #pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            float2 lo, hi;
                            widen4(words[c], lo, hi);
                            a = __ffma2_rn(xv[u][2 * c], lo, a);
                            a = __ffma2_rn(xv[u][2 * c + 1], hi, a);
                        }
                    }
                }
                acc[r] = a.x + a.y;
            }
        });
    }
    __syncthreads();
    if constexpr (MODE != kPeerNone) e = s_e;
    for (int i = threadIdx.x; i < rows; i += kStageThreads) {
        float sum = 0.0f;
        #pragma unroll
        for (int wv = 0; wv < kXsWarps; ++wv) sum += part[i * kXsWarps + wv];
        const float val = sum * __ldg(scale + r0 + i);
        if constexpr (MODE == kPeerGather) {
            const int64_t idx = pa.n_offset + r0 + i;
            out[idx] = val;
            const int64_t slot = (e & 1u) * pa.half_words + idx;
            for (int p = 0; p < pa.world; ++p) {
                if (p != pa.rank) st_relaxed_sys_u64(pa.recv[p] + slot, tagged(e, val));
            }
        } else if constexpr (MODE == kPeerReduce) {
            const int64_t slot = (e & 1u) * pa.half_words + pa.rank * N + r0 + i;
            for (int p = 0; p < pa.world; ++p) st_relaxed_sys_u64(pa.recv[p] + slot, tagged(e, val));
        } else {
            out[r0 + i] = val;
        }
    }
    if constexpr (MODE != kPeerNone) {
        __syncthreads();
        peer_finish<MODE>(pa, out, 1, N, e);
    }
}

// ---------------------------------------------------------- gemv_mma_kernel
// The staged decode GEMV (M = 1, K % 32 == 0, K <= 8192) with its dot
// products on the warp-level tensor path: mma.sync m16n8k32, signed 8-bit A
// and B, s32 accumulate. Staging is gemv_stage_kernel's (rows copied into
// shared memory by 1-D bulk copies before griddepcontrol.wait, two CTAs per
// SM so the next call's rows stream in during this call), except that rows
// sit K + 16 bytes apart: K % 32 == 0 makes the pitch an odd multiple of 16
// bytes, so the eight rows an ldmatrix phase reads fall in eight different
// 16-byte bank groups.
//
// K splits into 32-wide k-steps; warp w owns the contiguous steps
// [w S / 16, (w + 1) S / 16), S = K / 32, for every row of the CTA. Its activations become 32-bit fixed point
// X = rint(x 2^s) with one power of two per warp (max |X| < 2^30), written
// as four signed bytes X = sum_d d_d 256^d, d_d in [-128, 127] (the bytes of
// X + 0x80808080, each xor 0x80). B column n < 4 of a k-step holds digit n
// of the step's 32 activations, columns 4..7 are zero; A is 16 weight rows x
// 32 codes from ldmatrix. The four int32 column sums of a row are exact
// (|code * digit| <= 2^14, at most 16 x 32 terms per warp at K = 8192), so
// the warp's partial is the exact integer sum_d 256^d D_d times 2^-s, formed
// in double. The partials of the 16 warps are added in warp order in double
// and rounded once after the channel scale: the result is the dot product of
// the codes with x rounded to ~2^-30 of each warp's max |x|, correctly
// rounded -- closer to the exact product than popcorn's f32 sum, and the
// same bits however the rows are split over CTAs or ranks. A warp whose
// activations hold a non-finite value or a max |x| outside [2^-90, 2^100]
// adds its steps in f32 instead (codes widened exactly), so NaN and
// infinities propagate as in popcorn's.
// Staged bytes (rows x (K + 16)) of one CTA: two CTAs, each with 1 KB of
// reserved and a few bytes of static shared memory, fit in an SM's 228 KB.
constexpr int kMmaStageBytes = (228 * 1024 - 2 * 1024) / 2 - 64;

// Channel-scaled result of row i (sum of the 16 warp partials in warp
// order), stored to out or sent to the peers.
template <int MODE>
__device__ __forceinline__ void finish_row(float* out, const PeerArgs& pa, int64_t N, int64_t row, double sum,
                                           float sc, unsigned int e) {
    const float val = static_cast<float>(sum * static_cast<double>(sc));
    if constexpr (MODE == kPeerGather) {
        const int64_t idx = pa.n_offset + row;
        out[idx] = val;
        const int64_t slot = (e & 1u) * pa.half_words + idx;
        for (int p = 0; p < pa.world; ++p) {
            if (p != pa.rank) st_relaxed_sys_u64(pa.recv[p] + slot, tagged(e, val));
        }
    } else if constexpr (MODE == kPeerReduce) {
        const int64_t slot = (e & 1u) * pa.half_words + pa.rank * N + row;
        for (int p = 0; p < pa.world; ++p) st_relaxed_sys_u64(pa.recv[p] + slot, tagged(e, val));
    } else {
        out[row] = val;
    }
}

// KSMAX: most k-steps of one warp (K / 32 / 16, rounded up), EVEN: every
// warp has exactly KSMAX (K = 512 KSMAX); GROUPS: most
// 16-row groups of a CTA; SETS: accumulators per group that consecutive
// steps alternate between, so no chain of dependent MMAs is long.
template <int KSMAX, bool EVEN, int GROUPS, int SETS, int MODE>
__global__ void __launch_bounds__(kMmaThreads, 2)
gemv_mma_kernel(float* __restrict__ out, const float* __restrict__ x, const int8_t* __restrict__ q,
                const float* __restrict__ scale, int64_t N, int64_t K, const PeerArgs pa) {
    extern __shared__ __align__(16) uint8_t stage[];  // [rows][K + 16]
    __shared__ unsigned int s_e;
    __shared__ __align__(8) uint64_t s_full;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t G = gridDim.x;
    const int64_t r0 = N * blockIdx.x / G;
    const int rows = static_cast<int>(N * (blockIdx.x + 1) / G - r0);
    const int k32 = static_cast<int>(K);
    const int pitch = k32 + 16;
    const int steps = k32 >> 5;
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
    // Channel scales of the rows a thread will finish (weight-side, like the rows).
    const float sc_row = static_cast<int>(threadIdx.x) < rows ? __ldg(scale + r0 + threadIdx.x) : 0.0f;
    pdl_wait();
    if constexpr (MODE != kPeerNone) {
        if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile unsigned int*>(pa.state) + 1u;
    }
    const int c0 = EVEN ? warp * KSMAX : warp * steps / kMmaWarps;
    const int c1 = EVEN ? c0 + KSMAX : (warp + 1) * steps / kMmaWarps;
    const WarpScale ws = warp_scale<KSMAX, EVEN>(x, steps, c0, c1 - c0, lane);

    if (!sm100::mbar_wait(full, 0, &g_gemv_error, kStageTimeoutBit)) {
        sm100::mbar_wait(full, 0, &g_gemv_error, kStageTimeoutBit);
    }

    // This warp's partials, lane (g, t = 0) holding rows 16 j + g and 16 j + g + 8.
    const int g = lane >> 2;
    const int groups = (rows + 15) >> 4;
    double part_lo[GROUPS], part_hi[GROUPS];
    if (ws.fixed) {
        int d[GROUPS][SETS][4];
        #pragma unroll
        for (int j = 0; j < GROUPS; ++j) {
            #pragma unroll
            for (int e2 = 0; e2 < SETS; ++e2) d[j][e2][0] = d[j][e2][1] = d[j][e2][2] = d[j][e2][3] = 0;
        }
        // ldmatrix row addresses of this lane: matrix i = lane / 8 covers rows
        // + 8 (i & 1), codes + 16 (i >> 1); row lane % 8 of it.
        const int mi = lane >> 3;
        const int mrow = (lane & 7) + 8 * (mi & 1);
        const int mk = 16 * (mi >> 1);
        // Branch-free over the KSMAX steps: a step past the end multiplies
        // the codes of step steps - 1 by zero digits.
        #pragma unroll
        for (int i = 0; i < KSMAX; ++i) {
            const int cc = EVEN ? c0 + i : min(c0 + i, steps - 1);
            uint32_t b0, b1;
            b_fragment(x, cc, ws.up, lane, b0, b1);
            if (!EVEN && c0 + i >= c1) b0 = b1 = 0u;
            #pragma unroll
            for (int j = 0; j < GROUPS; ++j) {
                if (j < groups) {
                    int r = 16 * j + mrow;
                    r = r < rows ? r : rows - 1;  // past the last row: read it again, never stored
                    uint32_t a[4];
                    ldmatrix_x4(a, base + r * pitch + 32 * cc + mk);
                    mma_s8_16832(d[j][i % SETS], a, b0, b1);
                }
            }
        }
        #pragma unroll
        for (int j = 0; j < GROUPS; ++j) {
            #pragma unroll
            for (int e2 = 1; e2 < SETS; ++e2) {  // exact: |column sum| < 2^23
                #pragma unroll
                for (int v = 0; v < 4; ++v) d[j][0][v] += d[j][e2][v];
            }
            combine_digits(d[j][0], ws.s, part_lo[j], part_hi[j]);
        }
    } else {
        // f32 form (rare); lane r % 32 keeps row r's sum.
        float fb0 = 0.0f, fb1 = 0.0f;
        for (int r = 0; r < rows; ++r) {
            const float a = warp_row_f32(x, reinterpret_cast<const int8_t*>(stage + r * pitch), c0, c1, lane);
            if (lane == (r & 31)) {
                if (r < 32) fb0 = a;
                else fb1 = a;
            }
        }
        #pragma unroll
        for (int j = 0; j < GROUPS; ++j) part_lo[j] = part_hi[j] = 0.0;
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
    unsigned int e = 0;
    if constexpr (MODE != kPeerNone) e = s_e;
    if (static_cast<int>(threadIdx.x) < rows) {
        const int i = threadIdx.x;
        double sum = 0.0;
        #pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) sum += part[w * rows + i];
        finish_row<MODE>(out, pa, N, r0 + i, sum, sc_row, e);
    }
    if constexpr (MODE != kPeerNone) {
        __syncthreads();
        peer_finish<MODE>(pa, out, 1, N, e);
    }
}

// ------------------------------------------------------------ generic_kernel
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

// ------------------------------------------------------------------- host
bool g_smem_set[kMaxDevices][3] = {};

// Up to this many multiply-adds, with K at most kSeqMaxK, the sequential
// kernel runs (bit-identical to popcorn's kernel; the call is launch-bound at
// this size). Longer rows go to the parallel kernels even when small: one
// thread walking 4096 codes serially takes hundreds of microseconds.
constexpr int64_t kSeqMaxMacs = int64_t(1) << 22;
constexpr int64_t kSeqMaxK = 256;

bool vector_ok(const float* x, const int8_t* q, int64_t K) {
    return (K % 16 == 0) && aligned16(x) && aligned16(q);
}

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

// Rows per block for the x-stationary kernel so that the whole grid is
// resident at once (one wave).
template <typename Kern>
int xs_rows_per_block(Kern kernel, int slot, int64_t N) {
    static int occ_cache[kMaxDevices][16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int occ = (dev >= 0 && dev < kMaxDevices) ? occ_cache[dev][slot] : 0;
    if (occ == 0) {
        // Partial sums take at most 256 rows x 4 x 8 floats of shared memory.
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kXsThreads, 32 * 1024) != cudaSuccess ||
            occ < 1) {
            occ = 2;
        }
        if (dev >= 0 && dev < kMaxDevices) occ_cache[dev][slot] = occ;
    }
    const int64_t blocks = static_cast<int64_t>(device_sm_count()) * occ;
    int64_t rpc = ceil_div(N, blocks);
    if (rpc < 1) rpc = 1;
    if (rpc > 256) rpc = 256;
    return static_cast<int>(rpc);
}

template <int MT, int U, int R>
popcornStatus_t launch_xs(int slot, float* out, const float* x, const int8_t* q, const float* scale, int64_t M,
                          int64_t N, int64_t K, cudaStream_t stream, PeerMode mode = kPeerNone,
                          const PeerArgs* peer = nullptr) {
    // One row group of R rows per block while a single wave of resident
    // blocks holds the grid (every thread has all its loads in flight at
    // once); otherwise fewer, pipelined blocks that stream several groups.
    int rpc = xs_rows_per_block(gemv_xs_kernel<MT, U, R, false>, 2 * slot, N);
    const bool pipe = rpc > R;
    if (pipe) rpc = xs_rows_per_block(gemv_xs_kernel<MT, U, R, true>, 2 * slot + 1, N);
    if (rpc < R) rpc = R;
    const int smem = rpc * MT * kXsWarps * static_cast<int>(sizeof(float));
    const int64_t gx = ceil_div(N, rpc);
    int64_t gy = ceil_div(M, MT);
    if (gy > 65535) gy = 65535;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
    cfg.blockDim = dim3(kXsThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (mode != kPeerNone) {
        // Fused collective: plain stream order (the block counter and call
        // count must not be shared with an overlapping launch), and every
        // block resident at once, since blocks wait for other ranks' data.
        using Kernel = void (*)(float*, const float*, const int8_t*, const float*, int64_t, int64_t, int64_t, int,
                                const PeerArgs);
        Kernel kern;
        if (mode == kPeerGather) {
            kern = pipe ? gemv_xs_kernel<MT, U, R, true, kPeerGather> : gemv_xs_kernel<MT, U, R, false, kPeerGather>;
        } else {
            kern = pipe ? gemv_xs_kernel<MT, U, R, true, kPeerReduce> : gemv_xs_kernel<MT, U, R, false, kPeerReduce>;
        }
        static int resident_cache[kMaxDevices][kXsSlots * 4] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        const int key = slot * 4 + (mode == kPeerGather ? 0 : 2) + (pipe ? 1 : 0);
        int occ = (dev >= 0 && dev < kMaxDevices) ? resident_cache[dev][key] : 0;
        if (occ == 0) {
            // Partial sums take at most 256 rows x 4 x 8 floats of shared memory.
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kXsThreads, 32 * 1024);
            if (e != cudaSuccess) return record_cuda(e);
            if (dev >= 0 && dev < kMaxDevices) resident_cache[dev][key] = occ;
        }
        if (gx * gy > static_cast<int64_t>(occ) * device_sm_count()) return POPCORN_ERROR_INVALID_VALUE;
        cfg.numAttrs = 0;
        e = cudaLaunchKernelEx(&cfg, kern, out, x, q, scale, M, N, K, rpc, *peer);
    } else {
        const PeerArgs none = {};
        e = pipe ? cudaLaunchKernelEx(&cfg, gemv_xs_kernel<MT, U, R, true>, out, x, q, scale, M, N, K, rpc, none)
                 : cudaLaunchKernelEx(&cfg, gemv_xs_kernel<MT, U, R, false>, out, x, q, scale, M, N, K, rpc, none);
    }
    if (e != cudaSuccess) return record_cuda(e);
    return check_launch();
}

// Staged decode GEMV (M = 1): one CTA per SM while every CTA's rows fit in
// kStageBytes; returns false (nothing launched) when they do not.
template <int U, int SR, int MODE>
bool launch_stage_t(popcornStatus_t* st, float* out, const float* x, const int8_t* q, const float* scale, int64_t N,
                    int64_t K, cudaStream_t stream, const PeerArgs* peer) {
    const int64_t G = device_sm_count() < N ? device_sm_count() : N;
    const int64_t rows = ceil_div(N, G);
    if (rows > kStageMaxRows || rows * K > kStageBytes) return false;
    const int64_t smem = rows * K + rows * kXsWarps * static_cast<int64_t>(sizeof(float));
    auto kern = gemv_stage_kernel<U, SR, MODE>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool cached = dev >= 0 && dev < kMaxDevices;
    if (!cached || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kStageBytes + kStageMaxRows * kXsWarps * static_cast<int>(sizeof(float)));
        if (e == cudaSuccess) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
        }
        if (e != cudaSuccess) {
            *st = record_cuda(e);
            return true;
        }
        if (cached) attr_set[dev] = true;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(G)), dim3(kStageThreads),
                                        static_cast<size_t>(smem), stream, attr);
    const PeerArgs none = {};
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, out, x, q, scale, N, K, peer != nullptr ? *peer : none);
    *st = (e != cudaSuccess) ? record_cuda(e) : check_launch();
    return true;
}

template <int KSMAX, bool EVEN, int GROUPS, int SETS, int MODE>
popcornStatus_t launch_mma_t(float* out, const float* x, const int8_t* q, const float* scale, int64_t N, int64_t K,
                             int64_t G, int64_t smem, cudaStream_t stream, const PeerArgs* peer) {
    auto kern = gemv_mma_kernel<KSMAX, EVEN, GROUPS, SETS, MODE>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool cached = dev >= 0 && dev < kMaxDevices;
    if (!cached || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaStageBytes);
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
    const PeerArgs none = {};
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, out, x, q, scale, N, K, peer != nullptr ? *peer : none);
    return (e != cudaSuccess) ? record_cuda(e) : check_launch();
}

// Staged decode GEMV on the tensor pipe: K % 32 == 0, K <= 8192, and every
// CTA's rows (at most kStageMaxRows) within kMmaStageBytes at a pitch of
// K + 16; returns false (nothing launched) otherwise.
template <int MODE>
bool launch_mma(popcornStatus_t* st, float* out, const float* x, const int8_t* q, const float* scale, int64_t N,
                int64_t K, cudaStream_t stream, const PeerArgs* peer) {
    if (K < 32 || K > 8192 || K % 32 != 0) return false;
    const int64_t G = device_sm_count() < N ? device_sm_count() : N;
    const int64_t rows = ceil_div(N, G);
    // The staged rows, later reused for 16 doubles per row.
    const int64_t smem = rows * (K + 16 > 128 ? K + 16 : 128);
    if (rows > kStageMaxRows || smem > kMmaStageBytes) return false;
    const int64_t per_warp = ceil_div(K / 32, kMmaWarps);  // k-steps of one warp
    // Past ~20 MMAs per warp (16-row groups x k-steps) the legacy tensor
    // path's issue time outweighs what it saves: K = 3072 at 56 rows per CTA
    // took 9.8 us against 8.0 us on the CUDA-core kernels.
    if (ceil_div(rows, 16) * per_warp > 20) return false;
    // K a multiple of 512: every warp has the same steps (per_warp).
    const bool even = (K / 32) % kMmaWarps == 0;
    const bool wide = rows > 32;  // more than two 16-row groups
    popcornStatus_t r = POPCORN_SUCCESS;
#define PCB_MMA(KS, EV, GR, SE) r = launch_mma_t<KS, EV, GR, SE, MODE>(out, x, q, scale, N, K, G, smem, stream, peer)
    if (even && per_warp <= 4) {
        switch (per_warp) {
            case 1: PCB_MMA(1, true, 4, 1); break;
            case 2: PCB_MMA(2, true, 4, 2); break;
            case 3: PCB_MMA(3, true, 4, 2); break;
            default: PCB_MMA(4, true, 4, 2); break;
        }
    } else if (even && per_warp <= 6 && wide) {  // K = 2560, 3072: up to 44 rows
        if (per_warp == 5) PCB_MMA(5, true, 4, 2);
        else PCB_MMA(6, true, 4, 2);
    } else if (even && (per_warp <= 8 || per_warp % 2 == 0)) {  // at most 32 rows from here on
        switch (per_warp) {
            case 5: PCB_MMA(5, true, 2, 4); break;
            case 6: PCB_MMA(6, true, 2, 4); break;
            case 7: PCB_MMA(7, true, 2, 4); break;
            case 8: PCB_MMA(8, true, 2, 4); break;
            case 10: PCB_MMA(10, true, 2, 4); break;
            case 12: PCB_MMA(12, true, 2, 4); break;
            case 14: PCB_MMA(14, true, 2, 4); break;
            default: PCB_MMA(16, true, 2, 4); break;
        }
    } else if (per_warp <= 2) {
        PCB_MMA(2, false, 4, 2);
    } else if (per_warp <= 4) {
        PCB_MMA(4, false, 4, 2);
    } else if (per_warp <= 8 && wide) {
        PCB_MMA(8, false, 4, 2);
    } else if (per_warp <= 8) {
        PCB_MMA(8, false, 2, 4);
    } else {
        PCB_MMA(16, false, 2, 4);  // K > 4096: at most 27 rows
    }
#undef PCB_MMA
    *st = r;
    return true;
}

// K % 16 == 0, K <= 8192 (two slices per thread fit in 64 registers),
// 16-byte aligned x and q (vector_ok).
template <int MODE>
bool launch_stage(popcornStatus_t* st, float* out, const float* x, const int8_t* q, const float* scale, int64_t N,
                  int64_t K, cudaStream_t stream, const PeerArgs* peer = nullptr) {
    if (launch_mma<MODE>(st, out, x, q, scale, N, K, stream, peer)) return true;
    const int64_t slices = ceil_div(K / 16, kXsThreads);
    if (slices == 1) return launch_stage_t<1, 8, MODE>(st, out, x, q, scale, N, K, stream, peer);
    if (slices == 2) return launch_stage_t<2, 4, MODE>(st, out, x, q, scale, N, K, stream, peer);
    return false;
}

}  // namespace

cudaError_t gemv_take_errors(unsigned int* bits) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(bits, g_gemv_error, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(unsigned int));
    return e;
}

bool peer_supported(const float* x, const int8_t* q, int64_t M, int64_t K) {
    return M >= 1 && M <= 4 && vector_ok(x, q, K) && ceil_div(K / 16, kXsThreads) <= (M == 1 ? 4 : (M == 2 ? 2 : 1));
}

popcornStatus_t peer_dequant_matmul(PeerMode mode, const PeerArgs& pa, float* out, const float* x, const int8_t* q,
                                    const float* scale, int64_t M, int64_t rows, int64_t K, cudaStream_t stream) {
    const int64_t slices = ceil_div(K / 16, kXsThreads);
    if (M == 1) {
        popcornStatus_t st = POPCORN_SUCCESS;
        if (mode == kPeerGather && launch_stage<kPeerGather>(&st, out, x, q, scale, rows, K, stream, &pa)) return st;
        if (mode == kPeerReduce && launch_stage<kPeerReduce>(&st, out, x, q, scale, rows, K, stream, &pa)) return st;
        if (slices == 1) return launch_xs<1, 1, 8>(0, out, x, q, scale, M, rows, K, stream, mode, &pa);
        if (slices == 2) return launch_xs<1, 2, 4>(1, out, x, q, scale, M, rows, K, stream, mode, &pa);
        if (slices == 3) return launch_xs<1, 3, 2>(6, out, x, q, scale, M, rows, K, stream, mode, &pa);
        return launch_xs<1, 4, 2>(2, out, x, q, scale, M, rows, K, stream, mode, &pa);
    }
    if (M == 2) {
        if (slices == 1) return launch_xs<2, 1, 8>(3, out, x, q, scale, M, rows, K, stream, mode, &pa);
        return launch_xs<2, 2, 4>(4, out, x, q, scale, M, rows, K, stream, mode, &pa);
    }
    return launch_xs<4, 1, 4>(5, out, x, q, scale, M, rows, K, stream, mode, &pa);
}

int simt_launch_count(const float*, const int8_t*, int64_t M, int64_t N, int64_t K) {
    return (M > 0 && N > 0 && K > 0) ? 1 : 0;
}

popcornStatus_t simt_dequant_matmul(float* out, const float* x, const int8_t* q, const float* scale,
                                    int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    const bool tiny = (M * N <= kSeqMaxMacs) && (K <= kSeqMaxMacs / (M * N)) && K <= kSeqMaxK;
    if (tiny) {
        int64_t blocks = ceil_div(M * N, 256);
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
        if (blocks > cap) blocks = cap;
        seq_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(out, x, q, scale, M, N, K);
        return check_launch();
    }
    if (!vector_ok(x, q, K)) {
        int64_t blocks = ceil_div(M * N, 8);
        const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
        if (blocks > cap) blocks = cap;
        generic_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(out, x, q, scale, M, N, K);
        return check_launch();
    }
    const int64_t units = K / 16;
    const int64_t slices = ceil_div(units, kXsThreads);  // U needed
    popcornStatus_t st = POPCORN_SUCCESS;
    if (M == 1 && slices <= 4 && launch_stage<kPeerNone>(&st, out, x, q, scale, N, K, stream)) return st;
    if (M == 1 && slices <= 4) {
        if (slices == 1) return launch_xs<1, 1, 8>(0, out, x, q, scale, M, N, K, stream);
        if (slices == 2) return launch_xs<1, 2, 4>(1, out, x, q, scale, M, N, K, stream);
        if (slices == 3) return launch_xs<1, 3, 2>(6, out, x, q, scale, M, N, K, stream);
        return launch_xs<1, 4, 2>(2, out, x, q, scale, M, N, K, stream);
    }
    if (M == 2 && slices <= 2) {
        if (slices == 1) return launch_xs<2, 1, 8>(3, out, x, q, scale, M, N, K, stream);
        return launch_xs<2, 2, 4>(4, out, x, q, scale, M, N, K, stream);
    }
    // Up to eight rows: two row groups of four (grid.y = 2) read each weight
    // row twice, mostly from L2; still far ahead of gemv_kernel here.
    if (M <= 8 && slices == 1) return launch_xs<4, 1, 4>(5, out, x, q, scale, M, N, K, stream);
    if (M == 1) return launch_gemv<1, 2>(0, out, x, q, scale, M, N, K, stream);
    if (M == 2) return launch_gemv<2, 2>(1, out, x, q, scale, M, N, K, stream);
    return launch_gemv<4, 2>(2, out, x, q, scale, M, N, K, stream);
}

}  // namespace pcb
