// Warp-level int8 tensor-path helpers of the staged decode kernels
// (gemv.cu, grouped.cu, int4.cu): mma.sync m16n8k32 s8 x s8 -> s32 with the weight
// codes as A (16 rows x 32 codes from ldmatrix) and the activations as B
// (columns 0..3 the four signed base-256 digits of a per-warp 30-bit fixed
// point value, columns 4..7 zero).
#pragma once

#include "common.cuh"

namespace pcb {

constexpr int kMmaWarps = 16;
constexpr int kMmaThreads = kMmaWarps * 32;

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The same with unsigned 8-bit A (int4 codes widened to bytes).
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&a)[4], uint32_t saddr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(saddr));
}

// Per-warp fixed-point scaling of the activations a warp owns.
struct WarpScale {
    bool fixed;  // false: non-finite or extreme values, use the f32 form
    int s;       // X = rint(x 2^s)
    float up;    // 2^s
};

// Lane (g, t) = (lane / 4, lane % 4) reads, for k-step c, the four
// activations at 32 c + 4 t + 16 h, h = g / 4 (the first half of the step
// for g < 4, the second above): KSMAX steps c = c0 + i, those at i >= cnt
// masked out. The loads are unconditional (a step past the end reads step
// steps - 1) so that all of them are in flight at once.
template <int KSMAX, bool EVEN>
__device__ __forceinline__ WarpScale warp_scale(const float* x, int steps, int c0, int cnt, int lane) {
    const int g = lane >> 2;
    const float4* xl = reinterpret_cast<const float4*>(x + 4 * (lane & 3) + 16 * (g >> 2));
    uint32_t mb = 0;
    #pragma unroll
    for (int i = 0; i < KSMAX; ++i) {
        const float4 v = __ldg(xl + 8 * (EVEN ? c0 + i : min(c0 + i, steps - 1)));
        const uint32_t keep = (EVEN || i < cnt) ? 0x7FFFFFFFu : 0u;
        mb = max(mb, max(max(__float_as_uint(v.x) & keep, __float_as_uint(v.y) & keep),
                         max(__float_as_uint(v.z) & keep, __float_as_uint(v.w) & keep)));
    }
    mb = __reduce_max_sync(0xffffffffu, mb);
    WarpScale ws;
    ws.fixed = mb == 0u || (mb >= 0x12800000u && mb <= 0x71800000u);
    // max |x| 2^s in [2^29, 2^30): s = 29 - exponent of max |x|.
    ws.s = mb == 0u ? 0 : 29 - (static_cast<int>(mb >> 23) - 127);
    ws.up = mb == 0u ? 1.0f : __int_as_float((ws.s + 127) << 23);
    return ws;
}

// B fragment of k-step c: digit g % 4 of this lane's four activations in
// b0 (first half of the step) and b1 (second half) for g < 4, zero above.
__device__ __forceinline__ void b_fragment(const float* x, int c, float up, int lane, uint32_t& b0, uint32_t& b1) {
    const int g = lane >> 2;
    const float4 v = __ldg(reinterpret_cast<const float4*>(x + 32 * c + 4 * (lane & 3) + 16 * (g >> 2)));
    const uint32_t sel = static_cast<uint32_t>((g & 3) | (((g & 3) + 4) << 4));
    const uint32_t y0 = static_cast<uint32_t>(__float2int_rn(v.x * up)) + 0x80808080u;
    const uint32_t y1 = static_cast<uint32_t>(__float2int_rn(v.y * up)) + 0x80808080u;
    const uint32_t y2 = static_cast<uint32_t>(__float2int_rn(v.z * up)) + 0x80808080u;
    const uint32_t y3 = static_cast<uint32_t>(__float2int_rn(v.w * up)) + 0x80808080u;
    const uint32_t bw = __byte_perm(__byte_perm(y0, y1, sel), __byte_perm(y2, y3, sel), 0x5410) ^ 0x80808080u;
    const uint32_t odd = __shfl_down_sync(0xffffffffu, bw, 16);  // digit g of the step's second half
    b0 = g < 4 ? bw : 0u;
    b1 = g < 4 ? odd : 0u;
}

// Column sums d0, d1 = digits 2t, 2t + 1 of row g (d2, d3: row g + 8), lanes
// t = 0, 1 holding digits 0-1 and 2-3: lane t = 0 gets the exact partials
// of rows g and g + 8 times 2^-s.
__device__ __forceinline__ void combine_digits(const int (&d)[4], int s, double& lo_row, double& hi_row) {
    const double down = __longlong_as_double(static_cast<long long>(1023 - s) << 52);
    const double l0 = static_cast<double>(d[0]) + 256.0 * static_cast<double>(d[1]);
    const double l8 = static_cast<double>(d[2]) + 256.0 * static_cast<double>(d[3]);
    const double h0 = __shfl_down_sync(0xffffffffu, l0, 1);
    const double h8 = __shfl_down_sync(0xffffffffu, l8, 1);
    lo_row = (h0 * 65536.0 + l0) * down;
    hi_row = (h8 * 65536.0 + l8) * down;
}

// f32 form of a warp's steps [c0, c1) for one row of codes (lane-strided,
// butterfly).
__device__ __forceinline__ float warp_row_f32(const float* x, const int8_t* codes, int c0, int c1, int lane) {
    float a = 0.0f;
    for (int c = c0; c < c1; ++c) a = fmaf(__ldg(x + 32 * c + lane), static_cast<float>(codes[32 * c + lane]), a);
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    return a;
}

}  // namespace pcb
