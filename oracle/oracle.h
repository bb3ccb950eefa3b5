/*
 * CPU oracle of popcorn's int8 dequant-matmul path -- TEST INFRASTRUCTURE.
 *
 * Only the tests, the smoke check and the benchmark's CPU-baseline leg use
 * this library, and only as the checker / baseline; the product path never
 * links or calls it. Parity is pinned: the restatement is checked against
 * the reference's own CPU loops (built from popcorn's sources into
 * oracle/_ref by oracle/Makefile) and against golden vectors made by those
 * loops (tests/golden), and on the GPU against popcorn's own CUDA kernels
 * rebuilt for sm_100a.
 */
#ifndef POPCORN_ORACLE_H
#define POPCORN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[m,n] = sum_k x[m,k] * ((float)q[n,k] * scale[n]), k ascending, f32.
 * fused = 0: product and sum rounded separately, as popcorn's test loop
 *            (test/test_quantize.cu:24-41) compiles on x86-64;
 * fused = 1: acc = fmaf(x, w, acc), as popcorn's GPU kernel executes
 *            (src/quantize.cu:69-73, nvcc contracts the multiply-add). */
void oracle_dequant_matmul_i8(float* out, const float* x, const int8_t* q, const float* scale,
                              int64_t M, int64_t N, int64_t K, int fused);

/* Same arithmetic split over `threads` POSIX threads by output channel. */
void oracle_dequant_matmul_i8_mt(float* out, const float* x, const int8_t* q, const float* scale,
                                 int64_t M, int64_t N, int64_t K, int fused, int threads);

/* Per-row symmetric int8 quantization (src/quantize.cu:458-528).
 * ties = 0: rintf (half to even), popcorn's GPU kernel (:524);
 * ties = 1: roundf (half away from zero), popcorn's test loop
 *           (test/test_quantize.cu:700). */
void oracle_quantize_i8(int8_t* out, float* scale, const float* in, int64_t N, int64_t K, int ties);

/* Per-group variant (src/quantize.cu:114-218, test/test_quantize.cu:42-61):
 * out[m,n] = sum_k x[m,k] * ((float)q[n,k] * scale[n, k / gs]), k ascending,
 * scale [N, K/gs]; `fused` as above; split over `threads` by channel. */
void oracle_dequant_matmul_grouped_i8(float* out, const float* x, const int8_t* q, const float* scale, int64_t M,
                                      int64_t N, int64_t K, int64_t gs, int fused, int threads);

/* Per-group symmetric int8 quantization (src/quantize.cu:571-640,
 * test/test_quantize.cu:709-742): every group of gs consecutive values of a
 * row gets its own scale = max|v| / 127 (1 if 0), NaN skipped; `ties` as in
 * oracle_quantize_i8. scale is [N, K/gs]. */
void oracle_quantize_grouped_i8(int8_t* out, float* scale, const float* in, int64_t N, int64_t K, int64_t gs,
                                int ties);

/* Int4 packed asymmetric per-group dequant-matmul (src/quantize.cu:335-405,
 * test/test_quantize.cu:67-99): q is [N, K/2] bytes; element k of row n is
 * the low nibble of byte k/2 for even k, the high nibble for odd k; its
 * weight is ((float)nibble - zero[n, k/gs]) * scale[n, k/gs] (subtract, then
 * multiply, each rounded); k ascending; `fused` as above; split over
 * `threads` by channel. scale and zero are [N, K/gs]. */
void oracle_dequant_matmul_grouped_i4(float* out, const float* x, const uint8_t* q, const float* scale,
                                      const float* zero, int64_t M, int64_t N, int64_t K, int64_t gs, int fused,
                                      int threads);

/* Int4 asymmetric per-group quantization: per group min and max, then
 * scale = (max - min) / 15 (1 if 0), zero = -min / scale, and codes
 * clamp(round(v / scale + zero), 0, 15) packed two per byte, low nibble first.
 * variant 0: popcorn's GPU kernels (src/quantize.cu:705-827): min/max start
 *            at +inf/-inf and skip NaN, reduced the way its 256-thread block
 *            does (which fixes the sign of a zero min or max), codes by rintf
 *            (half to even), a NaN code packs as 0; any even K and any gs;
 * variant 1: popcorn's test loop (test/test_quantize.cu:747-789): min/max
 *            start at the group's first value, scanned in order, codes by
 *            roundf (half away from zero); even gs only. */
void oracle_quantize_grouped_i4(uint8_t* out, float* scale, float* zero, const float* in, int64_t N, int64_t K,
                                int64_t gs, int variant);

/* popcorn's RMSNorm (src/reduction.cu:290-321, one thread per row): the row's
 * sum of squares in k order (fused = 1: fmaf, as nvcc contracts
 * `sum_sq += x * x` in that kernel; fused = 0: product and sum rounded
 * separately), rms = sqrtf(sum / K + eps), inv = 1 / rms, then
 * out = (x * inv) * weight[k] (weight may be NULL: no scaling). */
void oracle_rmsnorm(float* out, const float* in, const float* weight, int64_t rows, int64_t K, float eps, int fused);

/* popcorn's SiLU (src/unary.cu:76-81): x / (1 + expf(-x)), with the host's expf. */
void oracle_silu(float* out, const float* in, int64_t n);

/* out[n,k] = (float)q[n,k] * scale[n]. */
void oracle_dequantize_i8(float* out, const int8_t* q, const float* scale, int64_t N, int64_t K);

/* The same f32 product rounded once to bf16 (nearest, ties to even); out
 * holds the bf16 bit patterns. */
void oracle_dequantize_i8_bf16(uint16_t* out, const int8_t* q, const float* scale, int64_t N, int64_t K);

/* Deterministic synthetic data: SplitMix64 stream (Steele, Lea & Flood 2014)
 * feeding an Irwin-Hall(12) normal approximation, sum of twelve 24-bit
 * uniforms minus 6, scaled by sigma. Integer and exactly-rounded float
 * arithmetic only, so every IEEE-754 machine produces the same bits.
 * Element i of a stream seeded `seed` depends only on (seed, i). */
void oracle_fill_normal(float* out, int64_t n, uint64_t seed, float sigma);

#ifdef __cplusplus
}
#endif

#endif /* POPCORN_ORACLE_H */
