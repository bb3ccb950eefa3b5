/*
 * CPU oracle of popcorn's int8 dequant-matmul path -- TEST INFRASTRUCTURE,
 * never part of the product path. See oracle.h for what each function
 * restates and how the restatement is pinned to the reference.
 *
 * Build flags matter for bit-exactness: -ffp-contract=off keeps the
 * unfused variant's multiply and add separately rounded.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>
#include <pthread.h>
#include <stdlib.h>

void oracle_dequant_matmul_i8(float* out, const float* x, const int8_t* q, const float* scale,
                              int64_t M, int64_t N, int64_t K, int fused) {
    /* popcorn test/test_quantize.cu:31-39 and src/quantize.cu:47-83: for each
     * output, walk k upward, widen the code, multiply by the channel scale,
     * then multiply-add with the activation. */
    for (int64_t m = 0; m < M; m++) {
        const float* xr = x + m * K;
        for (int64_t n = 0; n < N; n++) {
            const int8_t* qr = q + n * K;
            const float sc = scale[n];
            float acc = 0.0f;
            if (fused) {
                for (int64_t k = 0; k < K; k++) {
                    const float w = (float)qr[k] * sc;
                    acc = fmaf(xr[k], w, acc);
                }
            } else {
                for (int64_t k = 0; k < K; k++) {
                    const float w = (float)qr[k] * sc;
                    const float p = xr[k] * w;
                    acc = acc + p;
                }
            }
            out[m * N + n] = acc;
        }
    }
}

typedef struct {
    float* out;
    const float* x;
    const int8_t* q;
    const float* scale;
    int64_t M, N, K, n0, n1;
    int fused;
} mm_job;

static void* mm_worker(void* arg) {
    const mm_job* j = (const mm_job*)arg;
    for (int64_t m = 0; m < j->M; m++) {
        /* One activation row against this thread's channel range; the output
         * row pointer is offset so the layout stays [M, N]. */
        for (int64_t n = j->n0; n < j->n1; n++) {
            const int8_t* qr = j->q + n * j->K;
            const float* xr = j->x + m * j->K;
            const float sc = j->scale[n];
            float acc = 0.0f;
            if (j->fused) {
                for (int64_t k = 0; k < j->K; k++) acc = fmaf(xr[k], (float)qr[k] * sc, acc);
            } else {
                for (int64_t k = 0; k < j->K; k++) {
                    const float w = (float)qr[k] * sc;
                    const float p = xr[k] * w;
                    acc = acc + p;
                }
            }
            j->out[m * j->N + n] = acc;
        }
    }
    return NULL;
}

void oracle_dequant_matmul_i8_mt(float* out, const float* x, const int8_t* q, const float* scale,
                                 int64_t M, int64_t N, int64_t K, int fused, int threads) {
    if (threads < 1) threads = 1;
    if (threads > N) threads = (int)N;
    if (threads <= 1) {
        oracle_dequant_matmul_i8(out, x, q, scale, M, N, K, fused);
        return;
    }
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    mm_job* jobs = (mm_job*)malloc(sizeof(mm_job) * (size_t)threads);
    for (int t = 0; t < threads; t++) {
        jobs[t].out = out;
        jobs[t].x = x;
        jobs[t].q = q;
        jobs[t].scale = scale;
        jobs[t].M = M;
        jobs[t].N = N;
        jobs[t].K = K;
        jobs[t].n0 = N * t / threads;
        jobs[t].n1 = N * (t + 1) / threads;
        jobs[t].fused = fused;
        pthread_create(&tid[t], NULL, mm_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    free(jobs);
    free(tid);
}

void oracle_quantize_i8(int8_t* out, float* scale, const float* in, int64_t N, int64_t K, int ties) {
    for (int64_t n = 0; n < N; n++) {
        const float* r = in + n * K;
        /* Row max of |v|: NaN fails the compare and is skipped
         * (src/quantize.cu:470-477, test/test_quantize.cu:686-691). */
        float max_abs = 0.0f;
        for (int64_t k = 0; k < K; k++) {
            const float v = r[k];
            const float a = v < 0 ? -v : v;
            if (a > max_abs) max_abs = a;
        }
        float sc = max_abs / 127.0f;
        if (sc == 0.0f) sc = 1.0f;
        scale[n] = sc;
        for (int64_t k = 0; k < K; k++) {
            const float d = r[k] / sc;
            float qv = ties ? roundf(d) : rintf(d);
            if (qv > 127.0f) qv = 127.0f;
            if (qv < -128.0f) qv = -128.0f;
            /* A NaN code converts to 0 on the GPU (PTX float->int conversion
             * maps NaN to 0); state it explicitly rather than rely on the
             * host compiler's undefined cast. */
            out[n * K + k] = (qv != qv) ? (int8_t)0 : (int8_t)qv;
        }
    }
}

typedef struct {
    float* out;
    const float* x;
    const int8_t* q;
    const float* scale;
    int64_t M, N, K, gs, n0, n1;
    int fused;
} gmm_job;

static void* gmm_worker(void* arg) {
    /* popcorn test/test_quantize.cu:51-58 and src/quantize.cu:168-177: for
     * each output, walk k upward; the code times its group's scale, then the
     * multiply-add with the activation. */
    const gmm_job* j = (const gmm_job*)arg;
    const int64_t groups = j->K / j->gs;
    for (int64_t m = 0; m < j->M; m++) {
        const float* xr = j->x + m * j->K;
        for (int64_t n = j->n0; n < j->n1; n++) {
            const int8_t* qr = j->q + n * j->K;
            const float* sr = j->scale + n * groups;
            float acc = 0.0f;
            for (int64_t k = 0; k < j->K; k++) {
                const float w = (float)qr[k] * sr[k / j->gs];
                if (j->fused) {
                    acc = fmaf(xr[k], w, acc);
                } else {
                    const float p = xr[k] * w;
                    acc = acc + p;
                }
            }
            j->out[m * j->N + n] = acc;
        }
    }
    return NULL;
}

void oracle_dequant_matmul_grouped_i8(float* out, const float* x, const int8_t* q, const float* scale, int64_t M,
                                      int64_t N, int64_t K, int64_t gs, int fused, int threads) {
    if (threads < 1) threads = 1;
    if (threads > N) threads = (int)N;
    if (threads < 1) return;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    gmm_job* jobs = (gmm_job*)malloc(sizeof(gmm_job) * (size_t)threads);
    for (int t = 0; t < threads; t++) {
        gmm_job j = {out, x, q, scale, M, N, K, gs, N * t / threads, N * (t + 1) / threads, fused};
        jobs[t] = j;
        if (threads > 1) pthread_create(&tid[t], NULL, gmm_worker, &jobs[t]);
    }
    if (threads > 1) {
        for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    } else {
        gmm_worker(&jobs[0]);
    }
    free(jobs);
    free(tid);
}

void oracle_quantize_grouped_i8(int8_t* out, float* scale, const float* in, int64_t N, int64_t K, int64_t gs,
                                int ties) {
    const int64_t groups = K / gs;
    for (int64_t n = 0; n < N; n++) {
        for (int64_t g = 0; g < groups; g++) {
            const float* r = in + n * K + g * gs;
            /* Group max of |v|, NaN skipped by the compare (src/quantize.cu:585-592). */
            float max_abs = 0.0f;
            for (int64_t i = 0; i < gs; i++) {
                const float v = r[i];
                const float a = v < 0 ? -v : v;
                if (a > max_abs) max_abs = a;
            }
            float sc = max_abs / 127.0f;
            if (sc == 0.0f) sc = 1.0f;
            scale[n * groups + g] = sc;
            for (int64_t i = 0; i < gs; i++) {
                const float d = r[i] / sc;
                float qv = ties ? roundf(d) : rintf(d);
                if (qv > 127.0f) qv = 127.0f;
                if (qv < -128.0f) qv = -128.0f;
                out[n * K + g * gs + i] = (qv != qv) ? (int8_t)0 : (int8_t)qv;  /* NaN -> 0 as on the GPU */
            }
        }
    }
}

typedef struct {
    float* out;
    const float* x;
    const uint8_t* q;
    const float* scale;
    const float* zero;
    int64_t M, N, K, gs, n0, n1;
    int fused;
} i4mm_job;

static void* i4mm_worker(void* arg) {
    /* popcorn test/test_quantize.cu:80-96 and src/quantize.cu:374-395: for
     * each output, walk k upward; take the nibble of byte k/2 (low for even
     * k), subtract the group's zero point, multiply by its scale, then the
     * multiply-add with the activation. */
    const i4mm_job* j = (const i4mm_job*)arg;
    const int64_t groups = j->K / j->gs;
    const int64_t row_bytes = j->K / 2;
    for (int64_t m = 0; m < j->M; m++) {
        const float* xr = j->x + m * j->K;
        for (int64_t n = j->n0; n < j->n1; n++) {
            const uint8_t* qr = j->q + n * row_bytes;
            const float* sr = j->scale + n * groups;
            const float* zr = j->zero + n * groups;
            float acc = 0.0f;
            for (int64_t k = 0; k < j->K; k++) {
                const uint8_t b = qr[k / 2];
                const int nib = (k % 2 == 0) ? (b & 0x0F) : (b >> 4);
                const int64_t g = k / j->gs;
                const float d = (float)nib - zr[g];
                const float w = d * sr[g];
                if (j->fused) {
                    acc = fmaf(xr[k], w, acc);
                } else {
                    const float p = xr[k] * w;
                    acc = acc + p;
                }
            }
            j->out[m * j->N + n] = acc;
        }
    }
    return NULL;
}

void oracle_dequant_matmul_grouped_i4(float* out, const float* x, const uint8_t* q, const float* scale,
                                      const float* zero, int64_t M, int64_t N, int64_t K, int64_t gs, int fused,
                                      int threads) {
    if (threads < 1) threads = 1;
    if (threads > N) threads = (int)N;
    if (threads < 1) return;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    i4mm_job* jobs = (i4mm_job*)malloc(sizeof(i4mm_job) * (size_t)threads);
    for (int t = 0; t < threads; t++) {
        i4mm_job j = {out, x, q, scale, zero, M, N, K, gs, N * t / threads, N * (t + 1) / threads, fused};
        jobs[t] = j;
        if (threads > 1) pthread_create(&tid[t], NULL, i4mm_worker, &jobs[t]);
    }
    if (threads > 1) {
        for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    } else {
        i4mm_worker(&jobs[0]);
    }
    free(jobs);
    free(tid);
}

/* Group min and max as popcorn's min/max kernel forms them
 * (src/quantize.cu:705-750): a block of 256 threads, thread t scanning
 * elements t, t + 256, ... from +inf / -inf with strict compares (NaN never
 * wins), then a halving tree in which the lower-numbered partner is kept on
 * a tie. Values that compare equal have the same bits except +0 and -0, so
 * the order only decides the sign of a zero min or max. */
static void i4_group_minmax_kernel_order(const float* r, int64_t gs, float* mn_out, float* mx_out) {
    float mn[256], mx[256];
    for (int t = 0; t < 256; t++) {
        float a = INFINITY, b = -INFINITY;
        for (int64_t i = t; i < gs; i += 256) {
            const float v = r[i];
            if (v < a) a = v;
            if (v > b) b = v;
        }
        mn[t] = a;
        mx[t] = b;
    }
    for (int s = 128; s > 0; s >>= 1) {
        for (int t = 0; t < s; t++) {
            if (mn[t + s] < mn[t]) mn[t] = mn[t + s];
            if (mx[t + s] > mx[t]) mx[t] = mx[t + s];
        }
    }
    *mn_out = mn[0];
    *mx_out = mx[0];
}

static uint8_t i4_code(float v, float sc, float zp, int ties) {
    const float d = v / sc + zp;
    float qv = ties ? roundf(d) : rintf(d);
    if (qv < 0.0f) qv = 0.0f;
    if (qv > 15.0f) qv = 15.0f;
    return (qv != qv) ? (uint8_t)0 : (uint8_t)qv;  /* NaN -> 0 as the GPU converts it */
}

void oracle_quantize_grouped_i4(uint8_t* out, float* scale, float* zero, const float* in, int64_t N, int64_t K,
                                int64_t gs, int variant) {
    const int64_t groups = K / gs;
    for (int64_t n = 0; n < N; n++) {
        for (int64_t g = 0; g < groups; g++) {
            const float* r = in + n * K + g * gs;
            float mn, mx;
            if (variant == 0) {
                i4_group_minmax_kernel_order(r, gs, &mn, &mx);
            } else {
                /* test/test_quantize.cu:761-767: start at the first value. */
                mn = r[0];
                mx = r[0];
                for (int64_t i = 1; i < gs; i++) {
                    if (r[i] < mn) mn = r[i];
                    if (r[i] > mx) mx = r[i];
                }
            }
            const float range = mx - mn;
            float sc = range / 15.0f;
            if (sc == 0.0f) sc = 1.0f;
            scale[n * groups + g] = sc;
            zero[n * groups + g] = -mn / sc;
        }
        /* Codes: element k uses the parameters of its own group (a byte of an
         * odd group size straddles two groups; popcorn's apply kernel,
         * src/quantize.cu:772-823, computes each nibble with its own group). */
        for (int64_t k = 0; k < K; k += 2) {
            const int64_t glo = n * groups + k / gs, ghi = n * groups + (k + 1) / gs;
            const uint8_t lo = i4_code(in[n * K + k], scale[glo], zero[glo], variant);
            const uint8_t hi = i4_code(in[n * K + k + 1], scale[ghi], zero[ghi], variant);
            out[n * (K / 2) + k / 2] = (uint8_t)((hi << 4) | lo);
        }
    }
}

void oracle_rmsnorm(float* out, const float* in, const float* weight, int64_t rows, int64_t K, float eps, int fused) {
    for (int64_t r = 0; r < rows; r++) {
        const float* x = in + r * K;
        float* o = out + r * K;
        /* src/reduction.cu:303-313 */
        float sum_sq = 0.0f;
        for (int64_t k = 0; k < K; k++) {
            if (fused) {
                sum_sq = fmaf(x[k], x[k], sum_sq);
            } else {
                const float p = x[k] * x[k];
                sum_sq = sum_sq + p;
            }
        }
        const float rms = sqrtf(sum_sq / (float)K + eps);
        const float inv = 1.0f / rms;
        for (int64_t k = 0; k < K; k++) {
            float v = x[k] * inv;
            if (weight != NULL) v = v * weight[k];
            o[k] = v;
        }
    }
}

void oracle_silu(float* out, const float* in, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = in[i] / (1.0f + expf(-in[i]));
}

void oracle_dequantize_i8(float* out, const int8_t* q, const float* scale, int64_t N, int64_t K) {
    for (int64_t n = 0; n < N; n++) {
        const float sc = scale[n];
        for (int64_t k = 0; k < K; k++) out[n * K + k] = (float)q[n * K + k] * sc;
    }
}

/* f32 -> bf16 bit pattern, round to nearest, ties to even (IEEE-754 binary32
 * truncated to its upper 16 bits after adding half an ulp of the result plus
 * the tie bit); NaN keeps its sign and becomes a quiet NaN. */
static uint16_t f32_to_bf16_rne(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x0040u);
    b += 0x7FFFu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

void oracle_dequantize_i8_bf16(uint16_t* out, const int8_t* q, const float* scale, int64_t N, int64_t K) {
    for (int64_t n = 0; n < N; n++) {
        const float sc = scale[n];
        for (int64_t k = 0; k < K; k++) out[n * K + k] = f32_to_bf16_rne((float)q[n * K + k] * sc);
    }
}

static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void oracle_fill_normal(float* out, int64_t n, uint64_t seed, float sigma) {
    const double s = (double)sigma;
    for (int64_t i = 0; i < n; i++) {
        double acc = 0.0;
        for (int j = 0; j < 12; j++) {
            const uint64_t z = splitmix64(seed + (uint64_t)(12 * i + j) * 0x9E3779B97F4A7C15ull);
            /* 24-bit uniform, centred in its cell: ((z >> 40) + 0.5) / 2^24. */
            acc += ((double)(z >> 40) + 0.5) * (1.0 / 16777216.0);
        }
        out[i] = (float)((acc - 6.0) * s);
    }
}
