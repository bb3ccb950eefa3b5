/*
 * A C consumer of popcorn's quantized-linear ABI -- TEST PROGRAM.
 *
 * It is built the way a cgo program links popcorn (popcorn README.md:85-107):
 * plain C compiled by gcc, include/popcorn.h, lib/libpopcorn.a, the CUDA
 * runtime and libstdc++, nothing else. It plays the part of a linear layer in
 * popcorn's consumer (tendo, whose source is not available here): weights are
 * quantized once at load time with the library's quantizers, then each
 * forward call runs a dequant-matmul on the caller's stream.
 *
 * Several host threads run layers at the same time, each on its own
 * non-blocking stream, one on the legacy default stream (NULL, as popcorn's
 * own tests pass). Every result is checked against a double-precision host
 * computation from the codes and scales the library produced; per-channel
 * codes are also checked against a host quantizer with popcorn's arithmetic.
 * The argument conventions (null pointer -> invalid value before sizes, size
 * <= 0 -> success) and the per-thread CUDA error state are checked too.
 *
 * Exit status 0 when every check passed; each failure prints one line.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "popcorn.h"

#define GROUP 128
#define TOL 2e-3 /* normwise, the tensor path's bar; the f32 path is far below */

static int g_failures = 0;
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;

static void fail(const char* what, int thread, double value) {
    pthread_mutex_lock(&g_mu);
    fprintf(stderr, "FAIL [thread %d] %s (%g)\n", thread, what, value);
    g_failures++;
    pthread_mutex_unlock(&g_mu);
}

/* SplitMix64 stream -> uniform floats in [-1, 1). */
static uint64_t mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static void fill(float* a, int64_t n, uint64_t seed, float amp) {
    for (int64_t i = 0; i < n; i++) {
        const double u = (double)(mix(seed * 0x100000001B3ull + (uint64_t)i) >> 11) / 9007199254740992.0;
        a[i] = (float)((2.0 * u - 1.0) * amp);
    }
}

/* Host quantizer with popcorn's per-channel arithmetic (src/quantize.cu:458-528):
 * NaN-skipping row max, scale = max / 127 (1 when 0), rint(v / scale), clamp. */
static void host_quantize(int8_t* q, float* s, const float* w, int64_t N, int64_t K) {
    for (int64_t n = 0; n < N; n++) {
        float mx = 0.0f;
        for (int64_t k = 0; k < K; k++) {
            const float a = fabsf(w[n * K + k]);
            if (a > mx) mx = a;
        }
        float sc = mx / 127.0f;
        if (sc == 0.0f) sc = 1.0f;
        s[n] = sc;
        for (int64_t k = 0; k < K; k++) {
            float v = rintf(w[n * K + k] / sc);
            if (v > 127.0f) v = 127.0f;
            if (v < -128.0f) v = -128.0f;
            q[n * K + k] = (int8_t)v;
        }
    }
}

/* max |got - ref| / max |ref| over an [M, N] output. */
static double normwise(const float* got, const double* ref, int64_t n) {
    double num = 0.0, den = 0.0;
    for (int64_t i = 0; i < n; i++) {
        const double d = fabs((double)got[i] - ref[i]);
        if (d > num || d != d) num = d != d ? INFINITY : d;
        if (fabs(ref[i]) > den) den = fabs(ref[i]);
    }
    return den > 0.0 ? num / den : num;
}

/* Weight of (n, k) in each format, from the library's own codes. */
enum { FMT_CHANNEL, FMT_GROUP8, FMT_INT4 };

static double weight(int fmt, int64_t n, int64_t k, int64_t K, const int8_t* q8, const float* s, const uint8_t* q4,
                     const float* z) {
    const int64_t groups = K / GROUP;
    if (fmt == FMT_CHANNEL) return (double)q8[n * K + k] * s[n];
    if (fmt == FMT_GROUP8) return (double)q8[n * K + k] * s[n * groups + k / GROUP];
    const uint8_t b = q4[n * (K / 2) + k / 2];
    const int c = (k % 2 == 0) ? (b & 0x0F) : (b >> 4);
    return ((double)c - z[n * groups + k / GROUP]) * s[n * groups + k / GROUP];
}

static void host_matmul(double* y, const float* x, int64_t M, int64_t N, int64_t K, int fmt, const int8_t* q8,
                        const float* s, const uint8_t* q4, const float* z) {
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)x[m * K + k] * weight(fmt, n, k, K, q8, s, q4, z);
            y[m * N + n] = acc;
        }
    }
}

typedef struct {
    int id;
    int64_t M, N, K;
} Job;

#define CK(call)                                                     \
    do {                                                             \
        cudaError_t e_ = (call);                                     \
        if (e_ != cudaSuccess) {                                     \
            fail(#call, job->id, (double)e_);                        \
            goto done;                                               \
        }                                                            \
    } while (0)

#define PK(call)                                                               \
    do {                                                                       \
        popcornStatus_t st_ = (call);                                          \
        if (st_ != POPCORN_SUCCESS) {                                          \
            fail(#call, job->id, (double)st_);                                 \
            fprintf(stderr, "  %s: %s\n", popcornGetErrorString(st_),          \
                    popcornGetLastCudaErrorString());                          \
            goto done;                                                         \
        }                                                                      \
    } while (0)

/* One linear layer in each weight format: quantize at load time, then
 * forward passes on this thread's stream. */
static void* run_layer(void* arg) {
    const Job* job = (const Job*)arg;
    const int64_t M = job->M, N = job->N, K = job->K, G = K / GROUP;
    cudaStream_t stream = NULL;
    float *w = NULL, *x = NULL, *y = NULL, *s = NULL, *hs = NULL, *sg = NULL, *s4 = NULL, *z4 = NULL;
    int8_t *q = NULL, *hq = NULL, *qg = NULL;
    uint8_t* q4 = NULL;
    double* ref = NULL;
    float *d_w = NULL, *d_x = NULL, *d_y = NULL, *d_s = NULL, *d_sg = NULL, *d_s4 = NULL, *d_z4 = NULL;
    int8_t *d_q = NULL, *d_qg = NULL;
    uint8_t* d_q4 = NULL;

    if (job->id != 0) CK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    if (popcornGetLastCudaError() != cudaSuccess) fail("fresh thread has a CUDA error recorded", job->id, 0);

    w = malloc(sizeof(float) * N * K);
    x = malloc(sizeof(float) * M * K);
    y = malloc(sizeof(float) * M * N);
    s = malloc(sizeof(float) * N);
    hs = malloc(sizeof(float) * N);
    sg = malloc(sizeof(float) * N * G);
    s4 = malloc(sizeof(float) * N * G);
    z4 = malloc(sizeof(float) * N * G);
    q = malloc((size_t)(N * K));
    hq = malloc((size_t)(N * K));
    qg = malloc((size_t)(N * K));
    q4 = malloc((size_t)(N * K / 2));
    ref = malloc(sizeof(double) * M * N);
    if (!w || !x || !y || !s || !hs || !sg || !s4 || !z4 || !q || !hq || !qg || !q4 || !ref) {
        fail("host allocation", job->id, 0);
        goto done;
    }
    fill(w, N * K, 1000 + (uint64_t)job->id, 0.05f);
    fill(x, M * K, 2000 + (uint64_t)job->id, 1.0f);

    CK(cudaMalloc((void**)&d_w, sizeof(float) * N * K));
    CK(cudaMalloc((void**)&d_x, sizeof(float) * M * K));
    CK(cudaMalloc((void**)&d_y, sizeof(float) * M * N));
    CK(cudaMalloc((void**)&d_s, sizeof(float) * N));
    CK(cudaMalloc((void**)&d_sg, sizeof(float) * N * G));
    CK(cudaMalloc((void**)&d_s4, sizeof(float) * N * G));
    CK(cudaMalloc((void**)&d_z4, sizeof(float) * N * G));
    CK(cudaMalloc((void**)&d_q, (size_t)(N * K)));
    CK(cudaMalloc((void**)&d_qg, (size_t)(N * K)));
    CK(cudaMalloc((void**)&d_q4, (size_t)(N * K / 2)));
    CK(cudaMemcpyAsync(d_w, w, sizeof(float) * N * K, cudaMemcpyHostToDevice, stream));
    CK(cudaMemcpyAsync(d_x, x, sizeof(float) * M * K, cudaMemcpyHostToDevice, stream));

    /* Load time: quantize the layer's weights in all three formats. */
    PK(popcornQuantize_f32i8(d_q, d_s, d_w, N, K, stream));
    PK(popcornQuantizeGrouped_f32i8(d_qg, d_sg, d_w, N, K, GROUP, stream));
    PK(popcornQuantizeGrouped_f32i4(d_q4, d_s4, d_z4, d_w, N, K, GROUP, stream));
    CK(cudaMemcpyAsync(q, d_q, (size_t)(N * K), cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(s, d_s, sizeof(float) * N, cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(qg, d_qg, (size_t)(N * K), cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(sg, d_sg, sizeof(float) * N * G, cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(q4, d_q4, (size_t)(N * K / 2), cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(s4, d_s4, sizeof(float) * N * G, cudaMemcpyDeviceToHost, stream));
    CK(cudaMemcpyAsync(z4, d_z4, sizeof(float) * N * G, cudaMemcpyDeviceToHost, stream));
    CK(cudaStreamSynchronize(stream));

    host_quantize(hq, hs, w, N, K);
    if (memcmp(hq, q, (size_t)(N * K)) != 0) fail("per-channel codes differ from the host quantizer", job->id, 0);
    if (memcmp(hs, s, sizeof(float) * N) != 0) fail("per-channel scales differ from the host quantizer", job->id, 0);

    /* Forward passes: per-channel, batched (the same rows as two batches),
     * per-group int8 and int4. */
    for (int fmt = 0; fmt < 4; fmt++) {
        CK(cudaMemsetAsync(d_y, 0xFF, sizeof(float) * M * N, stream)); /* NaN: nothing stale can pass */
        if (fmt == 0) {
            PK(popcornDequantizeMatmul_i8f32(d_y, d_x, d_q, d_s, M, N, K, stream));
        } else if (fmt == 1) {
            if (M % 2 != 0) continue;
            PK(popcornDequantizeMatmulBatched_i8f32(d_y, d_x, d_q, d_s, 2, M / 2, N, K, stream));
        } else if (fmt == 2) {
            PK(popcornDequantizeMatmulGrouped_i8f32(d_y, d_x, d_qg, d_sg, M, N, K, GROUP, stream));
        } else {
            PK(popcornDequantizeMatmulGrouped_i4f32(d_y, d_x, d_q4, d_s4, d_z4, M, N, K, GROUP, stream));
        }
        CK(cudaMemcpyAsync(y, d_y, sizeof(float) * M * N, cudaMemcpyDeviceToHost, stream));
        CK(cudaStreamSynchronize(stream));
        const int wf = fmt <= 1 ? FMT_CHANNEL : (fmt == 2 ? FMT_GROUP8 : FMT_INT4);
        host_matmul(ref, x, M, N, K, wf, wf == FMT_GROUP8 ? qg : q, wf == FMT_CHANNEL ? s : (wf == FMT_GROUP8 ? sg : s4),
                    q4, z4);
        const double err = normwise(y, ref, M * N);
        if (!(err <= TOL)) {
            static const char* names[4] = {"per-channel", "batched", "per-group int8", "int4"};
            char what[96];
            snprintf(what, sizeof what, "%s matmul M=%lld N=%lld K=%lld normwise error", names[fmt], (long long)M,
                     (long long)N, (long long)K);
            fail(what, job->id, err);
        }
    }
    if (popcornGetLastCudaError() != cudaSuccess) fail("CUDA error recorded after successful calls", job->id, 0);

done:
    cudaFree(d_w);
    cudaFree(d_x);
    cudaFree(d_y);
    cudaFree(d_s);
    cudaFree(d_sg);
    cudaFree(d_s4);
    cudaFree(d_z4);
    cudaFree(d_q);
    cudaFree(d_qg);
    cudaFree(d_q4);
    if (stream != NULL) cudaStreamDestroy(stream);
    free(w);
    free(x);
    free(y);
    free(s);
    free(hs);
    free(sg);
    free(s4);
    free(z4);
    free(q);
    free(hq);
    free(qg);
    free(q4);
    free(ref);
    return NULL;
}

/* Argument conventions (popcorn src/quantize.cu:96-102, :190-202, :418-433):
 * these calls return before touching memory or the GPU. */
static void check_conventions(void) {
    float* fake = (float*)(uintptr_t)0x1000;
    if (popcornDequantizeMatmul_i8f32(NULL, fake, (const int8_t*)fake, fake, 1, 1, 1, NULL) !=
        POPCORN_ERROR_INVALID_VALUE)
        fail("null out is not invalid", -1, 0);
    if (popcornDequantizeMatmul_i8f32(fake, fake, (const int8_t*)fake, fake, 0, 4, 4, NULL) != POPCORN_SUCCESS)
        fail("M = 0 is not a no-op", -1, 0);
    if (popcornDequantizeMatmulGrouped_i4f32(fake, fake, (const uint8_t*)fake, fake, fake, 2, 2, 9, 3, NULL) !=
        POPCORN_ERROR_INVALID_VALUE)
        fail("odd K for int4 is not invalid", -1, 0);
    if (popcornQuantizeGrouped_f32i8((int8_t*)fake, fake, fake, 2, 10, 4, NULL) != POPCORN_ERROR_INVALID_VALUE)
        fail("group size not dividing K is not invalid", -1, 0);
    if (strcmp(popcornGetErrorString(POPCORN_ERROR_INVALID_VALUE), "invalid value") != 0)
        fail("error string", -1, 0);
    if (popcornGetLastCudaError() != cudaSuccess) fail("argument errors recorded a CUDA error", -1, 0);
}

int main(void) {
    int dev = 0;
    if (cudaGetDeviceCount(&dev) != cudaSuccess || dev < 1) {
        fprintf(stderr, "no CUDA device\n");
        return 2;
    }
    check_conventions();
    /* Decode (f32 path), a small batch, and a prefill-sized layer (tensor
     * path), on five threads at once; thread 0 uses the legacy default stream. */
    Job jobs[5] = {
        {0, 1, 1024, 4096}, {1, 4, 2048, 1024}, {2, 64, 1024, 4096}, {3, 1, 4096, 4096}, {4, 32, 768, 2048},
    };
    pthread_t tid[5];
    for (int i = 0; i < 5; i++) pthread_create(&tid[i], NULL, run_layer, &jobs[i]);
    for (int i = 0; i < 5; i++) pthread_join(tid[i], NULL);
    if (cudaDeviceSynchronize() != cudaSuccess) fail("device synchronize", -1, 0);
    if (g_failures == 0) {
        printf("consumer ok: 5 threads, per-channel / batched / per-group int8 / int4 layers\n");
        return 0;
    }
    fprintf(stderr, "%d check(s) failed\n", g_failures);
    return 1;
}
