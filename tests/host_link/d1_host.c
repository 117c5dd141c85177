/*
 * A non-Python host of libd1kernels, written the way the reference's Rust host drives its kernels: it links the
 * static archive (the drop-in for the library build.rs:11-40 archives) with the CUDA runtime only, binds the C ABI
 * of include/d1kernels.h (the declarations src/cuda.rs:102-175 makes) and runs one attention layer's chain on a
 * packed batch of two sequences, in the order src/model.rs:355-399 calls it:
 *
 *   d1_lt_init (src/cuda.rs:406) -> d1_rmsnorm -> d1_lt_tune + d1_lt_gemm (the QKV projection, fp16 out)
 *   -> d1_flash_attn with the reference's work list (one item per 64-row tile, src/model.rs:328-339)
 *
 * Each result is checked on the host in double precision against the device's own inputs to that step:
 * RMSNorm to one fp16 rounding, the GEMM to 2e-3 relative, the attention to 4e-3 absolute. Prints "ok" and
 * exits 0 when every check passes; exits 1 on a failed check or an error return.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "d1kernels.h"

enum { D = 1024, HEADS = 2, KVH = 1, HD = 64, NQKV = (HEADS + 2 * KVH) * HD, NSEQ = 2 };
static const int LENS[NSEQ] = {200, 100};

static uint32_t rng_state = 12345u;
static float uniform(void) { /* xorshift32 in [-1, 1) */
    rng_state ^= rng_state << 13;
    rng_state ^= rng_state >> 17;
    rng_state ^= rng_state << 5;
    return (float)(rng_state >> 8) / 8388608.0f - 1.0f;
}

static float h2f(uint16_t h) { /* IEEE binary16 -> float */
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else { /* subnormal */
            float f = ldexpf((float)m, -24);
            return s ? -f : f;
        }
    } else if (e == 31) {
        bits = s | 0x7F800000u | (m << 13);
    } else {
        bits = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t f2h(float f) { /* float -> binary16, round to nearest even (normal range only) */
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t s = (x >> 16) & 0x8000u;
    int e = (int)((x >> 23) & 255) - 127 + 15;
    uint32_t m = x & 0x7FFFFFu;
    if (e <= 0) return (uint16_t)s; /* flush tiny values (none occur here) */
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    uint32_t r = (uint32_t)(e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) r++;
    return (uint16_t)(s | r);
}

#define CHECK_CUDA(call)                                                                          \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) {                                                                  \
            fprintf(stderr, "%s failed: %s\n", #call, cudaGetErrorString(e_));                    \
            return 1;                                                                             \
        }                                                                                         \
    } while (0)
#define CHECK_D1(call)                                                                            \
    do {                                                                                          \
        int r_ = (call);                                                                          \
        if (r_ != 0) {                                                                            \
            fprintf(stderr, "%s returned %d\n", #call, r_);                                       \
            return 1;                                                                             \
        }                                                                                         \
    } while (0)

int main(void) {
    int t = 0;
    for (int i = 0; i < NSEQ; i++) t += LENS[i];
    CHECK_CUDA(cudaSetDevice(0));
    cudaStream_t st;
    CHECK_CUDA(cudaStreamCreate(&st));
    void* ctx = d1_lt_init((size_t)32 << 20);
    if (!ctx) {
        fprintf(stderr, "d1_lt_init failed\n");
        return 1;
    }

    /* host inputs */
    float* hx = malloc(sizeof(float) * t * D);
    float* hw = malloc(sizeof(float) * D);
    uint16_t* hW = malloc(sizeof(uint16_t) * NQKV * D);
    for (int i = 0; i < t * D; i++) hx[i] = 2.0f * uniform();
    for (int i = 0; i < D; i++) hw[i] = 1.0f + 0.25f * uniform();
    for (int i = 0; i < NQKV * D; i++) hW[i] = f2h(0.06f * uniform());

    AttnSeq seqs[NSEQ];
    int work[2 * 64], n_work = 0, off = 0;
    memset(seqs, 0, sizeof(seqs));
    for (int i = 0; i < NSEQ; i++) {
        seqs[i].q_start = seqs[i].kv_start = off;
        seqs[i].q_len = seqs[i].kv_len = LENS[i];
        for (int q = 0; q < LENS[i]; q += 64) {
            work[2 * n_work] = i;
            work[2 * n_work + 1] = q;
            n_work++;
        }
        off += LENS[i];
    }

    float *dx, *dw;
    uint16_t *dxn, *dW, *dY, *dO;
    AttnSeq* dseqs;
    int* dwork;
    CHECK_CUDA(cudaMalloc((void**)&dx, sizeof(float) * t * D));
    CHECK_CUDA(cudaMalloc((void**)&dw, sizeof(float) * D));
    CHECK_CUDA(cudaMalloc((void**)&dxn, 2 * (size_t)t * D));
    CHECK_CUDA(cudaMalloc((void**)&dW, 2 * (size_t)NQKV * D));
    CHECK_CUDA(cudaMalloc((void**)&dY, 2 * (size_t)t * NQKV));
    CHECK_CUDA(cudaMalloc((void**)&dO, 2 * (size_t)t * HEADS * HD));
    CHECK_CUDA(cudaMalloc((void**)&dseqs, sizeof(seqs)));
    CHECK_CUDA(cudaMalloc((void**)&dwork, sizeof(int) * 2 * n_work));
    CHECK_CUDA(cudaMemcpy(dx, hx, sizeof(float) * t * D, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dw, hw, sizeof(float) * D, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dW, hW, 2 * (size_t)NQKV * D, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dseqs, seqs, sizeof(seqs), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dwork, work, sizeof(int) * 2 * n_work, cudaMemcpyHostToDevice));

    const float eps = 1e-5f;
    CHECK_D1(d1_rmsnorm(dx, dw, (d1_half*)dxn, t, D, eps, st));
    const float us = d1_lt_tune(ctx, t, NQKV, D, D, D, 0, NQKV, 0, 0, 0, st);
    if (!(us > 0.0f)) {
        fprintf(stderr, "d1_lt_tune returned %g\n", us);
        return 1;
    }
    CHECK_D1(d1_lt_gemm(ctx, t, NQKV, D, dxn, D, dW, D, 0, dY, NQKV, 0, 0, 1.0f, 0.0f, st));
    const uint16_t* dQ = dY;
    const uint16_t* dK = dY + HEADS * HD;
    const uint16_t* dV = dY + (HEADS + KVH) * HD;
    CHECK_D1(d1_flash_attn((const d1_half*)dQ, NQKV, (const d1_half*)dK, (const d1_half*)dV, NQKV, 0, NULL, NULL,
                           NULL, (d1_half*)dO, HEADS * HD, dseqs, dwork, n_work, HEADS, HEADS / KVH, 0.125f, st));
    CHECK_CUDA(cudaStreamSynchronize(st));
    if (d1_lt_error(ctx) != 0) {
        fprintf(stderr, "d1_lt_error set\n");
        return 1;
    }

    uint16_t* hxn = malloc(2 * (size_t)t * D);
    uint16_t* hY = malloc(2 * (size_t)t * NQKV);
    uint16_t* hO = malloc(2 * (size_t)t * HEADS * HD);
    CHECK_CUDA(cudaMemcpy(hxn, dxn, 2 * (size_t)t * D, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(hY, dY, 2 * (size_t)t * NQKV, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(hO, dO, 2 * (size_t)t * HEADS * HD, cudaMemcpyDeviceToHost));

    int bad = 0;
    /* RMSNorm: y = x / sqrt(mean(x^2) + eps) * w, one fp16 rounding */
    double e_norm = 0.0;
    for (int r = 0; r < t; r++) {
        double ss = 0.0;
        for (int i = 0; i < D; i++) ss += (double)hx[r * D + i] * hx[r * D + i];
        const double inv = 1.0 / sqrt(ss / D + eps);
        for (int i = 0; i < D; i++) {
            const double want = hx[r * D + i] * inv * hw[i], got = h2f(hxn[r * D + i]);
            const double e = fabs(got - want) / (fabs(want) * 9.8e-4 + 1e-6);
            if (e > e_norm) e_norm = e;
        }
    }
    if (e_norm > 1.0) bad = 1;
    /* GEMM: Y = xn . W^T from the device's xn */
    double e_gemm = 0.0;
    for (int r = 0; r < t; r++)
        for (int n = 0; n < NQKV; n++) {
            double acc = 0.0, mag = 0.0;
            for (int k = 0; k < D; k++) {
                const double p = (double)h2f(hxn[r * D + k]) * h2f(hW[n * D + k]);
                acc += p;
                mag += fabs(p);
            }
            const double e = fabs(h2f(hY[r * NQKV + n]) - acc) / (mag + 1e-3);
            if (e > e_gemm) e_gemm = e;
        }
    if (e_gemm > 2e-3) bad = 1;
    /* attention from the device's Q, K, V */
    double e_attn = 0.0;
    double* p = malloc(sizeof(double) * 256);
    for (int s = 0; s < NSEQ; s++)
        for (int h = 0; h < HEADS; h++)
            for (int qi = 0; qi < seqs[s].q_len; qi++) {
                const int q = seqs[s].q_start + qi, g = h / (HEADS / KVH);
                double mx = -1e300, l = 0.0;
                for (int ki = 0; ki < seqs[s].kv_len; ki++) {
                    const int k = seqs[s].kv_start + ki;
                    double dot = 0.0;
                    for (int d = 0; d < HD; d++)
                        dot += (double)h2f(hY[q * NQKV + h * HD + d]) * h2f(hY[k * NQKV + HEADS * HD + g * HD + d]);
                    p[ki] = dot * 0.125;
                    if (p[ki] > mx) mx = p[ki];
                }
                for (int ki = 0; ki < seqs[s].kv_len; ki++) {
                    p[ki] = exp(p[ki] - mx);
                    l += p[ki];
                }
                for (int d = 0; d < HD; d++) {
                    double o = 0.0;
                    for (int ki = 0; ki < seqs[s].kv_len; ki++) {
                        const int k = seqs[s].kv_start + ki;
                        o += p[ki] * h2f(hY[k * NQKV + (HEADS + KVH) * HD + g * HD + d]);
                    }
                    const double e = fabs(h2f(hO[q * HEADS * HD + h * HD + d]) - o / l);
                    if (e > e_attn) e_attn = e;
                }
            }
    if (e_attn > 4e-3) bad = 1;
    printf("rmsnorm err/half-ulp %.3f  gemm rel err %.2e  attention abs err %.2e  (%d rows, %d work items)\n", e_norm,
           e_gemm, e_attn, t, n_work);
    printf(bad ? "FAILED\n" : "ok\n");
    return bad;
}
