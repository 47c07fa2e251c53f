/* gemm_hh_bench.c -- batched FP16 GEMM (sb_gemm_hh: tcgen05 tensor cores,
 * or mma.sync tiles for batches <= 16 on short outputs) or GEMV
 * (sb_gemv_hh, CUDA cores, B <= 8) check + bandwidth harness:
 *
 *   gemm_hh_bench N K B [reps] [--cuda-core]
 *
 * Y[b][n] = sum_k W[n][k] X[b][k], W fp16 N(0, 0.02) and X fp16 N(0, 1)
 * (seeded, subnormals flushed), FP32 output.  Verifies 64 sampled outputs
 * per batch row against a double-precision CPU loop over the same decoded
 * values, then times `reps` launches with CUDA events, rotating over enough
 * copies of W to exceed 4x the 126 MB L2 (fewer when memory is short), and
 * prints one JSON line: {"N", "K", "B", "us", "GB_s", "bytes", "max_rel"}. */
#define _GNU_SOURCE
#include <cuda.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/switch_b200.h"

#define CHK(x) do { CUresult r_ = (x); if (r_) { const char *s_ = NULL; cuGetErrorString(r_, &s_); \
    fprintf(stderr, "CUDA error %d (%s) at %s:%d\n", (int)r_, s_ ? s_ : "?", __FILE__, __LINE__); exit(1); } } while (0)
#define SBK(x) do { int r_ = (x); if (r_) { fprintf(stderr, "%s\n", sb_last_error()); exit(1); } } while (0)

static double h2d(uint16_t h) { /* IEEE half -> double; inputs carry no subnormals */
    const int e = (h >> 10) & 31, m = h & 1023;
    const double v = e == 0 ? 0.0 : ldexp(1.0 + m / 1024.0, e - 15);
    return (h & 0x8000) ? -v : v;
}

int main(int argc, char **argv) {
    if (argc < 4) {
        fprintf(stderr, "usage: gemm_hh_bench N K B [reps] [--cuda-core]\n");
        return 2;
    }
    const int N = atoi(argv[1]), K = atoi(argv[2]), B = atoi(argv[3]);
    const int reps = argc > 4 && argv[4][0] != '-' ? atoi(argv[4]) : 50;
    int cuda_core = 0;
    for (int i = 4; i < argc; i++)
        if (!strcmp(argv[i], "--cuda-core")) cuda_core = 1;
    if (N <= 0 || K <= 0 || K % 8 || B < 1 || B > (cuda_core ? 8 : 256) || reps < 1) {
        fprintf(stderr, "need N > 0, K %% 8 == 0, 1 <= B <= %d, reps >= 1\n", cuda_core ? 8 : 256);
        return 2;
    }
    SBK(sb_init(0));
    const size_t wn = (size_t)N * K, wbytes = wn * 2;
    size_t freeb = 0, totalb = 0;
    CHK(cuMemGetInfo(&freeb, &totalb));
    long copies = (long)((4 * 126e6) / wbytes) + 1;
    if (copies > 64) copies = 64;
    while (copies > 1 && (size_t)copies * wbytes > freeb / 2) copies--;
    uint16_t *hw = malloc(wbytes), *hx = malloc((size_t)B * K * 2);
    sb_synth_normal_h(hw, wn, 0.02f, 11);
    sb_synth_normal_h(hx, (size_t)B * K, 1.0f, 12);
    for (size_t i = 0; i < wn; i++)
        if ((hw[i] & 0x7C00) == 0) hw[i] = 0;
    for (long i = 0; i < (long)B * K; i++)
        if ((hx[i] & 0x7C00) == 0) hx[i] = 0;
    CUdeviceptr dw, dx, dy;
    CHK(cuMemAlloc(&dw, (size_t)copies * wbytes));
    CHK(cuMemAlloc(&dx, (size_t)B * K * 2));
    CHK(cuMemAlloc(&dy, (size_t)B * N * 4));
    for (long c = 0; c < copies; c++) CHK(cuMemcpyHtoD(dw + (size_t)c * wbytes, hw, wbytes));
    CHK(cuMemcpyHtoD(dx, hx, (size_t)B * K * 2));
#define RUN(w) (cuda_core ? sb_gemv_hh((const uint16_t *)(uintptr_t)(w), (const uint16_t *)(uintptr_t)dx, \
                                       (float *)(uintptr_t)dy, K, N, B, NULL)                            \
                          : sb_gemm_hh((const uint16_t *)(uintptr_t)(w), (const uint16_t *)(uintptr_t)dx, \
                                       (float *)(uintptr_t)dy, K, N, B, NULL))
    SBK(RUN(dw));
    CHK(cuCtxSynchronize());
    float *hy = malloc((size_t)B * N * 4);
    CHK(cuMemcpyDtoH(hy, dy, (size_t)B * N * 4));
    double max_rel = 0;
    for (int b = 0; b < B; b++)
        for (int s = 0; s < 64; s++) {
            const int n = (int)(((long)s * 7919 + b * 131) % N);
            double ref = 0, mag = 0;
            for (int k = 0; k < K; k++) {
                const double p = h2d(hw[(size_t)n * K + k]) * h2d(hx[(size_t)b * K + k]);
                ref += p;
                mag += fabs(p);
            }
            const double rel = fabs(hy[(size_t)b * N + n] - ref) / (mag > 0 ? mag : 1);
            if (rel > max_rel) max_rel = rel;
        }
    int err = 0;
    if (!cuda_core) SBK(sb_tc_error(&err));
    CUevent e0, e1;
    CHK(cuEventCreate(&e0, 0));
    CHK(cuEventCreate(&e1, 0));
    for (int r = 0; r < 3; r++) SBK(RUN(dw + (size_t)(r % copies) * wbytes));
    CHK(cuEventRecord(e0, NULL));
    for (int r = 0; r < reps; r++) SBK(RUN(dw + (size_t)(r % copies) * wbytes));
    CHK(cuEventRecord(e1, NULL));
    CHK(cuEventSynchronize(e1));
    float ms = 0;
    CHK(cuEventElapsedTime(&ms, e0, e1));
    const double us = ms * 1e3 / reps;
    const double bytes = (double)wbytes + (double)B * K * 2 + (double)B * N * 4;
    printf("{\"N\": %d, \"K\": %d, \"B\": %d, \"path\": \"%s\", \"us\": %.3f, \"GB_s\": %.1f, \"bytes\": %.0f, "
           "\"copies\": %ld, \"max_rel\": %.3g, \"device_error\": %d}\n",
           N, K, B,
           cuda_core ? "gemv_hh (CUDA cores)"
           : (B <= 16 && N < 128L * sb_sm_count()) ? "gemm_hh_mma (mma.sync, one launch)"
                                                    : "gemm_hh_tc (tcgen05)",
           us, bytes / (us * 1e-6) / 1e9,
           bytes, copies, max_rel, err);
    return (max_rel <= 1e-4 && !err) ? 0 : 1;
}
