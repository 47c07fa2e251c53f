/* gemv_test.c -- FP32 GEMV verify + bandwidth harness with the reference's
 * CLI and verdict contract (gpu-llm/harness/gemv_test.c):
 *
 *   gemv_test [module] [N] [K]      (defaults: gemv.cubin next to the binary, 4096 4096)
 *
 * Loads the module with cuModuleLoadData, launches gemv, gemv4 and gemv_warp
 * with the reference's geometry (block 256; grid ceil(N/256), or ceil(N/8)
 * for gemv_warp), checks each against the same serial CPU golden loop on
 * the same LCG inputs (seed 42, uniform [-0.5, 0.5)) with the same
 * tolerance (|d| > 1e-4 |ref| + 1e-4 is a mismatch), then times 20 launches
 * per rep (best of 3, CUDA events).  Unlike the reference, W is rotated over
 * enough copies to exceed the 126 MB L2, so the GB/s is an HBM figure.
 * Prints GEMV_TEST_DONE / GEMV_TEST_FAILED and exits 0 / 1. */
#define _GNU_SOURCE
#include <cuda.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define CHK(x) do { CUresult r_ = (x); if (r_) { const char *s_ = NULL; cuGetErrorString(r_, &s_); \
    fprintf(stderr, "CUDA error %d (%s) at %s:%d\n", (int)r_, s_ ? s_ : "?", __FILE__, __LINE__); exit(1); } } while (0)

static unsigned long rng_state = 42;
static float frand(void) { /* the reference harness's LCG, gemv_test.c:46-50 */
    rng_state = rng_state * 6364136223846793005UL + 1442695040888963407UL;
    return (float)((rng_state >> 40) & 0xFFFFFF) / (float)0x1000000;
}

static char *read_file(const char *path) {
    FILE *f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "cannot open %s\n", path); exit(1); }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    char *buf = malloc(n + 1);
    if (fread(buf, 1, n, f) != (size_t)n) { fprintf(stderr, "short read\n"); exit(1); }
    fclose(f);
    buf[n] = 0;
    return buf;
}

static const char *default_module(void) {
    static char p[4096];
    ssize_t n = readlink("/proc/self/exe", p, sizeof p - 64);
    if (n > 0) {
        p[n] = 0;
        char *s = strrchr(p, '/');
        if (s) {
            strcpy(s, "/../lib/gemv.cubin");
            if (access(p, R_OK) == 0) return p;
        }
    }
    return "gemv.cubin";
}

int main(int argc, char **argv) {
    const char *mod_path = argc > 1 ? argv[1] : default_module();
    int N = argc > 2 ? atoi(argv[2]) : 4096;
    int K = argc > 3 ? atoi(argv[3]) : 4096;
    if (K % 4) { fprintf(stderr, "K must be a multiple of 4\n"); return 1; }
    char *image = read_file(mod_path);
    CUdevice dev;
    CUcontext ctx;
    CUmodule mod;
    CHK(cuInit(0));
    CHK(cuDeviceGet(&dev, 0));
    char name[256];
    CHK(cuDeviceGetName(name, sizeof name, dev));
    printf("device: %s\n", name);
    CHK(cuDevicePrimaryCtxRetain(&ctx, dev));
    CHK(cuCtxSetCurrent(ctx));
    CHK(cuModuleLoadData(&mod, image));
    const char *names[3] = {"gemv", "gemv4", "gemv_warp"};
    CUfunction fns[3] = {NULL, NULL, NULL};
    CHK(cuModuleGetFunction(&fns[0], mod, "gemv"));
    cuModuleGetFunction(&fns[1], mod, "gemv4");
    cuModuleGetFunction(&fns[2], mod, "gemv_warp");
    printf("GEMV %dx%d (fp32), weights %.1f MB\n", N, K, (double)N * K * 4 / 1048576.0);

    const size_t wbytes = (size_t)N * K * 4;
    float *W = malloc(wbytes), *x = malloc((size_t)K * 4), *y = malloc((size_t)N * 4), *yref = malloc((size_t)N * 4);
    for (size_t i = 0; i < (size_t)N * K; i++) W[i] = frand() - 0.5f;
    for (int i = 0; i < K; i++) x[i] = frand() - 0.5f;
    for (int n = 0; n < N; n++) { /* CPU golden, gemv_test.c:85-90 */
        const float *row = W + (size_t)n * K;
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc += row[k] * x[k];
        yref[n] = acc;
    }
    /* enough copies of W to exceed L2 for the timing loop */
    int copies = (int)((512ull << 20) / wbytes) + 1;
    if (copies > 64) copies = 64;
    CUdeviceptr dW, dx, dy;
    CHK(cuMemAlloc(&dW, wbytes * copies));
    CHK(cuMemAlloc(&dx, (size_t)K * 4));
    CHK(cuMemAlloc(&dy, (size_t)N * 4));
    for (int c = 0; c < copies; c++) CHK(cuMemcpyHtoD(dW + wbytes * c, W, wbytes));
    CHK(cuMemcpyHtoD(dx, x, (size_t)K * 4));
    CUevent e0, e1;
    CHK(cuEventCreate(&e0, 0));
    CHK(cuEventCreate(&e1, 0));
    int fails = 0;
    for (int v = 0; v < 3; v++) {
        if (!fns[v]) { printf("note: %s not found in module, skipping\n", names[v]); continue; }
        void *args[] = {&dW, &dx, &dy, &K, &N};
        unsigned gx = (v == 2) ? (unsigned)((N + 7) / 8) : (unsigned)((N + 255) / 256);
        CHK(cuMemsetD32(dy, 0x7fc00000, N));
        CHK(cuLaunchKernel(fns[v], gx, 1, 1, 256, 1, 1, 0, NULL, args, NULL));
        CHK(cuCtxSynchronize());
        CHK(cuMemcpyDtoH(y, dy, (size_t)N * 4));
        int bad = 0;
        float maxabs = 0;
        for (int n = 0; n < N; n++) {
            float diff = y[n] - yref[n];
            if (diff < 0) diff = -diff;
            float ref = yref[n] < 0 ? -yref[n] : yref[n];
            if (!(diff <= maxabs)) maxabs = diff;
            if (!(diff <= 1e-4f * ref + 1e-4f) && ++bad <= 3) printf("  mismatch n=%d got=%f want=%f\n", n, y[n], yref[n]);
        }
        printf("%s: %s (max abs err %.2e)\n", names[v], bad ? "WRONG" : "CORRECT", maxabs);
        if (bad) fails++;
        float best = 1e30f;
        for (int rep = 0; rep < 3; rep++) {
            CHK(cuEventRecord(e0, NULL));
            for (int it = 0; it < 20; it++) {
                CUdeviceptr w = dW + wbytes * (size_t)((rep * 20 + it) % copies);
                void *a2[] = {&w, &dx, &dy, &K, &N};
                CHK(cuLaunchKernel(fns[v], gx, 1, 1, 256, 1, 1, 0, NULL, a2, NULL));
            }
            CHK(cuEventRecord(e1, NULL));
            CHK(cuEventSynchronize(e1));
            float ms;
            CHK(cuEventElapsedTime(&ms, e0, e1));
            if (ms < best) best = ms;
        }
        double bytes = 20.0 * ((double)N * K * 4 + (double)K * 4 + (double)N * 4);
        double gbps = bytes / (best * 1e-3) / 1e9;
        printf("%s: %.4f ms/call -> %.1f GB/s (HBM, W rotated over %d copies)\n", names[v], best / 20, gbps, copies);
    }
    printf("%s\n", fails ? "GEMV_TEST_FAILED" : "GEMV_TEST_DONE");
    return fails ? 1 : 0;
}
