/* gpu_workload.c -- the SGEMM + memory-bandwidth suite on B200, with the
 * reference harness's CLI and JSON contract (gpu_workload.c of
 * pkia/switch-l4t-gpu; consumed by deploy/cluster/gpu_task_example.py).
 *
 *   gpu_workload [--json] [--sizes 256,512,1024] [--membw-mib 2048] [--tf32x3]
 *                [--gpus N [--dist-n 16384]] [module]
 *
 * `module` is a cubin/PTX image loaded with cuModuleLoadData (default: the
 * switch_gpu.cubin installed next to this binary).  Kernels are resolved by
 * the reference's names; sgemm_tiled and membw_read4 are required,
 * sgemm_naive / sgemm_tiled4 / sgemm_opt optional (a failing lookup drops
 * their lines and JSON keys, gpu_workload.c:69-74).  Each SGEMM kernel is
 * launched with the reference's own geometry (grid n/32 or n/64 squared,
 * 16x16 threads), verified at n = 256 against the same CPU triple loop and
 * tolerance (|d| > 0.05|ref| + 1e-3 is a bad cell), then timed over 10
 * launches (CUDA events; the wall clock is kept for the "ms" the reference
 * reports).  Data: srand(42), (rand() % 2000 - 1000) / 1000, as the
 * reference.  The bandwidth probe streams a buffer far larger than the
 * 126 MB L2 (the reference's 64 MB would fit in it).
 *
 * JSON keys are the reference's (ptx, kernels, sgemm, sgemm4, sgemm_opt,
 * membw_gbps, done) plus additive ones (device, sm_count, sgemm_b200,
 * membw_bytes, fp32_peak_gflops_at_max_clock, and with --tf32x3 the opt-in
 * tensor-core SGEMM of this package: kernels.sgemm_3xtf32, sgemm_3xtf32).
 *
 * --gpus N (additive; the reference has no multi-GPU path): after the suite,
 * the dist-n^3 SGEMM sharded by row panels over devices 0..N-1, one host
 * thread per device on its primary context, each rank computing its panel
 * with sb_sgemm_rows and an in-place NCCL all-gather of C
 * (sb_sgemm_panel_allgather over a non-blocking communicator with bounded
 * waits).  Every rank then checks sampled cells of ALL panels of its
 * gathered C against the harness's CPU loop and tolerance.  JSON key
 * sgemm_dist; text line "sgemm_dist ...: CORRECT|WRONG". */
#define _GNU_SOURCE
#include <cuda.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "../../include/switch_b200.h"

static int json_mode;
#define OUT(...) do { if (!json_mode) printf(__VA_ARGS__); } while (0)
#define CHK(x) do { CUresult r_ = (x); if (r_) { const char *s_ = NULL; cuGetErrorString(r_, &s_); \
    fprintf(stderr, "CUDA error %d (%s) at %s:%d\n", (int)r_, s_ ? s_ : "?", __FILE__, __LINE__); exit(1); } } while (0)

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec / 1e9;
}

static char *read_file(const char *path, size_t *len) {
    FILE *f = fopen(path, "rb");
    if (!f) { perror(path); exit(1); }
    fseek(f, 0, SEEK_END);
    *len = (size_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    char *buf = malloc(*len + 1);
    if (fread(buf, 1, *len, f) != *len) exit(1);
    buf[*len] = 0;
    fclose(f);
    return buf;
}

static const char *default_module(void) {
    static char p[4096];
    ssize_t n = readlink("/proc/self/exe", p, sizeof p - 64);
    if (n > 0) {
        p[n] = 0;
        char *s = strrchr(p, '/');
        if (s) {
            strcpy(s, "/../lib/switch_gpu.cubin");
            if (access(p, R_OK) == 0) return p;
        }
    }
    return "switch_gpu.cubin";
}

/* CPU golden check of gpu_workload.c:92-115: returns the bad-row count
 * (stops at the first bad column of a row, at most 5 rows). */
static int verify(const float *A, const float *B, const float *C, int n, int full) {
    int bad = 0;
    for (int i = 0; i < n && (full || bad < 5); i++)
        for (int j = 0; j < n; j++) {
            float ref = 0;
            for (int k = 0; k < n; k++) ref += A[i * n + k] * B[k * n + j];
            float d = C[i * n + j] - ref;
            if (d < 0) d = -d;
            if (d > 0.05f * (ref < 0 ? -ref : ref) + 1e-3f) {
                if (bad < 3) OUT("  mismatch [%d][%d]: got %.4f want %.4f\n", i, j, C[i * n + j], ref);
                bad++;
                if (!full) break;
            }
        }
    return bad;
}

/* ---- --gpus N: row-panel SGEMM + NCCL all-gather, one thread per device */
typedef struct {
    int rank, world, n;
    const unsigned char *uid;
    const float *hB; /* the replicated B, n x n, on the host */
    double comp_ms, tot_ms;
    int bad, checked, rc;
    char msg[256];
} dist_rank;

#define DIST_SEED_A 5000ull
#define DIST_CELLS 16 /* sampled cells per panel */
#define DIST_TIMEOUT_S 120.0

static void *dist_thread(void *p) {
    dist_rank *a = p;
    const int n = a->n, R = (n + a->world - 1) / a->world;
    const int row0 = a->rank * R < n ? a->rank * R : n, row1 = row0 + R < n ? row0 + R : n;
    CUdevice dev;
    CUcontext ctx;
    void *comm = NULL;
    CUstream st = NULL;
    CUdeviceptr dA = 0, dB = 0, dC = 0;
    CUevent ev[4] = {NULL, NULL, NULL, NULL};
    float *row = malloc((size_t)n * 4), *crow = malloc((size_t)n * 4);
#define DFAIL(what) do { snprintf(a->msg, sizeof a->msg, "rank %d: %s: %s", a->rank, what, sb_last_error()); a->rc = 1; goto out; } while (0)
#define DCK(x) do { if ((x) != CUDA_SUCCESS) DFAIL(#x); } while (0)
    DCK(cuDeviceGet(&dev, a->rank));
    DCK(cuDevicePrimaryCtxRetain(&ctx, dev));
    DCK(cuCtxSetCurrent(ctx));
    if (sb_nccl_comm_init(&comm, a->world, a->uid, a->rank, DIST_TIMEOUT_S)) DFAIL("communicator");
    DCK(cuStreamCreate(&st, CU_STREAM_NON_BLOCKING));
    const size_t nn = (size_t)n * n * 4;
    DCK(cuMemAlloc(&dA, nn));
    DCK(cuMemAlloc(&dB, nn));
    DCK(cuMemAlloc(&dC, (size_t)a->world * R * n * 4));
    for (int i = row0; i < row1; i++) { /* this rank's rows of A: row i from its own seeded stream */
        sb_synth_uniform(row, (size_t)n, -1.0f, 1.0f, DIST_SEED_A + (uint64_t)i);
        DCK(cuMemcpyHtoD(dA + (size_t)i * n * 4, row, (size_t)n * 4));
    }
    DCK(cuMemcpyHtoD(dB, a->hB, nn));
    for (int k = 0; k < 4; k++) DCK(cuEventCreate(&ev[k], 0));
    const float *pA = (const float *)(uintptr_t)dA, *pB = (const float *)(uintptr_t)dB;
    float *pC = (float *)(uintptr_t)dC;
    const int reps = 5;
    for (int it = 0; it < 2 + reps; it++) { /* 2 warm-up iterations */
        if (it == 2) DCK(cuEventRecord(ev[0], st));
        if (sb_sgemm_panel_allgather(pA, pB, pC, n, n, n, a->rank, a->world, comm, 0, st)) DFAIL("panel");
    }
    DCK(cuEventRecord(ev[1], st));
    DCK(cuEventRecord(ev[2], st));
    for (int it = 0; it < reps; it++)
        if (sb_sgemm_panel_allgather(pA, pB, pC, n, n, n, a->rank, a->world, comm, 1, st)) DFAIL("panel + gather");
    DCK(cuEventRecord(ev[3], st));
    if (sb_nccl_wait(comm, st, DIST_TIMEOUT_S)) DFAIL("wait");
    float ms = 0;
    DCK(cuEventElapsedTime(&ms, ev[0], ev[1]));
    a->comp_ms = ms / reps;
    DCK(cuEventElapsedTime(&ms, ev[2], ev[3]));
    a->tot_ms = ms / reps;
    /* the gathered C: sampled cells of every panel against the harness loop */
    for (int q = 0; q < a->world; q++) {
        const int q0 = q * R, q1 = q0 + R < n ? q0 + R : n;
        for (int c = 0; c < DIST_CELLS && q1 > q0; c++) {
            const int i = q0 + (int)(((long)c * 7919 + q * 131) % (q1 - q0));
            const int j = (int)(((long)c * 104729 + q * 31 + 17) % n);
            sb_synth_uniform(row, (size_t)n, -1.0f, 1.0f, DIST_SEED_A + (uint64_t)i);
            float ref = 0; /* gpu_workload.c:97-98 */
            for (int k = 0; k < n; k++) ref += row[k] * a->hB[(size_t)k * n + j];
            DCK(cuMemcpyDtoH(crow, dC + ((size_t)i * n + j) * 4, 4));
            float d = crow[0] - ref;
            if (d < 0) d = -d;
            if (d > 0.05f * (ref < 0 ? -ref : ref) + 1e-3f) a->bad++;
            a->checked++;
        }
    }
out:
    for (int k = 0; k < 4; k++)
        if (ev[k]) cuEventDestroy(ev[k]);
    if (comm) {
        if (a->rc) sb_nccl_abort(comm);
        else if (sb_nccl_comm_destroy(comm, DIST_TIMEOUT_S)) {
            snprintf(a->msg, sizeof a->msg, "rank %d: destroy: %s", a->rank, sb_last_error());
            a->rc = 1;
        }
    }
    if (dA) cuMemFree(dA);
    if (dB) cuMemFree(dB);
    if (dC) cuMemFree(dC);
    if (st) cuStreamDestroy(st);
    free(row);
    free(crow);
    return NULL;
#undef DCK
#undef DFAIL
}

typedef struct {
    const char *name, *json_key;
    CUfunction f;
    int tile; /* reference grid divisor */
    double ms[16], gf[16];
    const char *verdict;
} kern;

int main(int argc, char **argv) {
    const char *mod_path = NULL;
    int sizes[16] = {256, 512, 1024}, nsizes = 3;
    long membw_mib = 2048;
    int tf32x3 = 0, gpus = 0, dist_n = 16384;
    const char *v_t3 = NULL;
    double t3_ms[16] = {0}, t3_gf[16] = {0};
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "--json")) json_mode = 1;
        else if (!strcmp(argv[i], "--sizes") && i + 1 < argc) {
            nsizes = 0;
            for (char *t = strtok(argv[++i], ","); t && nsizes < 16; t = strtok(NULL, ",")) sizes[nsizes++] = atoi(t);
        } else if (!strcmp(argv[i], "--membw-mib") && i + 1 < argc) membw_mib = atol(argv[++i]);
        else if (!strcmp(argv[i], "--tf32x3")) tf32x3 = 1;
        else if (!strcmp(argv[i], "--gpus") && i + 1 < argc) gpus = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--dist-n") && i + 1 < argc) dist_n = atoi(argv[++i]);
        else mod_path = argv[i];
    }
    if (!mod_path) mod_path = default_module();
    size_t plen;
    char *image = read_file(mod_path, &plen);

    CUdevice dev;
    CUcontext ctx;
    CUmodule mod;
    CHK(cuInit(0));
    CHK(cuDeviceGet(&dev, 0));
    CHK(cuDevicePrimaryCtxRetain(&ctx, dev)); /* primary context: shared with the runtime/NCCL */
    CHK(cuCtxSetCurrent(ctx));
    CHK(cuModuleLoadData(&mod, image));
    char devname[256] = "";
    int sms = 0, clk_khz = 0;
    cuDeviceGetName(devname, sizeof devname, dev);
    cuDeviceGetAttribute(&sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev);
    cuDeviceGetAttribute(&clk_khz, CU_DEVICE_ATTRIBUTE_CLOCK_RATE, dev);

    kern ks[4] = {{"sgemm", "sgemm", NULL, 32, {0}, {0}, NULL},
                  {"sgemm_tiled4", "sgemm4", NULL, 64, {0}, {0}, NULL},
                  {"sgemm_opt", "sgemm_opt", NULL, 64, {0}, {0}, NULL},
                  {"sgemm_b200", "sgemm_b200", NULL, 0, {0}, {0}, NULL}};
    CUfunction membw, naive = NULL;
    CHK(cuModuleGetFunction(&ks[0].f, mod, "sgemm_tiled"));
    CHK(cuModuleGetFunction(&membw, mod, "membw_read4"));
    cuModuleGetFunction(&naive, mod, "sgemm_naive");
    cuModuleGetFunction(&ks[1].f, mod, "sgemm_tiled4");
    cuModuleGetFunction(&ks[2].f, mod, "sgemm_opt");
    cuModuleGetFunction(&ks[3].f, mod, "sgemm_b200");
    const char *v_naive = NULL;
    CUevent e0, e1;
    CHK(cuEventCreate(&e0, 0));
    CHK(cuEventCreate(&e1, 0));

    for (int si = 0; si < nsizes; si++) {
        const int n = sizes[si];
        const size_t bytes = (size_t)n * n * 4;
        float *A = malloc(bytes), *B = malloc(bytes), *C = malloc(bytes);
        srand(42);
        for (size_t i = 0; i < (size_t)n * n; i++) {
            A[i] = (rand() % 2000 - 1000) / 1000.0f;
            B[i] = (rand() % 2000 - 1000) / 1000.0f;
        }
        CUdeviceptr dA, dB, dC;
        CHK(cuMemAlloc(&dA, bytes));
        CHK(cuMemAlloc(&dB, bytes));
        CHK(cuMemAlloc(&dC, bytes));
        CHK(cuMemcpyHtoD(dA, A, bytes));
        CHK(cuMemcpyHtoD(dB, B, bytes));
        int Mn = n, Nn = n, Kn = n;
        void *args[] = {&dA, &dB, &dC, &Mn, &Nn, &Kn};
        for (int ki = 0; ki < 4; ki++) {
            kern *k = &ks[ki];
            if (!k->f) continue;
            unsigned gx, gy = 1;
            if (k->tile) { gx = (unsigned)((n + k->tile - 1) / k->tile); gy = gx; }
            else gx = (unsigned)((n + 127) / 128) * (unsigned)((n + 127) / 128); /* one CTA per tile */
            const unsigned bx = k->tile ? 16 : 256, by = k->tile ? 16 : 1;
            CHK(cuMemsetD32(dC, 0, (size_t)n * n));
            CHK(cuLaunchKernel(k->f, gx, gy, 1, bx, by, 1, 0, NULL, args, NULL));
            CHK(cuCtxSynchronize());
            if (n == 256) {
                CHK(cuMemcpyDtoH(C, dC, bytes));
                k->verdict = verify(A, B, C, n, 0) ? "WRONG" : "CORRECT";
                OUT("%s %d: %s\n", k->name, n, k->verdict);
                if (ki == 0 && naive) {
                    CHK(cuMemsetD32(dC, 0, (size_t)n * n));
                    CHK(cuLaunchKernel(naive, n / 16, n / 16, 1, 16, 16, 1, 0, NULL, args, NULL));
                    CHK(cuCtxSynchronize());
                    CHK(cuMemcpyDtoH(C, dC, bytes));
                    int nbad = verify(A, B, C, n, 1);
                    v_naive = nbad ? "WRONG" : "CORRECT";
                    OUT("sgemm_naive %d: %s (%d bad cells)\n", n, v_naive, nbad);
                }
            }
            CHK(cuEventRecord(e0, NULL));
            double t0 = now_s();
            for (int r = 0; r < 10; r++) CHK(cuLaunchKernel(k->f, gx, gy, 1, bx, by, 1, 0, NULL, args, NULL));
            CHK(cuEventRecord(e1, NULL));
            CHK(cuEventSynchronize(e1));
            (void)t0;
            float ms10 = 0;
            CHK(cuEventElapsedTime(&ms10, e0, e1));
            k->ms[si] = ms10 / 10.0;
            k->gf[si] = 2.0 * n * (double)n * n / (k->ms[si] * 1e-3) / 1e9;
            OUT("%s %dx%dx%d: %.3f ms/iter, %.1f GFLOPS\n", ki == 0 ? "sgemm" : k->name, n, n, n, k->ms[si], k->gf[si]);
        }
        if (tf32x3) { /* opt-in: sb_sgemm_3xtf32 through the C-ABI library */
            const float *pa = (const float *)(uintptr_t)dA, *pb = (const float *)(uintptr_t)dB;
            float *pc = (float *)(uintptr_t)dC;
            CHK(cuMemsetD32(dC, 0, (size_t)n * n));
            if (sb_sgemm_3xtf32(pa, pb, pc, n, n, n, NULL)) { fprintf(stderr, "%s\n", sb_last_error()); exit(1); }
            CHK(cuCtxSynchronize());
            if (n == 256) {
                CHK(cuMemcpyDtoH(C, dC, bytes));
                v_t3 = verify(A, B, C, n, 0) ? "WRONG" : "CORRECT";
                OUT("sgemm_3xtf32 %d: %s\n", n, v_t3);
            }
            CHK(cuEventRecord(e0, NULL));
            for (int r = 0; r < 10; r++)
                if (sb_sgemm_3xtf32(pa, pb, pc, n, n, n, NULL)) { fprintf(stderr, "%s\n", sb_last_error()); exit(1); }
            CHK(cuEventRecord(e1, NULL));
            CHK(cuEventSynchronize(e1));
            float ms10 = 0;
            CHK(cuEventElapsedTime(&ms10, e0, e1));
            t3_ms[si] = ms10 / 10.0;
            t3_gf[si] = 2.0 * n * (double)n * n / (t3_ms[si] * 1e-3) / 1e9;
            OUT("sgemm_3xtf32 %dx%dx%d: %.3f ms/iter, %.1f GFLOPS\n", n, n, n, t3_ms[si], t3_gf[si]);
        }
        cuMemFree(dA);
        cuMemFree(dB);
        cuMemFree(dC);
        free(A);
        free(B);
        free(C);
    }

    /* ---- memory bandwidth (read), buffer >> L2 */
    double membw_gbs = 0, mbytes = 0;
    {
        long n4l = membw_mib * 1024L * 1024L / 16;
        if (n4l > 0x7fffffffL) n4l = 0x7fffffffL;
        int n4 = (int)n4l, iters = 4;
        size_t bytes = (size_t)n4 * 16;
        CUdeviceptr dbuf, dout;
        CHK(cuMemAlloc(&dbuf, bytes));
        CHK(cuMemsetD32(dbuf, 0x3a83126f, bytes / 4)); /* 0.001f */
        unsigned grid = 4 * (unsigned)sms;
        CHK(cuMemAlloc(&dout, (size_t)grid * 256 * 4));
        void *margs[] = {&dbuf, &dout, &n4, &iters};
        CHK(cuLaunchKernel(membw, grid, 1, 1, 256, 1, 1, 0, NULL, margs, NULL));
        CHK(cuCtxSynchronize());
        CHK(cuEventRecord(e0, NULL));
        CHK(cuLaunchKernel(membw, grid, 1, 1, 256, 1, 1, 0, NULL, margs, NULL));
        CHK(cuEventRecord(e1, NULL));
        CHK(cuEventSynchronize(e1));
        float ms = 0;
        CHK(cuEventElapsedTime(&ms, e0, e1));
        mbytes = (double)bytes * iters;
        membw_gbs = mbytes / (ms * 1e-3) / 1e9;
        OUT("membw read (%ld MiB x%d): %.3f s, %.1f GB/s\n", membw_mib, iters, ms * 1e-3, membw_gbs);
        cuMemFree(dbuf);
        cuMemFree(dout);
    }

    /* ---- --gpus N: row-panel SGEMM over N devices + NCCL all-gather of C */
    dist_rank dr[64];
    double dist_comp = 0, dist_tot = 0;
    int dist_bad = 0, dist_checked = 0;
    if (gpus > 0) {
        int ndev = 0;
        CHK(cuDeviceGetCount(&ndev));
        if (gpus > ndev || gpus > 64 || dist_n < 1) {
            fprintf(stderr, "--gpus %d: only %d device(s) visible (or bad --dist-n)\n", gpus, ndev);
            return 1;
        }
        unsigned char uid[128];
        if (sb_nccl_unique_id(uid)) { fprintf(stderr, "%s\n", sb_last_error()); return 1; }
        float *hB = malloc((size_t)dist_n * dist_n * 4);
        for (int k = 0; k < dist_n; k++) /* row k of B from its own seeded stream */
            sb_synth_uniform(hB + (size_t)k * dist_n, (size_t)dist_n, -1.0f, 1.0f, 777000ull + (uint64_t)k);
        pthread_t th[64];
        for (int r = 0; r < gpus; r++) {
            memset(&dr[r], 0, sizeof dr[r]);
            dr[r].rank = r;
            dr[r].world = gpus;
            dr[r].n = dist_n;
            dr[r].uid = uid;
            dr[r].hB = hB;
            pthread_create(&th[r], NULL, dist_thread, &dr[r]);
        }
        int failed = 0;
        for (int r = 0; r < gpus; r++) {
            pthread_join(th[r], NULL);
            if (dr[r].rc) { fprintf(stderr, "%s\n", dr[r].msg); failed = 1; }
            if (dr[r].comp_ms > dist_comp) dist_comp = dr[r].comp_ms;
            if (dr[r].tot_ms > dist_tot) dist_tot = dr[r].tot_ms;
            dist_bad += dr[r].bad;
            dist_checked += dr[r].checked;
        }
        free(hB);
        CHK(cuCtxSetCurrent(ctx));
        if (failed) return 1;
        const double fl = 2.0 * dist_n * (double)dist_n * dist_n;
        OUT("sgemm_dist %d^3 over %d GPU(s): compute %.3f ms (%.1f TFLOP/s), with all-gather %.3f ms (%.1f TFLOP/s); "
            "%d cells of the gathered C checked on every rank: %s\n", dist_n, gpus, dist_comp, fl / (dist_comp * 1e9),
            dist_tot, fl / (dist_tot * 1e9), dist_checked, dist_bad ? "WRONG" : "CORRECT");
    }

    if (json_mode) {
        printf("{\"ptx\":\"");
        for (const char *p = mod_path; *p; p++) {
            if (*p == '"' || *p == '\\') putchar('\\');
            putchar(*p);
        }
        printf("\",\"kernels\":{\"sgemm\":\"%s\"", ks[0].verdict ? ks[0].verdict : "NOT_RUN");
        if (v_naive) printf(",\"sgemm_naive\":\"%s\"", v_naive);
        if (ks[1].verdict) printf(",\"sgemm_tiled4\":\"%s\"", ks[1].verdict);
        if (ks[2].verdict) printf(",\"sgemm_opt\":\"%s\"", ks[2].verdict);
        if (ks[3].verdict) printf(",\"sgemm_b200\":\"%s\"", ks[3].verdict);
        if (v_t3) printf(",\"sgemm_3xtf32\":\"%s\"", v_t3);
        printf("}");
        for (int ki = 0; ki < 4; ki++) {
            if (!ks[ki].f) continue;
            printf(",\"%s\":[", ks[ki].json_key);
            for (int i = 0; i < nsizes; i++)
                printf("%s{\"n\":%d,\"ms\":%.3f,\"gflops\":%.1f}", i ? "," : "", sizes[i], ks[ki].ms[i], ks[ki].gf[i]);
            printf("]");
        }
        if (tf32x3) {
            printf(",\"sgemm_3xtf32\":[");
            for (int i = 0; i < nsizes; i++)
                printf("%s{\"n\":%d,\"ms\":%.3f,\"gflops\":%.1f}", i ? "," : "", sizes[i], t3_ms[i], t3_gf[i]);
            printf("]");
        }
        if (gpus > 0) {
            const double fl = 2.0 * dist_n * (double)dist_n * dist_n;
            printf(",\"sgemm_dist\":{\"n\":%d,\"gpus\":%d,\"compute_ms\":%.3f,\"ms\":%.3f,\"allgather_ms\":%.3f,"
                   "\"compute_tflops\":%.2f,\"tflops\":%.2f,\"cells_checked\":%d,\"verdict\":\"%s\"}",
                   dist_n, gpus, dist_comp, dist_tot, dist_tot - dist_comp, fl / (dist_comp * 1e9),
                   fl / (dist_tot * 1e9), dist_checked, dist_bad ? "WRONG" : "CORRECT");
        }
        printf(",\"membw_gbps\":%.1f,\"membw_bytes\":%.0f,\"device\":\"%s\",\"sm_count\":%d,"
               "\"fp32_peak_gflops_at_max_clock\":%.1f,\"done\":true}\n",
               membw_gbs, mbytes, devname, sms, sms * 128.0 * 2.0 * clk_khz / 1e6);
    } else {
        printf("WORKLOAD_DONE\n");
    }
    return 0;
}
