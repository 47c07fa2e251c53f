// gemv_m0.cu -- the "gemv" module image (sm_100a cubin): the reference's
// milestone-0 FP32 GEMV kernels (gpu-llm/kernels/gemv.cu), y[n] = W[n,:] . x,
// W row-major [N][K].  All three names run the same warp-per-row streaming
// body (grid-stride over every warp of the launch), so the stock launches of
// gemv_test.c:109 (grid ceil(N/256) for gemv/gemv4, ceil(N/8) for gemv_warp,
// block 256) and any others are correct.  This also removes the reference
// gemv_warp's divergent-barrier hazard (gemv.cu:27-47): there is no block
// barrier at all.
#include "sb_gemv.cuh"

SB_DEV void gemv_m0_body(const float *__restrict__ W, const float *__restrict__ x, float *__restrict__ y, int K,
                         int N) {
    const int nthreads = gridDim.x * blockDim.x;
    const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec = ((K & 3) == 0) && ((((uintptr_t)W) & 15) == 0) && ((((uintptr_t)x) & 15) == 0);
    if (vec && (blockDim.x & 31) == 0) {
        const int warp = gtid >> 5, nwarp = nthreads >> 5, cpr = K >> 2;
        XGlob4 xa{x};
        for (int n0 = warp * 2; n0 < N; n0 += nwarp * 2) {
            int rows[2];
            consecutive_rows<2>(n0, N, rows);
            float acc[2];
            warp_dot_f<2, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cpr, xa, acc);
            const int lane = threadIdx.x & 31;
            if (lane < 2 && rows[lane] >= 0) y[rows[lane]] = acc[lane];
        }
        return;
    }
    for (int n = gtid; n < N; n += nthreads) {
        const float *row = W + (size_t)n * K;
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc = fmaf(row[k], x[k], acc);
        y[n] = acc;
    }
}

// Reference: gemv.cu:3-14 (thread per row).
extern "C" __global__ void gemv(const float *__restrict__ W, const float *__restrict__ x, float *__restrict__ y,
                                int K, int N) {
    gemv_m0_body(W, x, y, K, N);
}
// Reference: gemv.cu:18-48 (warp per row).
extern "C" __global__ void gemv_warp(const float *__restrict__ W, const float *__restrict__ x,
                                     float *__restrict__ y, int K, int N) {
    gemv_m0_body(W, x, y, K, N);
}
// Reference: gemv.cu:51-71 (thread per row, float4).
extern "C" __global__ void gemv4(const float *__restrict__ W, const float *__restrict__ x, float *__restrict__ y,
                                 int K, int N) {
    gemv_m0_body(W, x, y, K, N);
}
