// sb_resid.cuh -- split-K projection with the residual add fused:
//   x[n] = x[n] + (sum_k W[n][k] v[k] (+ b[n]))
// for the short-and-wide decode projections (O: 896x896; down: 896x4864;
// GPT-2 proj: 768x3072).  With only ~900 rows, one warp per row leaves most
// of HBM's latency-bandwidth product unused, so each row is split over
// `ksplit` warps of one CTA (contiguous chunk slices), partials are reduced
// through shared memory in a fixed order, and one thread applies the
// residual.  v is read through L1 (no shared staging), so a CTA touches only
// its slice of v.
#pragma once
#include "sb_gemv.cuh"
#include "sb_finalize.cuh"

// F16: weights fp16 (flush-to-zero decode) else fp32.  bias may be null.
template <bool F16>
SB_DEV void resid_splitk_body(const void *__restrict__ W, const float *__restrict__ bias,
                              const float *__restrict__ v, SbStep *__restrict__ st, float *__restrict__ x, int K,
                              int N, int ksplit) {
    __shared__ float part[32];
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
    const int ngroups = nw / ksplit, grp = warp / ksplit, slice = warp % ksplit;
    const int E = F16 ? 8 : 4;
    const int cpr = K / E;
    const int cps = (cpr + ksplit - 1) / ksplit;
    const int cb = slice * cps, ce = min(cpr, cb + cps);
    int t0, t1;
    cta_task_range(N, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0) prefetch_rows(W, (long)K * (F16 ? 2 : 4), t0, t1, 512L << 10);
    pdl_wait();
    if (st && sb_step_idle(st)) return;
    const int iters = (t1 - t0 + ngroups - 1) / ngroups;
    for (int it = 0; it < iters; it++) {
        const int row = t0 + it * ngroups + grp;
        const int rows[1] = {(row < t1 && grp < ngroups) ? row : -1};
        float acc[1];
        if (F16) warp_dot_h_range<1, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cb, ce, XGlob8{v}, acc);
        else warp_dot_f_range<1, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cb, ce, XGlob4{v}, acc);
        if (lane == 0) part[warp] = acc[0];
        __syncthreads();
        if (threadIdx.x < ngroups) {
            const int r = t0 + it * ngroups + threadIdx.x;
            if (r < t1) {
                float s = 0.0f;
                for (int k = 0; k < ksplit; k++) s += part[threadIdx.x * ksplit + k];
                const float y = bias ? __fadd_rn(s, bias[r]) : s;
                x[r] = __fadd_rn(x[r], y);
            }
        }
        __syncthreads();
    }
}
