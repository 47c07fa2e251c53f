// sb_gemv.cuh -- the row-streaming GEMV core every decode matvec of this
// package is built from (FP16 or FP32 weights, FP32 activations, FP32
// accumulation).
//
// Layout: W is row-major [N][K] ("[out,in]", the reference's gemv layout,
// conv_qwen.py:12), so a run of rows is one contiguous byte range.  A warp
// owns a TASK of R rows; its lanes stride the row in 16-byte chunks (8 fp16
// or 4 fp32 weights), so every warp-wide load instruction moves 512
// contiguous bytes per row.  U chunk-iterations are unrolled and all R*U
// loads are issued before any arithmetic, which keeps R*U*16 bytes per lane
// in flight -- enough for HBM3e's latency-bandwidth product with 4-8 warps
// per SM.  Partial sums are combined with xor-shuffles (no shared memory, no
// block barriers, so any row/grid count is safe), after which every lane
// holds all R row sums and the epilogue functor runs on lane 0.
#pragma once
#include "sb_common.cuh"

// ---- weight formats: one 16-byte chunk -> 8 or 4 weights
struct WH {  // fp16 weights, reference flush-to-zero decode
    static constexpr int E = 8;
};
struct WF {  // fp32 weights
    static constexpr int E = 4;
};

// ---- activation accessors (x[c*E .. c*E+E-1] for chunk c)
// Shared-memory x for fp16 weights, split into two float4 planes so the two
// 16-byte reads of a chunk are bank-conflict free across a warp.
struct XSplit8 {
    const float4 *lo, *hi;
    SB_DEV void get8(int c, float4 &a, float4 &b) const { a = lo[c]; b = hi[c]; }
};
// Global (L1-cached) x, used by the geometry-agnostic drop-in kernels.
struct XGlob8 {
    const float *x;
    SB_DEV void get8(int c, float4 &a, float4 &b) const {
        a = ld_f4(x + 8 * c);
        b = ld_f4(x + 8 * c + 4);
    }
};
struct XSmem4 {
    const float4 *x;
    SB_DEV float4 get4(int c) const { return x[c]; }
};
struct XGlob4 {
    const float *x;
    SB_DEV float4 get4(int c) const { return ld_f4(x + 4 * c); }
};

SB_DEV float dot_chunk(WH, const uint4 &w, const float4 &a, const float4 &b, float acc) {
    float2 f0 = h2x2_ftz(w.x), f1 = h2x2_ftz(w.y), f2 = h2x2_ftz(w.z), f3 = h2x2_ftz(w.w);
    acc = fmaf(f0.x, a.x, acc);
    acc = fmaf(f0.y, a.y, acc);
    acc = fmaf(f1.x, a.z, acc);
    acc = fmaf(f1.y, a.w, acc);
    acc = fmaf(f2.x, b.x, acc);
    acc = fmaf(f2.y, b.y, acc);
    acc = fmaf(f3.x, b.z, acc);
    acc = fmaf(f3.y, b.w, acc);
    return acc;
}
// fp16 weights x fp16 activations, FP32 accumulation, with sm_100's
// mixed-precision FMA (fma.rn.f32.f16: the f16 x f16 product is exact and
// the sum is rounded once, so each step equals fmaf on the decoded values)
// -- no fp16 -> fp32 conversions, which bound the CUDA-core dot otherwise.
// The weight halves are flushed to zero first (mul.ftz by 1.0: subnormals
// -> 0, normals exact), the reference's h2f rule; x is staged pre-flushed.
SB_DEV float fma_hh(float acc, unsigned short a, unsigned short b) {
    asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(a), "h"(b));
    return acc;
}
SB_DEV unsigned ftz_h2(unsigned w) {
    unsigned r;
    asm("mul.rn.ftz.f16x2 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(0x3C003C00u));
    return r;
}
SB_DEV float dot_chunk_hh(const uint4 &w, const uint4 &x, float acc) {
    const unsigned ws[4] = {ftz_h2(w.x), ftz_h2(w.y), ftz_h2(w.z), ftz_h2(w.w)}, xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        acc = fma_hh(acc, (unsigned short)(ws[j] & 0xffffu), (unsigned short)(xs[j] & 0xffffu));
        acc = fma_hh(acc, (unsigned short)(ws[j] >> 16), (unsigned short)(xs[j] >> 16));
    }
    return acc;
}
SB_DEV float dot_chunk(WF, const uint4 &w, const float4 &a, float acc) {
    acc = fmaf(__uint_as_float(w.x), a.x, acc);
    acc = fmaf(__uint_as_float(w.y), a.y, acc);
    acc = fmaf(__uint_as_float(w.z), a.z, acc);
    acc = fmaf(__uint_as_float(w.w), a.w, acc);
    return acc;
}

// Dot products of R rows with x.  rows[r] < 0 skips that row; every row is
// `cpr` chunks long (cpr = K / E) with row stride `ld_chunks` chunks.  All
// R*U loads of an iteration are issued before any arithmetic.  Returns
// warp-reduced sums in acc[] (identical on every lane).
template <int R, int U, class XA>
SB_DEV void warp_dot_h_range(const uint4 *W, long ld_chunks, const int (&rows)[R], int cb, int ce, XA xa,
                       float (&acc)[R], bool reduce = true) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.0f;
    for (int c0 = cb + lane; c0 < ce; c0 += 32 * U) {
        uint4 w[U][R];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (c < ce && rows[r] >= 0) w[u][r] = ld_stream_u4(W + (long)rows[r] * ld_chunks + c);
                else w[u][r] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
            if (c < ce) {
                float4 a, b;
                xa.get8(c, a, b);
#pragma unroll
                for (int r = 0; r < R; r++) acc[r] = dot_chunk(WH(), w[u][r], a, b, acc[r]);
            }
        }
    }
    if (reduce) {
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = warp_sum(acc[r]);
    }
}

template <int R, int U, class XA>
SB_DEV void warp_dot_f_range(const uint4 *W, long ld_chunks, const int (&rows)[R], int cb, int ce, XA xa,
                       float (&acc)[R], bool reduce = true) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.0f;
    for (int c0 = cb + lane; c0 < ce; c0 += 32 * U) {
        uint4 w[U][R];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (c < ce && rows[r] >= 0) w[u][r] = ld_stream_u4(W + (long)rows[r] * ld_chunks + c);
                else w[u][r] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
            if (c < ce) {
                float4 a = xa.get4(c);
#pragma unroll
                for (int r = 0; r < R; r++) acc[r] = dot_chunk(WF(), w[u][r], a, acc[r]);
            }
        }
    }
    if (reduce) {
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = warp_sum(acc[r]);
    }
}

// Whole-row forms.
template <int R, int U, class XA>
SB_DEV void warp_dot_h(const uint4 *W, long ld_chunks, const int (&rows)[R], int cpr, XA xa, float (&acc)[R]) {
    warp_dot_h_range<R, U>(W, ld_chunks, rows, 0, cpr, xa, acc);
}
template <int R, int U, class XA>
SB_DEV void warp_dot_f(const uint4 *W, long ld_chunks, const int (&rows)[R], int cpr, XA xa, float (&acc)[R]) {
    warp_dot_f_range<R, U>(W, ld_chunks, rows, 0, cpr, xa, acc);
}

// R consecutive rows from n0, rows >= nlim skipped.
template <int R>
SB_DEV void consecutive_rows(int n0, int nlim, int (&rows)[R]) {
#pragma unroll
    for (int r = 0; r < R; r++) rows[r] = (n0 + r < nlim) ? n0 + r : -1;
}

// Bulk-prefetch rows [r0, r1) of a row-major matrix with `row_bytes` per row
// (capped at `cap` bytes) into L2.
SB_DEV void prefetch_rows(const void *W, long row_bytes, long r0, long r1, long cap) {
    if (r1 <= r0) return;
    long bytes = (r1 - r0) * row_bytes;
    if (bytes > cap) bytes = cap;
    l2_prefetch_bulk((const char *)W + r0 * row_bytes, (uint32_t)(bytes & ~15L));
}

// Contiguous task range of this CTA (tasks split evenly over the grid);
// warps stride inside it.
SB_DEV void cta_task_range(int ntasks, int &t0, int &t1) {
    const int per = (ntasks + gridDim.x - 1) / gridDim.x;
    t0 = blockIdx.x * per;
    t1 = min(ntasks, t0 + per);
}

// Stage x (length K, K % 8 == 0) into the split shared layout, optionally
// scaled elementwise: xs = x * scale * g[i] (g fp16 decoded with FTZ), the
// RMSNorm prologue; pass g == nullptr for a plain copy.
SB_DEV void stage_x_split8(const float *x, int K, float4 *lo, float4 *hi, float scale,
                           const uint16_t *g) {
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
        float4 a = ld_f4(x + 8 * c), b = ld_f4(x + 8 * c + 4);
        if (g) {
            // y = x * inv * h2f(w): two roundings in the reference order
            const uint16_t *gg = g + 8 * c;
            a.x = __fmul_rn(__fmul_rn(a.x, scale), h2f_ftz(gg[0]));
            a.y = __fmul_rn(__fmul_rn(a.y, scale), h2f_ftz(gg[1]));
            a.z = __fmul_rn(__fmul_rn(a.z, scale), h2f_ftz(gg[2]));
            a.w = __fmul_rn(__fmul_rn(a.w, scale), h2f_ftz(gg[3]));
            b.x = __fmul_rn(__fmul_rn(b.x, scale), h2f_ftz(gg[4]));
            b.y = __fmul_rn(__fmul_rn(b.y, scale), h2f_ftz(gg[5]));
            b.z = __fmul_rn(__fmul_rn(b.z, scale), h2f_ftz(gg[6]));
            b.w = __fmul_rn(__fmul_rn(b.w, scale), h2f_ftz(gg[7]));
        }
        lo[c] = a;
        hi[c] = b;
    }
}

// RMSNorm scale 1/sqrt(mean(x^2)+eps) computed by the whole block (every
// thread receives it).  Same formula as cpu_rms (qwen_engine.c:285-290).
SB_DEV float block_rms_scale(const float *x, int n, float eps, float *red) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(x[i], x[i], s);
    s = block_sum(s, red);
    return 1.0f / sqrtf(__fdiv_rn(s, (float)n) + eps);
}

// Batched variant for B activation vectors (FP16 weights): x planes for
// batch b start at lo + b*(K/8), hi + b*(K/8).  acc[r][b].
// R rows x B fp16 activation rows (x: B * cpr flushed 16-byte chunks in
// shared memory), mixed-precision FMAs; warp-reduced sums in acc[][].
template <int R, int U, int B>
SB_DEV void warp_dot_hh(const uint4 *W, long ld_chunks, const int (&rows)[R], int cpr, const uint4 *xh,
                        float (&acc)[R][B]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < B; b++) acc[r][b] = 0.0f;
    for (int c0 = lane; c0 < cpr; c0 += 32 * U) {
        uint4 w[U][R];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (c < cpr && rows[r] >= 0) w[u][r] = ld_stream_u4(W + (long)rows[r] * ld_chunks + c);
                else w[u][r] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
            if (c < cpr) {
#pragma unroll
                for (int b = 0; b < B; b++) {
                    const uint4 x = xh[b * cpr + c];
#pragma unroll
                    for (int r = 0; r < R; r++) acc[r][b] = dot_chunk_hh(w[u][r], x, acc[r][b]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < B; b++) acc[r][b] = warp_sum(acc[r][b]);
}

template <int R, int U, int B>
SB_DEV void warp_dot_hb(const uint4 *W, long ld_chunks, const int (&rows)[R], int cpr, const float4 *lo,
                        const float4 *hi, float (&acc)[R][B]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < B; b++) acc[r][b] = 0.0f;
    for (int c0 = lane; c0 < cpr; c0 += 32 * U) {
        uint4 w[U][R];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (c < cpr && rows[r] >= 0) w[u][r] = ld_stream_u4(W + (long)rows[r] * ld_chunks + c);
                else w[u][r] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
            if (c < cpr) {
#pragma unroll
                for (int b = 0; b < B; b++) {
                    const float4 a = lo[b * cpr + c], bb = hi[b * cpr + c];
#pragma unroll
                    for (int r = 0; r < R; r++) acc[r][b] = dot_chunk(WH(), w[u][r], a, bb, acc[r][b]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < B; b++) acc[r][b] = warp_sum(acc[r][b]);
}

// Split-K task loop for short outputs (fewer four-row tasks than two per
// SM, where a warp per task would leave most SMs idle): one CTA per task;
// its 8 warps (block 256) take contiguous eighths of the row's `cpr` chunks,
// `dot(rows, cb, ce, acc)` leaves each warp's reduced partials in acc, and
// the partials are added in warp order in shared memory.  y[row] = sum
// (+ bias[row]).
template <class Dot>
SB_DEV void splitk_rows4(int N, int cpr, const float *bias, float *y, Dot dot) {
    constexpr int R = 4, NW = 8;
    __shared__ float part[NW][R];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (cpr + NW - 1) / NW;
    const int cb = min(cpr, warp * per), ce = min(cpr, cb + per);
    for (int t = blockIdx.x; t < (N + R - 1) / R; t += gridDim.x) {
        int rows[R];
        consecutive_rows<R>(t * R, N, rows);
        float acc[R];
        dot(rows, cb, ce, acc);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; r++) part[warp][r] = acc[r];
        }
        __syncthreads();
        if (threadIdx.x < R) {
            const int row = t * R + threadIdx.x;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) s += part[w][threadIdx.x];
            if (row < N) y[row] = s + (bias ? bias[row] : 0.0f);
        }
        __syncthreads();  // part is reused by the CTA's next task
    }
}
