// qwen_kernels.cu -- the "qwen" module image (sm_100a cubin).
//
// Part 1: drop-in kernels with the reference's exact names and parameter
// lists (gpu-llm/kernels/qwen_kernels.cu), correct under the launch geometry
// the reference host hard-codes (qwen_engine.c:216-265) or any other.
// Part 2: fused decode-step kernels used by this package's engine; they take
// the step position from device memory so one captured CUDA graph replays
// every token, and they use programmatic dependent launch so each kernel's
// weight prefetch overlaps its predecessor's tail.
#include "sb_attn.cuh"
#include "sb_gemv.cuh"

// =====================================================================
// Part 1 -- drop-ins
// =====================================================================

// y[n] = sum_k h2f(W[n*K+k]) * x[k] (+ bias[n]).  Reference:
// qwen_kernels.cu:34-70 (grid ceil(N/8), block 256).  Warp-per-row-task,
// grid-stride over all warps, so any grid works; fp16 flush-to-zero decode.
extern "C" __global__ void gemv_h(const unsigned short *__restrict__ W, const float *__restrict__ x,
                                  const float *__restrict__ bias, float *__restrict__ y, int K, int N) {
    const int nthreads = gridDim.x * blockDim.x;
    const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec = ((K & 7) == 0) && ((((uintptr_t)W) & 15) == 0) && ((((uintptr_t)x) & 15) == 0);
    if (vec && (blockDim.x & 31) == 0) {
        const int warp = gtid >> 5, nwarp = nthreads >> 5;
        const int cpr = K >> 3;
        XGlob8 xa{x};
        for (int n = warp; n < N; n += nwarp) {
            float acc[1];
            const int rows[1] = {n};
            warp_dot_h<1, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cpr, xa, acc);
            if ((threadIdx.x & 31) == 0) y[n] = acc[0] + (bias ? bias[n] : 0.0f);
        }
        return;
    }
    // K % 8 != 0 (the reference only needs K % 4 == 0) or odd block shape:
    // one thread per row, still exact fp16 decode.
    for (int n = gtid; n < N; n += nthreads) {
        const unsigned short *row = W + (size_t)n * K;
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc = fmaf(h2f_ftz(row[k]), x[k], acc);
        y[n] = acc + (bias ? bias[n] : 0.0f);
    }
}

// y = x * rsqrt(mean(x^2) + eps) * h2f(w); one block per row (grid = T).
// Reference: qwen_kernels.cu:74-93.
extern "C" __global__ void rmsnorm(const float *__restrict__ x, const unsigned short *__restrict__ w,
                                   float *__restrict__ y, int n, float eps) {
    __shared__ float red[32];
    x += (size_t)blockIdx.x * n;
    y += (size_t)blockIdx.x * n;
    const float inv = block_rms_scale(x, n, eps, red);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], inv), h2f_ftz(w[i]));
}

// Half-split RoPE from cos/sin tables; one thread per (t, head, pair).
// Reference: qwen_kernels.cu:97-116.  Products and the difference are
// rounded separately, as the reference's C computes them.
extern "C" __global__ void rope(float *__restrict__ x, const float *__restrict__ cosT,
                                const float *__restrict__ sinT, int T, int H, int HD, int pos0) {
    const int hd2 = HD / 2;
    const long total = (long)T * H * hd2;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total;
         idx += (long)gridDim.x * blockDim.x) {
        const int t = (int)(idx / (H * hd2));
        const int r = (int)(idx % (H * hd2));
        const int h = r / hd2, i = r % hd2;
        float *row = x + (size_t)t * H * HD;
        const float a = row[h * HD + i], b = row[h * HD + hd2 + i];
        const float c = cosT[(size_t)(pos0 + t) * hd2 + i], s = sinT[(size_t)(pos0 + t) * hd2 + i];
        row[h * HD + i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        row[h * HD + hd2 + i] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
}

SB_DEV float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// y = silu(g) * u.  Reference: qwen_kernels.cu:119-126.
extern "C" __global__ void swiglu(const float *__restrict__ g, const float *__restrict__ u,
                                  float *__restrict__ y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = silu_mul(g[i], u[i]);
}

// scores[t*NH+h] = scale * q_h . kc[t*KV + g*HD ..], g = h / (NH/(KV/HD)).
// Reference: qwen_kernels.cu:130-144 (one thread per (t, h)).
extern "C" __global__ void attn_scores_gqa(const float *__restrict__ q, const float *__restrict__ kc,
                                           float *__restrict__ scores, int T, float scale, int NH,
                                           int KV, int HD) {
    const int grp = NH / (KV / HD);
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < T * NH; idx += gridDim.x * blockDim.x) {
        const int t = idx / NH, h = idx % NH, g = h / grp;
        const float *qp = q + h * HD;
        const float *kp = kc + (size_t)t * KV + g * HD;
        float acc = 0.0f;
        for (int d = 0; d < HD; d++) acc = fmaf(qp[d], kp[d], acc);
        scores[idx] = acc * scale;
    }
}

// Per-head softmax over T (the stock host launches NH threads).
// Reference: qwen_kernels.cu:147-164.
extern "C" __global__ void attn_softmax(const float *__restrict__ scores, float *__restrict__ probs,
                                        int T, int NH) {
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < NH; h += gridDim.x * blockDim.x) {
        float maxv = -1e30f;
        for (int t = 0; t < T; t++) maxv = fmaxf(maxv, scores[(size_t)t * NH + h]);
        float sum = 0.0f;
        for (int t = 0; t < T; t++) {
            float e = expf(scores[(size_t)t * NH + h] - maxv);
            probs[(size_t)t * NH + h] = e;
            sum += e;
        }
        const float inv = 1.0f / sum;
        for (int t = 0; t < T; t++) probs[(size_t)t * NH + h] *= inv;
    }
}

// out[h*HD+d] = sum_t probs[t*NH+h] * vc[t*KV + g*HD + d].
// Reference: qwen_kernels.cu:167-180.
extern "C" __global__ void attn_mix_gqa(const float *__restrict__ probs, const float *__restrict__ vc,
                                        float *__restrict__ out, int T, int NH, int KV, int HD) {
    const int grp = NH / (KV / HD);
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < NH * HD; idx += gridDim.x * blockDim.x) {
        const int h = idx / HD, d = idx % HD, g = h / grp;
        float acc = 0.0f;
        for (int t = 0; t < T; t++) acc = fmaf(probs[(size_t)t * NH + h], vc[(size_t)t * KV + g * HD + d], acc);
        out[idx] = acc;
    }
}

// out = a + b.  Reference: qwen_kernels.cu:183-189.
extern "C" __global__ void add2(const float *__restrict__ a, const float *__restrict__ b,
                                float *__restrict__ out, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
}

// =====================================================================
// Part 1b -- this package's standalone entry kernels (tuned geometry)
// =====================================================================

// y = W x (+bias) with x staged once per CTA in shared memory and 4-row
// warp tasks; a contiguous row range per CTA.  Launched by sb_gemv_h with
// grid ~ 4 CTAs/SM, block 256, dynamic smem K*4.  K % 8 == 0.
extern "C" __global__ void __launch_bounds__(256) gemv_h_b200(const unsigned short *__restrict__ W,
                                                              const float *__restrict__ x,
                                                              const float *__restrict__ bias,
                                                              float *__restrict__ y, int K, int N) {
    extern __shared__ float4 xs4[];
    constexpr int R = 4;
    int t0, t1;
    cta_task_range((N + R - 1) / R, t0, t1);
    float4 *lo = xs4, *hi = xs4 + K / 8;
    stage_x_split8(x, K, lo, hi, 1.0f, nullptr);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = K / 8, lane = threadIdx.x & 31;
    XSplit8 xa{lo, hi};
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, N, rows);
        float acc[R];
        warp_dot_h<R, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cpr, xa, acc);
#pragma unroll
        for (int r = 0; r < R; r++)
            if (lane == r && rows[r] >= 0) y[rows[r]] = acc[r] + (bias ? bias[rows[r]] : 0.0f);
    }
}

// gemv_h_b200 for short outputs: split-K over a CTA's warps (splitk_rows4),
// x read through L1.  Block 256, no dynamic shared memory, K % 8 == 0.
extern "C" __global__ void __launch_bounds__(256) gemv_h_sk(const unsigned short *__restrict__ W,
                                                            const float *__restrict__ x,
                                                            const float *__restrict__ bias,
                                                            float *__restrict__ y, int K, int N) {
    const uint4 *W4 = reinterpret_cast<const uint4 *>(W);
    const int cpr = K / 8;
    const XGlob8 xa{x};
    splitk_rows4(N, cpr, bias, y, [&](const int (&rows)[4], int cb, int ce, float (&acc)[4]) {
        warp_dot_h_range<4, 4>(W4, cpr, rows, cb, ce, xa, acc);
    });
}

// Y[b][n] = sum_k h2f(W[n][k]) h2f(X[b][k]) for B activation rows (fp16,
// decoded with the same flush-to-zero rule), FP32 out, on sm_100's
// mixed-precision FMA (each step equal to fmaf on the decoded values, in the
// same order).  dynamic smem >= B*K*2.  K % 8 == 0.
template <int B>
__device__ void gemv_hh_body(const unsigned short *__restrict__ W, const unsigned short *__restrict__ X,
                             float *__restrict__ Y, int K, int N) {
    extern __shared__ uint4 xhb[];
    constexpr int R = 4;
    int t0, t1;
    cta_task_range((N + R - 1) / R, t0, t1);
    const int cpr = K / 8;
    for (int i = threadIdx.x; i < B * cpr; i += blockDim.x) {
        const uint4 v = *reinterpret_cast<const uint4 *>(X + (size_t)i * 8);
        xhb[i] = make_uint4(ftz_half2_bits(v.x), ftz_half2_bits(v.y), ftz_half2_bits(v.z), ftz_half2_bits(v.w));
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, N, rows);
        float acc[R][B];
        warp_dot_hh<R, (B > 2 ? 2 : 4), B>(reinterpret_cast<const uint4 *>(W), cpr, rows, cpr, xhb, acc);
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int b = 0; b < B; b++)
                if (lane == r * B + b && rows[r] >= 0) Y[(size_t)b * N + rows[r]] = acc[r][b];
    }
}
extern "C" __global__ void __launch_bounds__(256) gemv_hh1(const unsigned short *W, const unsigned short *X,
                                                           float *Y, int K, int N) {
    gemv_hh_body<1>(W, X, Y, K, N);
}
extern "C" __global__ void __launch_bounds__(256) gemv_hh2(const unsigned short *W, const unsigned short *X,
                                                           float *Y, int K, int N) {
    gemv_hh_body<2>(W, X, Y, K, N);
}
extern "C" __global__ void __launch_bounds__(256) gemv_hh4(const unsigned short *W, const unsigned short *X,
                                                           float *Y, int K, int N) {
    gemv_hh_body<4>(W, X, Y, K, N);
}

// The same product for short outputs (N = 896 gives 224 four-row tasks:
// a warp per task would leave most SMs idle with a few KB in flight each).
// One CTA per four-row task; its 8 warps take contiguous eighths of K, so
// a CTA keeps 8 warps x 16 row-chunks of 16 B in flight.  x is read from
// global memory (L1-cached, shared by the CTAs of an SM) and flushed per
// use, so there is no staging round trip.  Warp partials are added in
// warp order in shared memory.  Block 256.
template <int B>
__device__ void gemv_hh_sk_body(const unsigned short *__restrict__ W, const unsigned short *__restrict__ X,
                                float *__restrict__ Y, int K, int N) {
    constexpr int R = 4, NW = 8, U = 4;
    __shared__ float part[NW][R * B];
    const int cpr = K / 8, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (cpr + NW - 1) / NW;
    const int c_lo = min(cpr, warp * per), c_hi = min(cpr, c_lo + per);
    const uint4 *W4 = reinterpret_cast<const uint4 *>(W);
    const uint4 *X4 = reinterpret_cast<const uint4 *>(X);
    for (int t = blockIdx.x; t < (N + R - 1) / R; t += gridDim.x) {
        int rows[R];
        consecutive_rows<R>(t * R, N, rows);
        float acc[R][B];
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int b = 0; b < B; b++) acc[r][b] = 0.0f;
        for (int c0 = c_lo + lane; c0 < c_hi; c0 += 32 * U) {
            uint4 w[U][R];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = c0 + 32 * u;
#pragma unroll
                for (int r = 0; r < R; r++)
                    w[u][r] = (c < c_hi && rows[r] >= 0) ? ld_stream_u4(W4 + (long)rows[r] * cpr + c)
                                                          : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = c0 + 32 * u;
                if (c < c_hi) {
#pragma unroll
                    for (int b = 0; b < B; b++) {
                        const uint4 v = __ldg(X4 + (long)b * cpr + c);
                        const uint4 x = make_uint4(ftz_half2_bits(v.x), ftz_half2_bits(v.y), ftz_half2_bits(v.z),
                                                   ftz_half2_bits(v.w));
#pragma unroll
                        for (int r = 0; r < R; r++) acc[r][b] = dot_chunk_hh(w[u][r], x, acc[r][b]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int b = 0; b < B; b++) {
                const float v = warp_sum(acc[r][b]);
                if (lane == 0) part[warp][r * B + b] = v;
            }
        __syncthreads();
        if (threadIdx.x < R * B) {
            const int r = threadIdx.x / B, b = threadIdx.x % B;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) s += part[w][threadIdx.x];
            if (t * R + r < N) Y[(size_t)b * N + t * R + r] = s;
        }
        __syncthreads();  // part is reused by the CTA's next task
    }
}
extern "C" __global__ void __launch_bounds__(256) gemv_hh_sk1(const unsigned short *W, const unsigned short *X,
                                                              float *Y, int K, int N) {
    gemv_hh_sk_body<1>(W, X, Y, K, N);
}
extern "C" __global__ void __launch_bounds__(256) gemv_hh_sk2(const unsigned short *W, const unsigned short *X,
                                                              float *Y, int K, int N) {
    gemv_hh_sk_body<2>(W, X, Y, K, N);
}
extern "C" __global__ void __launch_bounds__(256) gemv_hh_sk4(const unsigned short *W, const unsigned short *X,
                                                              float *Y, int K, int N) {
    gemv_hh_sk_body<4>(W, X, Y, K, N);
}

// sb_gemm_hh's small batches (B <= 16) on short outputs (fewer than ~300
// row tiles), in ONE launch: the tcgen05 kernel needs split-K there, with a
// second launch to add the partials, and the CUDA-core dot needs B fma per
// weight.  One CTA per 8 rows of W; its 16 warps take contiguous sixteenths
// of K and add their partial tiles in warp order in shared memory
// (deterministic).  The products run on mma.sync m16n8k16 (fp16 in, FP32
// accumulation; fp16 subnormals kept, as the tensor pipe of gemm_hh_tc):
// A = 16 activation rows (zero beyond B), B = 8 weight rows (zero beyond N).
// Per 32-element K block, lane (g, q) holds elements 8q .. 8q+7 of its
// rows: the first four in the block's first MMA's fragment slots, the last
// four in the second's -- the same order for both operands, so every
// weight still meets its own activation -- and loads them as one 16-byte
// chunk (W streamed past L1, X through L1).  A warp issues the loads of up
// to U blocks before their MMAs: a CTA keeps its whole slice of W in flight
// for K up to NW x U x 32.  WIDE: B > 8 (rows g + 8 of A).  NW = 16 for
// fewer tiles than SMs can hold twice; NW = 4 (four CTAs per SM) for more.
// grid ceil(N/8); block 32 NW.  K % 8 == 0.
template <bool WIDE, int NW>
__device__ void gemm_hh_mma_body(const unsigned short *__restrict__ W, const unsigned short *__restrict__ X,
                                 float *__restrict__ Y, int K, int N, int B) {
    constexpr int U = WIDE ? 8 : 10;
    __shared__ float red[NW][32][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int n0 = blockIdx.x * 8, nblk = (K + 31) / 32;
    const int blk0 = nblk * warp / NW, blk1 = nblk * (warp + 1) / NW;
    const bool wrow = n0 + g < N, xr0 = g < B, xr1 = WIDE && g + 8 < B;
    const uint4 *wp = reinterpret_cast<const uint4 *>(W + (long)(n0 + g) * K) + q;
    const uint4 *x0p = reinterpret_cast<const uint4 *>(X + (long)g * K) + q;
    const uint4 *x1p = reinterpret_cast<const uint4 *>(X + (long)(g + 8) * K) + q;
    const int kc = K / 8;  // 16-byte chunks per row
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int b = blk0; b < blk1; b += U) {
        uint4 w[U], a[U], c[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int ch = (b + u) * 4;  // this lane's chunk: ch + q
            const bool ok = b + u < blk1 && ch + q < kc;
            w[u] = ok && wrow ? ld_stream_u4(wp + ch) : make_uint4(0u, 0u, 0u, 0u);
            a[u] = ok && xr0 ? __ldg(x0p + ch) : make_uint4(0u, 0u, 0u, 0u);
            c[u] = ok && xr1 ? __ldg(x1p + ch) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (b + u >= blk1) break;
            float(&d)[4] = (u & 1) ? d1 : d0;
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                "{%0, %1, %2, %3};"
                : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                : "r"(a[u].x), "r"(c[u].x), "r"(a[u].y), "r"(c[u].y), "r"(w[u].x), "r"(w[u].y));
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                "{%0, %1, %2, %3};"
                : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                : "r"(a[u].z), "r"(c[u].z), "r"(a[u].w), "r"(c[u].w), "r"(w[u].z), "r"(w[u].w));
        }
    }
    // D[b][n]: lane (g, q) holds (b = g, n = 2q, 2q+1) and (b = g + 8, same n)
#pragma unroll
    for (int i = 0; i < 4; i++) red[warp][lane][i] = d0[i] + d1[i];
    __syncthreads();
    if (threadIdx.x < 128) {
        const int l = threadIdx.x >> 2, i = threadIdx.x & 3;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < NW; w++) s += red[w][l][i];
        const int b = (l >> 2) + ((i >> 1) << 3), n = n0 + 2 * (l & 3) + (i & 1);
        if (b < B && n < N) Y[(long)b * N + n] = s;
    }
}
extern "C" __global__ void __launch_bounds__(512) gemm_hh_mma8(const unsigned short *W, const unsigned short *X,
                                                               float *Y, int K, int N, int B) {
    gemm_hh_mma_body<false, 16>(W, X, Y, K, N, B);
}
extern "C" __global__ void __launch_bounds__(512) gemm_hh_mma16(const unsigned short *W, const unsigned short *X,
                                                                float *Y, int K, int N, int B) {
    gemm_hh_mma_body<true, 16>(W, X, Y, K, N, B);
}
extern "C" __global__ void __launch_bounds__(128, 4)
    gemm_hh_mma8_w4(const unsigned short *W, const unsigned short *X, float *Y, int K, int N, int B) {
    gemm_hh_mma_body<false, 4>(W, X, Y, K, N, B);
}
extern "C" __global__ void __launch_bounds__(128, 4)
    gemm_hh_mma16_w4(const unsigned short *W, const unsigned short *X, float *Y, int K, int N, int B) {
    gemm_hh_mma_body<true, 4>(W, X, Y, K, N, B);
}

// ---- next-token candidates for the Qwen sampler (qwen_engine.c:375-390):
// the reference penalises each context id's logit once per occurrence
// (divide when positive, else multiply), divides every logit by the
// temperature, then takes k passes of first-index argmax.  The k winners
// are the first k of all w[i] ordered by (value descending, index
// ascending), so here each CTA takes the first k of its 1024 ids and one
// CTA merges them.  The same IEEE operations in the same order give the
// same w[i] bit for bit; the softmax / top-p / draw over the k values stays
// on the host (20 values instead of the 608 KB logits vector).
//
// No sorting network: every step ranks a small candidate set.  A candidate
// is a 64-bit key -- the value's bits mapped to an order-preserving
// unsigned (-0 taken as +0: the reference's comparisons treat them as
// equal) above an id rank that is larger for a smaller id -- so keys are
// distinct and a larger key is a better candidate; 0 = empty.  The first k
// of a set S are the keys whose rank (the number of larger keys in S) is
// below k.  A lower bound T of the k-th best key shrinks S first: the k-th
// best of per-thread (or per-list) maxima is one, since k holders each
// have a key at least that good; then at most 4k keys (k lists x k in the
// merge) reach T.  (Bitonic networks -- block-wide or in one warp's
// registers -- took 13 and 18 us: latency chains on one SM.)
constexpr int TK_CHUNK = 1024;
SB_DEV unsigned tk_ord(float v) {
    const unsigned u = __float_as_uint(v == 0.f ? 0.f : v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// key of (value, id) with `low` (< 2^14) in the lowest bits; ids < 2^18
SB_DEV unsigned long long tk_key(float v, int id, int low) {
    return ((unsigned long long)tk_ord(v) << 32) | ((unsigned)(0x3FFFF - id) << 14) | (unsigned)low;
}
// the first k of the n keys in s (all distinct on bits 14 and up, since
// they differ in value or id): out(rank, key) for each key whose rank < k
template <typename F>
SB_DEV void tk_rank(const unsigned long long *s, int n, int k, F out) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long me = s[i] >> 14;
        int r = 0;
        for (int j = 0; j < n; j++) r += (s[j] >> 14) > me;
        if (r < k) out(r, s[i]);
    }
}
// one shared atomic per warp: returns this lane's slot (or -1) for `keep`
SB_DEV int tk_append(bool keep, int *count) {
    const int lane = threadIdx.x & 31;
    const unsigned ball = __ballot_sync(SB_FULL, keep);
    int base = 0;
    if (lane == 0 && ball) base = atomicAdd(count, __popc(ball));
    base = __shfl_sync(SB_FULL, base, 0);
    return keep ? base + __popc(ball & ((1u << lane) - 1u)) : -1;
}
// grid ceil(V / 1024), block 256: CTA b's first k of ids [1024 b, 1024 b +
// 1024) -> cand_*[b * k ..] in order; empty slots get id -1.  k <= 64.
extern "C" __global__ void __launch_bounds__(256) topk_partial(const float *__restrict__ logits, int V,
                                                               const int *__restrict__ ctx, int ctx_len,
                                                               float temperature, float rep_penalty, int k,
                                                               int *__restrict__ cand_i, float *__restrict__ cand_v) {
    __shared__ int cnt[TK_CHUNK];
    __shared__ float w[TK_CHUNK];
    __shared__ unsigned long long tmax[256], surv[4 * 64];
    __shared__ unsigned long long thr;
    __shared__ int nsurv;
    const int i0 = blockIdx.x * TK_CHUNK, n = min(TK_CHUNK, V - i0);
    float lg[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {  // issued before the context scan
        const int j = threadIdx.x + 256 * r;
        lg[r] = j < n ? logits[i0 + j] : 0.f;
    }
    for (int j = threadIdx.x; j < TK_CHUNK; j += blockDim.x) cnt[j] = 0;
    if (threadIdx.x == 0) {
        thr = 0ull;
        nsurv = 0;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < ctx_len; p += blockDim.x) {
        const int t = ctx[p];
        if (t >= i0 && t < i0 + n) atomicAdd(&cnt[t - i0], 1);
    }
    __syncthreads();
    unsigned long long key[4], mx = 0ull;
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int j = threadIdx.x + 256 * r;
        key[r] = 0ull;
        if (j < n) {
            float v = lg[r];
            for (int c = cnt[j]; c > 0; c--) v = v > 0.f ? __fdiv_rn(v, rep_penalty) : __fmul_rn(v, rep_penalty);
            v = __fdiv_rn(v, temperature);
            w[j] = v;
            key[r] = tk_key(v, i0 + j, j);
            mx = key[r] > mx ? key[r] : mx;
        }
    }
    tmax[threadIdx.x] = mx;
    __syncthreads();
    if (mx) {  // T = the k-th best thread maximum
        int r = 0;
        for (int t = 0; t < 256; t++) r += tmax[t] > mx;
        if (r == k - 1) thr = mx;
    }
    __syncthreads();
    const unsigned long long T = thr;
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int pos = tk_append(key[r] && key[r] >= T, &nsurv);
        if (pos >= 0) surv[pos] = key[r];
    }
    __syncthreads();
    const int ns = nsurv;  // <= 4 k: only threads whose maximum reached T hold survivors
    int *ci = cand_i + (size_t)blockIdx.x * k;
    float *cv = cand_v + (size_t)blockIdx.x * k;
    tk_rank(surv, ns, k, [&](int r, unsigned long long kk) {
        const int j = (int)(kk & 0x3FFFu);
        ci[r] = i0 + j;
        cv[r] = w[j];
    });
    for (int r = ns + threadIdx.x; r < k; r += blockDim.x) {
        ci[r] = -1;
        cv[r] = 0.f;
    }
}
// one CTA of 1024 threads: the first k of the ncand (<= 16384) partial
// candidates (ids < 2^18; G = ncand / k <= 256 lists of k, each in order)
// -> out_*[0 .. k).  Every candidate is loaded once, all loads issued
// together.  T = the larger of two lower bounds of the k-th best key: the
// k-th best of the G lists' first keys, and each list's k-th key; at most
// k lists have a first key >= T, so at most k * k candidates are ranked.
extern "C" __global__ void __launch_bounds__(1024) topk_merge(const int *__restrict__ cand_i,
                                                              const float *__restrict__ cand_v, int ncand, int k,
                                                              int *__restrict__ out_i, float *__restrict__ out_v) {
    __shared__ unsigned long long surv[4096], first[256];
    __shared__ unsigned long long thr;
    __shared__ int nsurv;
    const int G = ncand / k, lane = threadIdx.x & 31;
    constexpr int PER = 16;  // candidates per thread (ncand <= 16384)
    unsigned long long key[PER];
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int j = threadIdx.x + 1024 * u;
        const int id = j < ncand ? cand_i[j] : -1;
        const float v = j < ncand ? cand_v[j] : 0.f;
        key[u] = id >= 0 ? tk_key(v, id, j) : 0ull;
    }
    if (threadIdx.x == 0) {
        thr = 0ull;
        nsurv = 0;
    }
    if (threadIdx.x < 256) first[threadIdx.x] = 0ull;
    __syncthreads();
    unsigned long long kth = 0ull;
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int j = threadIdx.x + 1024 * u;
        if (!key[u]) continue;
        if (j % k == k - 1 && key[u] > kth) kth = key[u];  // a list's k-th key
        if (j % k == 0) first[j / k] = key[u];            // a list's first key
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ob = __shfl_xor_sync(SB_FULL, kth, o);
        kth = ob > kth ? ob : kth;
    }
    if (lane == 0 && kth) atomicMax(&thr, kth);
    __syncthreads();
    if (threadIdx.x < G && G >= k && first[threadIdx.x]) {  // the k-th best list maximum
        const unsigned long long me = first[threadIdx.x];
        int r = 0;
        for (int c = 0; c < G; c++) r += first[c] > me;
        if (r == k - 1) atomicMax(&thr, me);
    }
    __syncthreads();
    const unsigned long long T = thr >> 14;
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int pos = tk_append(key[u] && (key[u] >> 14) >= T, &nsurv);
        if (pos >= 0 && pos < 4096) surv[pos] = key[u];
    }
    __syncthreads();
    const int ns = min(nsurv, 4096);  // <= k * k
    tk_rank(surv, ns, k, [&](int r, unsigned long long kk) {
        const int j = (int)(kk & 0x3FFFu);
        out_i[r] = cand_i[j];
        out_v[r] = cand_v[j];
    });
    for (int r = ns + threadIdx.x; r < k; r += blockDim.x) {
        out_i[r] = -1;
        out_v[r] = 0.f;
    }
}

// GQA decode attention with an explicit T (no step state); 7 query heads
// per KV head.  grid (NKV, max_splits), block SB_ATTN_THREADS.
extern "C" __global__ void attn_decode_g7(const float *__restrict__ q, const float *__restrict__ kc,
                                          const float *__restrict__ vc, int T, float *__restrict__ out,
                                          float *__restrict__ part, unsigned *__restrict__ counters,
                                          int kv_stride, float scale, int max_splits) {
    attn_decode_body<7>(q, kc, vc, T, out, part, counters, kv_stride, scale, max_splits);
}

// =====================================================================
// Part 2 -- fused decode-step kernels (this package's engine)
// =====================================================================
#include "sb_step.h"
#include "sb_finalize.cuh"
#include "sb_resid.cuh"

// x = h2f(emb[tokens[pos]]): the embedding gather the reference does on the
// host each token (qwen_engine.c:207-211).
extern "C" __global__ void qwen_embed(const unsigned short *__restrict__ emb, const int *__restrict__ tokens,
                                      SbStep *__restrict__ st, float *__restrict__ x, int C) {
    pdl_launch_dependents();
    pdl_wait();
    if (sb_step_idle(st)) return;
    const int tok = tokens[st->pos];
    const unsigned short *row = emb + (size_t)tok * C;
    for (int i = threadIdx.x; i < C; i += blockDim.x) x[i] = h2f_ftz(row[i]);
}

// RMSNorm(x) -> QKV GEMV (+bias) -> RoPE(q, k) -> q out, k/v straight into
// the KV cache at `pos`.  Replaces rmsnorm + gemv_h + 2x rope + 2 DtoD copies
// of qwen_engine.c:216-230.  A warp owns the RoPE pair rows (i, i+HD/2) of
// one head, so the rotation happens in its epilogue.
// grid: any; block: multiple of 32; dynamic smem: C * 4 bytes.
extern "C" __global__ void qwen_qkv_rope(const unsigned short *__restrict__ Wqkv,
                                         const unsigned short *__restrict__ bqkv,
                                         const unsigned short *__restrict__ g_in,
                                         const float *__restrict__ x, const float *__restrict__ cosT,
                                         const float *__restrict__ sinT, SbStep *__restrict__ st,
                                         float *__restrict__ q_out, float *__restrict__ kc,
                                         float *__restrict__ vc, int C, int NH, int NKV, int HD, float eps) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    const int KVD = NKV * HD, NQKV = C + 2 * KVD, hd2 = HD / 2;
    const int ntasks = NQKV / 2;  // (head, i) pairs
    int t0, t1;
    cta_task_range(ntasks, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0 && t1 > t0) {
        for (int h = t0 / hd2; h <= (t1 - 1) / hd2; h++) {
            const int i0 = max(t0 - h * hd2, 0), i1 = min(t1 - h * hd2, hd2);
            prefetch_rows(Wqkv, (long)C * 2, h * HD + i0, h * HD + i1, 1L << 20);
            prefetch_rows(Wqkv, (long)C * 2, h * HD + hd2 + i0, h * HD + hd2 + i1, 1L << 20);
        }
    }
    pdl_wait();
    if (sb_step_idle(st)) return;
    const int pos = st->pos;
    const float inv = block_rms_scale(x, C, eps, red);
    float4 *lo = xs4, *hi = xs4 + C / 8;
    stage_x_split8(x, C, lo, hi, inv, g_in);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int cpr = C / 8;
    XSplit8 xa{lo, hi};
    for (int t = t0 + warp; t < t1; t += nw) {
        const int h = t / hd2, i = t % hd2;
        const int rows[2] = {h * HD + i, h * HD + hd2 + i};
        float a[2];
        warp_dot_h<2, 4>(reinterpret_cast<const uint4 *>(Wqkv), cpr, rows, cpr, xa, a);
        if ((threadIdx.x & 31) == 0) {
            float y0 = __fadd_rn(a[0], h2f_ftz(bqkv[rows[0]]));
            float y1 = __fadd_rn(a[1], h2f_ftz(bqkv[rows[1]]));
            if (h < NH + NKV) {  // q and k heads are rotated
                const float c = cosT[(size_t)pos * hd2 + i], s = sinT[(size_t)pos * hd2 + i];
                const float o0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
                const float o1 = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
                y0 = o0;
                y1 = o1;
            }
            if (h < NH) {
                q_out[rows[0]] = y0;
                q_out[rows[1]] = y1;
            } else if (h < NH + NKV) {
                kc[(size_t)pos * KVD + (rows[0] - C)] = y0;
                kc[(size_t)pos * KVD + (rows[1] - C)] = y1;
            } else {
                vc[(size_t)pos * KVD + (rows[0] - C - KVD)] = y0;
                vc[(size_t)pos * KVD + (rows[1] - C - KVD)] = y1;
            }
        }
    }
}

// GQA decode attention at the step's position.  grid (NKV, max_splits),
// block SB_ATTN_THREADS.  Replaces attn_scores_gqa + attn_softmax +
// attn_mix_gqa (qwen_engine.c:231-236).  part/counters are scratch owned by
// the caller: (NKV*max_splits*7*66) floats and NKV zeroed counters.
extern "C" __global__ void qwen_attn(const float *__restrict__ q, const float *__restrict__ kc,
                                     const float *__restrict__ vc, SbStep *__restrict__ st,
                                     float *__restrict__ out, float *__restrict__ part,
                                     unsigned *__restrict__ counters, int kv_stride, float scale,
                                     int max_splits) {
    pdl_launch_dependents();
    pdl_wait();
    if (sb_step_idle(st)) return;
    attn_decode_body<7>(q, kc, vc, st->pos + 1, out, part, counters, kv_stride, scale, max_splits);
}

// x[n] += sum_k h2f(W[n][k]) v[k]: the O and down projections with the
// residual add fused (replaces gemv_h + add2, qwen_engine.c:242-245,256-259);
// each row split over `ksplit` warps.  grid: any; block: multiple of 32 with
// (block/32) % ksplit == 0; no dynamic smem.
extern "C" __global__ void qwen_gemv_resid(const unsigned short *__restrict__ W, const float *__restrict__ v,
                                           SbStep *__restrict__ st, float *__restrict__ x, int K, int N,
                                           int ksplit) {
    resid_splitk_body<true>(W, nullptr, v, st, x, K, N, ksplit);
}

// RMSNorm(x) -> gate|up GEMV -> SwiGLU: hid[i] = silu(g_i) * u_i; a warp owns
// gate rows (i, i+1) and up rows (FC+i, FC+i+1).  Replaces rmsnorm + gemv_h
// + swiglu (qwen_engine.c:247-254).  dynamic smem: C * 4 bytes.
extern "C" __global__ void qwen_gateup_swiglu(const unsigned short *__restrict__ Wgu,
                                              const unsigned short *__restrict__ g_post,
                                              const float *__restrict__ x, SbStep *__restrict__ st,
                                              float *__restrict__ hid, int C, int FC, float eps) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    int t0, t1;
    cta_task_range((FC + 1) / 2, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        const long r0 = 2L * t0, r1 = min(2L * t1, (long)FC);
        prefetch_rows(Wgu, (long)C * 2, r0, r1, 1L << 20);
        prefetch_rows(Wgu, (long)C * 2, FC + r0, FC + r1, 1L << 20);
    }
    pdl_wait();
    if (sb_step_idle(st)) return;
    const float inv = block_rms_scale(x, C, eps, red);
    float4 *lo = xs4, *hi = xs4 + C / 8;
    stage_x_split8(x, C, lo, hi, inv, g_post);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = C / 8;
    XSplit8 xa{lo, hi};
    for (int t = t0 + warp; t < t1; t += nw) {
        const int i = 2 * t;
        const bool two = (i + 1 < FC);
        const int rows[4] = {i, two ? i + 1 : -1, FC + i, two ? FC + i + 1 : -1};
        float a[4];
        warp_dot_h<4, 4>(reinterpret_cast<const uint4 *>(Wgu), cpr, rows, cpr, xa, a);
        const int lane = threadIdx.x & 31;
        if (lane == 0) hid[i] = silu_mul(a[0], a[2]);
        if (lane == 1 && two) hid[i + 1] = silu_mul(a[1], a[3]);
    }
}

// Final RMSNorm -> tied LM head GEMV (logits) -> argmax, fused.  Replaces
// rmsnorm + gemv_h + the host argmax over V logits (qwen_engine.c:263-268,
// 360-364).  dynamic smem: C * 4 bytes.
extern "C" __global__ void qwen_lmhead(const unsigned short *__restrict__ Wemb,
                                       const unsigned short *__restrict__ g_final,
                                       const float *__restrict__ x, SbStep *__restrict__ st,
                                       float *__restrict__ logits, int C, int V, float eps) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    __shared__ unsigned long long best_s;
    constexpr int R = 4;
    int t0, t1;
    cta_task_range((V + R - 1) / R, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0) prefetch_rows(Wemb, (long)C * 2, (long)t0 * R, min((long)t1 * R, (long)V), 96L << 10);
    pdl_wait();
    if (sb_step_idle(st)) return;
    if (threadIdx.x == 0) best_s = 0ull;
    const float inv = block_rms_scale(x, C, eps, red);
    float4 *lo = xs4, *hi = xs4 + C / 8;
    stage_x_split8(x, C, lo, hi, inv, g_final);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = C / 8, lane = threadIdx.x & 31;
    XSplit8 xa{lo, hi};
    unsigned long long best = 0ull;
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, V, rows);
        float acc[R];
        warp_dot_h<R, 4>(reinterpret_cast<const uint4 *>(Wemb), cpr, rows, cpr, xa, acc);
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (rows[r] >= 0) {
                if (lane == r) logits[rows[r]] = acc[r];
                const unsigned long long k = argmax_key(acc[r], rows[r]);
                best = k > best ? k : best;
            }
        }
    }
    if (lane == 0 && best) atomicMax(&best_s, best);
    __syncthreads();
    if (threadIdx.x == 0 && best_s) atomicMax(&st->key, best_s);
}


// Flush fp16 subnormals (exponent 0) to +0 in place, 16 bytes per thread
// step.  The reference decodes exponent-0 weights as 0 (qwen_engine.c:90-98);
// once the engine's device copy holds them as 0, its kernels can use the
// plain hardware conversion and get exactly the reference's values.
extern "C" __global__ void fp16_flush_subnormals(uint4 *__restrict__ p, long n16) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n16; i += (long)gridDim.x * blockDim.x) {
        uint4 w = p[i];
        w.x = ftz_half2_bits(w.x);
        w.y = ftz_half2_bits(w.y);
        w.z = ftz_half2_bits(w.z);
        w.w = ftz_half2_bits(w.w);
        p[i] = w;
    }
}

// out[z][c][r] = in[z][r][c]: per layer z, an fp16 rows x cols matrix
// transposed through 32 x 32 shared-memory tiles (both sides coalesced).
// The engine writes W_down's transpose with it once at load time, for the
// persistent kernel's split-K down projection.  grid (ceil(cols/32),
// ceil(rows/32), layers), block 256.
extern "C" __global__ void __launch_bounds__(256) transpose_u16(const unsigned short *__restrict__ in,
                                                               unsigned short *__restrict__ out, int rows, int cols,
                                                               long in_stride, long out_stride) {
    __shared__ unsigned short t[32][33];
    if (blockDim.x != 256) return;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    in += blockIdx.z * in_stride;
    out += blockIdx.z * out_stride;
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + tx;
        if (r < rows && c < cols) t[i][tx] = in[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + tx;
        if (c < cols && r < rows) out[(size_t)c * rows + r] = t[tx][i];
    }
}

// =====================================================================
// Part 3 -- the persistent whole-step kernels
// =====================================================================
#include "qwen_mk.cuh"
#include "qwen_mk2.cuh"

// ===========================================================================
// Batched prompt prefill: T prompt tokens at positions pos0..pos0+T-1 run
// through each layer together, the weight products on the tensor cores
// (gemm_hh_tc) instead of T separate matvec passes (the reference primes the
// prompt one token at a time through cpu/gpu_forward, qwen_engine.c:529).
// Activations enter the fp16 tensor-core GEMM as two rows each:
// hi = fp16(x) and lo = fp16(x - hi), so W.x = W.hi + W.lo keeps ~22 bits
// of x; the GEMM output holds the hi products in rows [0, T) and the lo
// products in rows [T, 2T).  Prompt tokens need no logits, so only the KV
// cache is the product of a prefill.

SB_DEV void pf_split(float v, unsigned short *hi, unsigned short *lo) {
    const __half h = __float2half_rn(v);
    *hi = __half_as_ushort(h);
    *lo = __half_as_ushort(__float2half_rn(v - __half2float(h)));
}

// X[t][:] = embedding row of tokens[pos0 + t].  grid (T, any), block 256.
extern "C" __global__ void qwen_pf_embed(const unsigned short *__restrict__ emb, const int *__restrict__ tokens,
                                         float *__restrict__ X, int pos0, int C) {
    const int t = blockIdx.x, tok = tokens[pos0 + t];
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < C; i += gridDim.y * blockDim.x) X[(size_t)t * C + i] = h2f_ftz(emb[(size_t)tok * C + i]);
}

// XH rows t (hi) and T + t (lo) = split(RMSNorm(X[t]) * g).  grid T, block 256.
extern "C" __global__ void qwen_pf_rms_split(const float *__restrict__ X, const unsigned short *__restrict__ g,
                                             unsigned short *__restrict__ XH, int T, int C, float eps) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    const float *x = X + (size_t)t * C;
    float s = 0.f;
    for (int i = threadIdx.x; i < C; i += blockDim.x) s = fmaf(x[i], x[i], s);
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(__fdiv_rn(s, (float)C) + eps);
    for (int i = threadIdx.x; i < C; i += blockDim.x)
        pf_split(__fmul_rn(__fmul_rn(x[i], inv), h2f_ftz(g[i])), XH + (size_t)t * C + i, XH + (size_t)(T + t) * C + i);
}

// XH rows t / T + t = split(X[t]).  grid (T, any), block 256.
extern "C" __global__ void qwen_pf_split(const float *__restrict__ X, unsigned short *__restrict__ XH, int T, int n) {
    const int t = blockIdx.x;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < n; i += gridDim.y * blockDim.x)
        pf_split(X[(size_t)t * n + i], XH + (size_t)t * n + i, XH + (size_t)(T + t) * n + i);
}

// QKV of token t = Y[t] + Y[T + t] + bias, RoPE (pairs i, i + HD/2) at
// pos0 + t for the q and k heads; q -> Q[t], k and v -> the cache rows.
// grid (T, any), block 256.
extern "C" __global__ void qwen_pf_qkv(const float *__restrict__ Y, const unsigned short *__restrict__ bqkv,
                                       const float *__restrict__ cosT, const float *__restrict__ sinT,
                                       float *__restrict__ Q, float *__restrict__ kc, float *__restrict__ vc, int T,
                                       int pos0, int C, int NH, int NKV, int HD) {
    const int t = blockIdx.x, pos = pos0 + t;
    const int KVD = NKV * HD, NQKV = C + 2 * KVD, hd2 = HD / 2;
    const float *yh = Y + (size_t)t * NQKV, *yl = Y + (size_t)(T + t) * NQKV;
    for (int p = blockIdx.y * blockDim.x + threadIdx.x; p < NQKV / 2; p += gridDim.y * blockDim.x) {
        const int h = p / hd2, i = p % hd2, r0 = h * HD + i, r1 = r0 + hd2;
        float y0 = __fadd_rn(__fadd_rn(yh[r0], yl[r0]), h2f_ftz(bqkv[r0]));
        float y1 = __fadd_rn(__fadd_rn(yh[r1], yl[r1]), h2f_ftz(bqkv[r1]));
        if (h < NH + NKV) {
            const float c = cosT[(size_t)pos * hd2 + i], s = sinT[(size_t)pos * hd2 + i];
            const float o0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
            const float o1 = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
            y0 = o0;
            y1 = o1;
        }
        if (h < NH) {
            Q[(size_t)t * C + r0] = y0;
            Q[(size_t)t * C + r1] = y1;
        } else if (h < NH + NKV) {
            kc[(size_t)pos * KVD + r0 - C] = y0;
            kc[(size_t)pos * KVD + r1 - C] = y1;
        } else {
            vc[(size_t)pos * KVD + r0 - C - KVD] = y0;
            vc[(size_t)pos * KVD + r1 - C - KVD] = y1;
        }
    }
}

// Causal GQA attention of token t, head h over positions 0..pos0+t, the
// reference's arithmetic (scores, max-subtracted softmax, mix; FP32).
// grid (T, NH), block 128, dynamic smem (pos0 + T) * 4 bytes.
extern "C" __global__ void qwen_pf_attn(const float *__restrict__ Q, const float *__restrict__ kc,
                                        const float *__restrict__ vc, float *__restrict__ ATT, int pos0, int C, int NH,
                                        int NKV, int HD, float scale) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    const int t = blockIdx.x, h = blockIdx.y, g = h / (NH / NKV), KVD = NKV * HD;
    const int n = pos0 + t + 1;
    const float *q = Q + (size_t)t * C + h * HD;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        const float *k = kc + (size_t)p * KVD + g * HD;
        float d = 0.f;
        for (int j = 0; j < HD; j++) d = fmaf(q[j], k[j], d);
        sc[p] = d * scale;
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // the row maximum, by one warp
        float mm = -1e30f;
        for (int p = threadIdx.x; p < n; p += 32) mm = fmaxf(mm, sc[p]);
        mm = warp_max(mm);
        if (threadIdx.x == 0) red[0] = mm;
    }
    __syncthreads();
    const float mx = red[0];
    __syncthreads();
    float l = 0.f;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        const float e = expf(sc[p] - mx);
        sc[p] = e;
        l += e;
    }
    l = block_sum(l, red);
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float acc = 0.f;
        for (int p = 0; p < n; p++) acc = fmaf(sc[p], vc[(size_t)p * KVD + g * HD + d], acc);
        ATT[(size_t)t * C + h * HD + d] = acc / l;
    }
}

// X[t] += Y[t] + Y[T + t] (the residual add of a product).  grid (T, any), block 256.
extern "C" __global__ void qwen_pf_resid(const float *__restrict__ Y, float *__restrict__ X, int T, int n) {
    const int t = blockIdx.x;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < n; i += gridDim.y * blockDim.x)
        X[(size_t)t * n + i] = __fadd_rn(X[(size_t)t * n + i], __fadd_rn(Y[(size_t)t * n + i], Y[(size_t)(T + t) * n + i]));
}

// hid = silu(gate) * up from the gate|up product Y (rows of 2*FC), split into
// hi/lo rows of XH for the down projection.  grid (T, any), block 256.
extern "C" __global__ void qwen_pf_swiglu_split(const float *__restrict__ Y, unsigned short *__restrict__ XH, int T,
                                                int FC) {
    const int t = blockIdx.x;
    const float *yh = Y + (size_t)t * 2 * FC, *yl = Y + (size_t)(T + t) * 2 * FC;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < FC; i += gridDim.y * blockDim.x) {
        const float gt = __fadd_rn(yh[i], yl[i]), up = __fadd_rn(yh[FC + i], yl[FC + i]);
        pf_split(__fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up), XH + (size_t)t * FC + i,
                 XH + (size_t)(T + t) * FC + i);
    }
}
