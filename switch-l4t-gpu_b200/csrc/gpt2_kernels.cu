// gpt2_kernels.cu -- the "gpt2" module image (sm_100a cubin).
//
// Part 1: drop-ins with the reference's names and parameter lists
// (gpu-llm/kernels/gpt2_kernels.cu), correct under the stock launch geometry
// of gpt2_engine.c:181-325 or any other.
// Part 2: fused FP32 decode-step kernels for this package's engine (device
// step state, programmatic dependent launch; see qwen_kernels.cu).
#include "sb_attn.cuh"
#include "sb_gemv.cuh"
#include "sb_step.h"
#include "sb_finalize.cuh"
#include "sb_resid.cuh"

// =====================================================================
// Part 1 -- drop-ins
// =====================================================================

// Warp-per-row FP32 GEMV over all warps of any grid (K % 4 == 0, 16-byte
// aligned rows), else one thread per row.
SB_DEV void gemv_f32_any(const float *__restrict__ W, const float *__restrict__ x,
                         const float *__restrict__ bias, float *__restrict__ y, int K, int N) {
    const int nthreads = gridDim.x * blockDim.x;
    const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec = ((K & 3) == 0) && ((((uintptr_t)W) & 15) == 0) && ((((uintptr_t)x) & 15) == 0);
    if (vec && (blockDim.x & 31) == 0) {
        const int warp = gtid >> 5, nwarp = nthreads >> 5, cpr = K >> 2;
        XGlob4 xa{x};
        for (int n = warp; n < N; n += nwarp) {
            float acc[1];
            const int rows[1] = {n};
            warp_dot_f<1, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cpr, xa, acc);
            if ((threadIdx.x & 31) == 0) y[n] = acc[0] + (bias ? bias[n] : 0.0f);
        }
        return;
    }
    for (int n = gtid; n < N; n += nthreads) {
        const float *row = W + (size_t)n * K;
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc = fmaf(row[k], x[k], acc);
        y[n] = acc + (bias ? bias[n] : 0.0f);
    }
}

// y = W x.  Reference: gpt2_kernels.cu:38-72 (grid ceil(N/8), block 256).
extern "C" __global__ void gemv_warp(const float *__restrict__ W, const float *__restrict__ x,
                                     float *__restrict__ y, int K, int N) {
    gemv_f32_any(W, x, nullptr, y, K, N);
}

// y = W x + bias.  Reference: gpt2_kernels.cu:75-108.
extern "C" __global__ void gemv_warp_b(const float *__restrict__ W, const float *__restrict__ x,
                                       const float *__restrict__ bias, float *__restrict__ y, int K, int N) {
    gemv_f32_any(W, x, bias, y, K, N);
}

// Y[t*N+n] = sum_k W[n*K+k] X[t*K+k] (+bias[n]).  Reference:
// gpt2_kernels.cu:115-155 (grid (ceil(N/8), ceil(T/16)), block 256).  A
// warp streams its W row chunk once and applies it to up to 16 token rows
// held in 16 accumulators; tasks (row, 16-token chunk) are grid-strided over
// every warp of the launch, so any grid is correct.
extern "C" __global__ void gemv_multi(const float *__restrict__ W, const float *__restrict__ X,
                                      const float *__restrict__ bias, float *__restrict__ Y, int K, int N,
                                      int T) {
    constexpr int TW = 16;
    const int nthreads = gridDim.x * gridDim.y * blockDim.x;
    const int gtid = (blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x;
    const int nchunks = (T + TW - 1) / TW;
    const long ntasks = (long)N * nchunks;
    const bool vec = ((K & 3) == 0) && ((((uintptr_t)W) & 15) == 0) && ((((uintptr_t)X) & 15) == 0);
    if (vec && (blockDim.x & 31) == 0) {
        const int lane = threadIdx.x & 31, warp = gtid >> 5, nwarp = nthreads >> 5, cpr = K >> 2;
        for (long task = warp; task < ntasks; task += nwarp) {
            const int n = (int)(task / nchunks), t0 = (int)(task % nchunks) * TW;
            const int tmax = min(TW, T - t0);
            float acc[TW];
#pragma unroll
            for (int j = 0; j < TW; j++) acc[j] = 0.0f;
            const uint4 *wrow = reinterpret_cast<const uint4 *>(W + (size_t)n * K);
            for (int c = lane; c < cpr; c += 32) {
                const uint4 w = ld_stream_u4(wrow + c);
#pragma unroll
                for (int j = 0; j < TW; j++)
                    if (j < tmax) acc[j] = dot_chunk(WF(), w, ld_f4(X + (size_t)(t0 + j) * K + 4 * c), acc[j]);
            }
#pragma unroll
            for (int j = 0; j < TW; j++) {
                const float s = warp_sum(acc[j]);
                if (lane == 0 && j < tmax) Y[(size_t)(t0 + j) * N + n] = s + (bias ? bias[n] : 0.0f);
            }
        }
        return;
    }
    for (long task = gtid; task < (long)N * T; task += nthreads) {
        const int n = (int)(task % N), t = (int)(task / N);
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc = fmaf(W[(size_t)n * K + k], X[(size_t)t * K + k], acc);
        Y[(size_t)t * N + n] = acc + (bias ? bias[n] : 0.0f);
    }
}

// LayerNorm scale/shift statistics of one row: centred two-pass variance, as
// the reference's CPU golden model computes it (gpt2_engine.c:333-341).
SB_DEV void block_ln_stats(const float *x, int n, float eps, float *red, float &mean, float &inv) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
    mean = __fdiv_rn(block_sum(s, red), (float)n);
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float d = x[i] - mean;
        v = fmaf(d, d, v);
    }
    const float var = __fdiv_rn(block_sum(v, red), (float)n);
    inv = 1.0f / sqrtf(var + eps);
}
SB_DEV float ln_apply(float x, float mean, float inv, float w, float b) {
    return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, mean), inv), w), b);
}

// y = (x-mean)/sqrt(var+eps)*w + b, one block per row (grid = T).
// Reference: gpt2_kernels.cu:160-196.
extern "C" __global__ void layernorm(const float *__restrict__ x, const float *__restrict__ w,
                                     const float *__restrict__ b, float *__restrict__ y, int n, float eps) {
    __shared__ float red[32];
    x += (size_t)blockIdx.x * n;
    y += (size_t)blockIdx.x * n;
    float mean, inv;
    block_ln_stats(x, n, eps, red, mean, inv);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = ln_apply(x[i], mean, inv, w[i], b[i]);
}

// tanh-GELU with every product/sum rounded in the reference C's order
// (gpt2_engine.c:406-410).
SB_DEV float gelu_ref(float v) {
    const float p = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    const float t = __fmul_rn(0.7978845608f, __fadd_rn(v, p));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(t)));
}

// Reference: gpt2_kernels.cu:199-206.
extern "C" __global__ void gelu(const float *__restrict__ x, float *__restrict__ y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = gelu_ref(x[i]);
}
// Reference: gpt2_kernels.cu:209-212.
extern "C" __global__ void add_bias(float *__restrict__ y, const float *__restrict__ b, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] += b[i];
}
// Reference: gpt2_kernels.cu:213-217.
extern "C" __global__ void add2(const float *__restrict__ a, const float *__restrict__ b,
                                float *__restrict__ out, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = a[i] + b[i];
}

// scores[t*12+h] = q_h . kcache[t*768 + h*64 ..] * scale (12 heads of 64).
// Reference: gpt2_kernels.cu:221-235.
extern "C" __global__ void attn_scores(const float *__restrict__ q, const float *__restrict__ kcache,
                                       float *__restrict__ scores, int T, float scale) {
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < T * 12; idx += gridDim.x * blockDim.x) {
        const int t = idx / 12, h = idx % 12;
        const float *qh = q + h * 64, *kh = kcache + (size_t)t * 768 + h * 64;
        float acc = 0.0f;
        for (int d = 0; d < 64; d++) acc = fmaf(qh[d], kh[d], acc);
        scores[idx] = acc * scale;
    }
}
// Per-head softmax over T, 12 heads.  Reference: gpt2_kernels.cu:238-255.
extern "C" __global__ void attn_softmax(const float *__restrict__ scores, float *__restrict__ probs, int T) {
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < 12; h += gridDim.x * blockDim.x) {
        float maxv = scores[h];
        for (int t = 1; t < T; t++) maxv = fmaxf(maxv, scores[(size_t)t * 12 + h]);
        float sum = 0.0f;
        for (int t = 0; t < T; t++) {
            const float e = expf(scores[(size_t)t * 12 + h] - maxv);
            probs[(size_t)t * 12 + h] = e;
            sum += e;
        }
        const float inv = 1.0f / sum;
        for (int t = 0; t < T; t++) probs[(size_t)t * 12 + h] *= inv;
    }
}
// out[d] = sum_t probs[t*12 + d/64] vcache[t*768 + d].  Reference:
// gpt2_kernels.cu:258-268.
extern "C" __global__ void attn_mix(const float *__restrict__ probs, const float *__restrict__ vcache,
                                    float *__restrict__ out, int T) {
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < 768; d += gridDim.x * blockDim.x) {
        const int h = d / 64;
        float acc = 0.0f;
        for (int t = 0; t < T; t++) acc = fmaf(probs[(size_t)t * 12 + h], vcache[(size_t)t * 768 + d], acc);
        out[d] = acc;
    }
}

// =====================================================================
// Part 1b -- this package's standalone entry kernels (tuned geometry)
// =====================================================================

// y = W x (+bias), FP32; x staged in shared memory, 4-row warp tasks, a
// contiguous row range per CTA.  dynamic smem K*4, K % 4 == 0.
extern "C" __global__ void __launch_bounds__(256) gemv_f32_b200(const float *__restrict__ W,
                                                                const float *__restrict__ x,
                                                                const float *__restrict__ bias,
                                                                float *__restrict__ y, int K, int N) {
    extern __shared__ float4 xs4[];
    constexpr int R = 4;
    int t0, t1;
    cta_task_range((N + R - 1) / R, t0, t1);
    for (int c = threadIdx.x; c < K / 4; c += blockDim.x) xs4[c] = ld_f4(x + 4 * c);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = K / 4, lane = threadIdx.x & 31;
    XSmem4 xa{xs4};
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, N, rows);
        float acc[R];
        warp_dot_f<R, 4>(reinterpret_cast<const uint4 *>(W), cpr, rows, cpr, xa, acc);
#pragma unroll
        for (int r = 0; r < R; r++)
            if (lane == r && rows[r] >= 0) y[rows[r]] = acc[r] + (bias ? bias[rows[r]] : 0.0f);
    }
}

// gemv_f32_b200 for short outputs: split-K over a CTA's warps
// (splitk_rows4), x read through L1.  Block 256, no dynamic shared memory,
// K % 4 == 0.
extern "C" __global__ void __launch_bounds__(256) gemv_f32_sk(const float *__restrict__ W,
                                                              const float *__restrict__ x,
                                                              const float *__restrict__ bias,
                                                              float *__restrict__ y, int K, int N) {
    const uint4 *W4 = reinterpret_cast<const uint4 *>(W);
    const int cpr = K / 4;
    const XGlob4 xa{x};
    splitk_rows4(N, cpr, bias, y, [&](const int (&rows)[4], int cb, int ce, float (&acc)[4]) {
        warp_dot_f_range<4, 4>(W4, cpr, rows, cb, ce, xa, acc);
    });
}

// MHA decode attention with an explicit T; one query head per KV slot.
extern "C" __global__ void attn_decode_g1(const float *__restrict__ q, const float *__restrict__ kc,
                                          const float *__restrict__ vc, int T, float *__restrict__ out,
                                          float *__restrict__ part, unsigned *__restrict__ counters,
                                          int kv_stride, float scale, int max_splits) {
    attn_decode_body<1>(q, kc, vc, T, out, part, counters, kv_stride, scale, max_splits);
}

// =====================================================================
// Part 2 -- fused FP32 decode-step kernels
// =====================================================================

// x = wte[token] + wpe[pos] (gpt2_engine.c:176-179, done on the host there).
extern "C" __global__ void gpt2_embed(const float *__restrict__ wte, const float *__restrict__ wpe,
                                      const int *__restrict__ tokens, SbStep *__restrict__ st,
                                      float *__restrict__ x, int C) {
    pdl_launch_dependents();
    pdl_wait();
    if (sb_step_idle(st)) return;
    const int tok = tokens[st->pos], pos = st->pos;
    for (int i = threadIdx.x; i < C; i += blockDim.x)
        x[i] = __fadd_rn(wte[(size_t)tok * C + i], wpe[(size_t)pos * C + i]);
}

// Stage LayerNorm(x) into shared memory as K/4 float4.
SB_DEV void stage_ln4(const float *x, int C, const float *w, const float *b, float eps, float *red, float4 *xs) {
    float mean, inv;
    block_ln_stats(x, C, eps, red, mean, inv);
    for (int c = threadIdx.x; c < C / 4; c += blockDim.x) {
        const float4 v = ld_f4(x + 4 * c), ww = ld_f4(w + 4 * c), bb = ld_f4(b + 4 * c);
        xs[c] = make_float4(ln_apply(v.x, mean, inv, ww.x, bb.x), ln_apply(v.y, mean, inv, ww.y, bb.y),
                            ln_apply(v.z, mean, inv, ww.z, bb.z), ln_apply(v.w, mean, inv, ww.w, bb.w));
    }
}
SB_DEV void stage_copy4(const float *x, int K, float4 *xs) {
    for (int c = threadIdx.x; c < K / 4; c += blockDim.x) xs[c] = ld_f4(x + 4 * c);
}

// LN1(x) -> QKV GEMV + bias -> q out, k/v into the cache at pos.  Replaces
// layernorm + gemv_warp(_b) + add_bias + 2 DtoD copies (gpt2_engine.c:181-196).
// dynamic smem: C * 4 bytes.
extern "C" __global__ void gpt2_ln_qkv(const float *__restrict__ Wqkv, const float *__restrict__ bqkv,
                                       const float *__restrict__ lnw, const float *__restrict__ lnb,
                                       const float *__restrict__ x, SbStep *__restrict__ st,
                                       float *__restrict__ q_out, float *__restrict__ kc,
                                       float *__restrict__ vc, int C, float eps) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    constexpr int R = 2;
    const int N = 3 * C;
    int t0, t1;
    cta_task_range(N / R, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0) prefetch_rows(Wqkv, (long)C * 4, (long)t0 * R, (long)t1 * R, 1L << 20);
    pdl_wait();
    if (sb_step_idle(st)) return;
    const int pos = st->pos;
    stage_ln4(x, C, lnw, lnb, eps, red, xs4);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = C / 4, lane = threadIdx.x & 31;
    XSmem4 xa{xs4};
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, N, rows);
        float acc[R];
        warp_dot_f<R, 4>(reinterpret_cast<const uint4 *>(Wqkv), cpr, rows, cpr, xa, acc);
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (lane == r && rows[r] >= 0) {
                const int n = rows[r];
                const float y = __fadd_rn(acc[r], bqkv[n]);
                if (n < C) q_out[n] = y;
                else if (n < 2 * C) kc[(size_t)pos * C + (n - C)] = y;
                else vc[(size_t)pos * C + (n - 2 * C)] = y;
            }
        }
    }
}

// MHA decode attention at the step's position; grid (12, max_splits).
// Replaces attn_scores + attn_softmax + attn_mix (gpt2_engine.c:197-204).
extern "C" __global__ void gpt2_attn(const float *__restrict__ q, const float *__restrict__ kc,
                                     const float *__restrict__ vc, SbStep *__restrict__ st,
                                     float *__restrict__ out, float *__restrict__ part,
                                     unsigned *__restrict__ counters, int kv_stride, float scale,
                                     int max_splits) {
    pdl_launch_dependents();
    pdl_wait();
    if (sb_step_idle(st)) return;
    attn_decode_body<1>(q, kc, vc, st->pos + 1, out, part, counters, kv_stride, scale, max_splits);
}

// x[n] += (W v)[n] + b[n]: attention-out and MLP projections with bias and
// residual fused (gpt2_engine.c:210-221, 239-250); each row split over
// `ksplit` warps.  No dynamic smem.
extern "C" __global__ void gpt2_gemv_resid(const float *__restrict__ W, const float *__restrict__ b,
                                           const float *__restrict__ v, SbStep *__restrict__ st,
                                           float *__restrict__ x, int K, int N, int ksplit) {
    resid_splitk_body<false>(W, b, v, st, x, K, N, ksplit);
}

// LN2(x) -> fc GEMV + bias -> GELU (gpt2_engine.c:223-238).  dynamic smem C*4.
extern "C" __global__ void gpt2_ln_fc_gelu(const float *__restrict__ Wfc, const float *__restrict__ bfc,
                                           const float *__restrict__ lnw, const float *__restrict__ lnb,
                                           const float *__restrict__ x, SbStep *__restrict__ st,
                                           float *__restrict__ hid, int C, int FC, float eps) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    constexpr int R = 4;
    int t0, t1;
    cta_task_range((FC + R - 1) / R, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0) prefetch_rows(Wfc, (long)C * 4, (long)t0 * R, min((long)t1 * R, (long)FC), 1L << 20);
    pdl_wait();
    if (sb_step_idle(st)) return;
    stage_ln4(x, C, lnw, lnb, eps, red, xs4);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = C / 4, lane = threadIdx.x & 31;
    XSmem4 xa{xs4};
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, FC, rows);
        float acc[R];
        warp_dot_f<R, 4>(reinterpret_cast<const uint4 *>(Wfc), cpr, rows, cpr, xa, acc);
#pragma unroll
        for (int r = 0; r < R; r++)
            if (lane == r && rows[r] >= 0) hid[rows[r]] = gelu_ref(__fadd_rn(acc[r], bfc[rows[r]]));
    }
}

// LN_f(x) -> tied LM head (wte) -> logits + argmax (gpt2_engine.c:257-263,
// 424-428).  dynamic smem: C * 4 bytes.
extern "C" __global__ void gpt2_lmhead(const float *__restrict__ wte, const float *__restrict__ lnw,
                                       const float *__restrict__ lnb, const float *__restrict__ x,
                                       SbStep *__restrict__ st, float *__restrict__ logits, int C, int V,
                                       float eps) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    __shared__ unsigned long long best_s;
    constexpr int R = 4;
    int t0, t1;
    cta_task_range((V + R - 1) / R, t0, t1);
    pdl_launch_dependents();
    if (threadIdx.x == 0) prefetch_rows(wte, (long)C * 4, (long)t0 * R, min((long)t1 * R, (long)V), 96L << 10);
    pdl_wait();
    if (sb_step_idle(st)) return;
    if (threadIdx.x == 0) best_s = 0ull;
    stage_ln4(x, C, lnw, lnb, eps, red, xs4);
    __syncthreads();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, cpr = C / 4, lane = threadIdx.x & 31;
    XSmem4 xa{xs4};
    unsigned long long best = 0ull;
    for (int t = t0 + warp; t < t1; t += nw) {
        int rows[R];
        consecutive_rows<R>(t * R, V, rows);
        float acc[R];
        warp_dot_f<R, 4>(reinterpret_cast<const uint4 *>(wte), cpr, rows, cpr, xa, acc);
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

// ===========================================================================
// Batched prompt prefill (the reference's gpu_prefill, gpt2_engine.c:269-326,
// which batches the weight products through gemv_multi): T prompt tokens at
// positions pos0..pos0+T-1 per layer, the products as 3xTF32 tensor-core
// GEMMs (FP32 accuracy) against the [out][in] weights, these kernels for the
// element-wise steps, causal attention per (token, head).  Only the KV cache
// is produced (prompt tokens need no logits).

// X[t] = wte[tokens[pos0 + t]] + wpe[pos0 + t] (gpt2_engine.c:178-180).  grid (T, any), block 256.
extern "C" __global__ void gpt2_pf_embed(const float *__restrict__ wte, const float *__restrict__ wpe,
                                         const int *__restrict__ tokens, float *__restrict__ X, int pos0, int C) {
    const int t = blockIdx.x, tok = tokens[pos0 + t];
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < C; i += gridDim.y * blockDim.x)
        X[(size_t)t * C + i] = __fadd_rn(wte[(size_t)tok * C + i], wpe[(size_t)(pos0 + t) * C + i]);
}

// q, k, v of token t = Y[t] + bias; q -> Q[t], k and v -> the cache rows at
// pos0 + t.  grid (T, any), block 256.
extern "C" __global__ void gpt2_pf_qkv(const float *__restrict__ Y, const float *__restrict__ b,
                                       float *__restrict__ Q, float *__restrict__ kc, float *__restrict__ vc, int pos0,
                                       int C) {
    const int t = blockIdx.x, pos = pos0 + t;
    const float *y = Y + (size_t)t * 3 * C;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < C; i += gridDim.y * blockDim.x) {
        Q[(size_t)t * C + i] = __fadd_rn(y[i], b[i]);
        kc[(size_t)pos * C + i] = __fadd_rn(y[C + i], b[C + i]);
        vc[(size_t)pos * C + i] = __fadd_rn(y[2 * C + i], b[2 * C + i]);
    }
}

// X[t] += Y[t] + bias (gemv_warp_b then add2).  grid (T, any), block 256.
extern "C" __global__ void gpt2_pf_bias_resid(const float *__restrict__ Y, const float *__restrict__ b,
                                              float *__restrict__ X, int n) {
    const int t = blockIdx.x;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < n; i += gridDim.y * blockDim.x)
        X[(size_t)t * n + i] = __fadd_rn(X[(size_t)t * n + i], __fadd_rn(Y[(size_t)t * n + i], b[i]));
}

// A[t] = gelu(Y[t] + bias) (gemv_warp_b then gelu).  grid (T, any), block 256.
extern "C" __global__ void gpt2_pf_bias_gelu(const float *__restrict__ Y, const float *__restrict__ b,
                                             float *__restrict__ A, int n) {
    const int t = blockIdx.x;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < n; i += gridDim.y * blockDim.x)
        A[(size_t)t * n + i] = gelu_ref(__fadd_rn(Y[(size_t)t * n + i], b[i]));
}

// The whole decode step as one persistent kernel.
#include "gpt2_mk.cuh"
