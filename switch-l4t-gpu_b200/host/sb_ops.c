/* sb_ops.c -- host entry points for the individual hot-path operations.
 * Each one validates its arguments, picks the launch shape for this device
 * and issues one (or a few) kernel launches on the caller's stream. */
#include <stdint.h>
#include <string.h>

#include "sb_internal.h"

#define CEIL_DIV(a, b) (((a) + (b)-1) / (b))
#define DP(p) ((CUdeviceptr)(uintptr_t)(p))
#define ALIGNED16(p) ((((uintptr_t)(p)) & 15) == 0)


/* The library-owned split-K workspace of this context (grown on demand;
 * shared by every split-K product, which run in order on their streams). */
static int ws_reserve(sb_ctx *c, size_t need, CUdeviceptr *ws) {
    if (c->tc_ws_bytes < need) {
        if (c->tc_ws) cuMemFree(c->tc_ws);
        c->tc_ws = 0;
        c->tc_ws_bytes = 0;
        SB_CK(cuMemAlloc(&c->tc_ws, need));
        c->tc_ws_bytes = need;
    }
    *ws = c->tc_ws;
    return 0;
}

/* Y = the split-K partials ws[splits][total] added in split order */
static int splitk_reduce(sb_ctx *c, CUdeviceptr ws, CUdeviceptr y, long total, int splits, void *stream) {
    void *rargs[] = {&ws, &y, &total, &splits};
    const int v4 = total % 4 == 0 && (y & 15) == 0 && (ws & 15) == 0;
    long g = CEIL_DIV(v4 ? total / 4 : total, 256);
    if (g > 8L * c->sms) g = 8L * c->sms;
    return sb_launch(c, v4 ? F_SPLITK_REDUCE4 : F_SPLITK_REDUCE, (unsigned)g, 1, 256, 0, (CUstream)stream, rargs, 0);
}

/* ------------------------------------------------------------------ SGEMM */
int sb_sgemm_rows(const float *A, const float *B, float *C, int M, int N, int K, int row0, int row1,
                  void *stream) {
    SB_ARG(M >= 0 && N >= 0 && K >= 0 && 0 <= row0 && row0 <= row1 && row1 <= M, "bad SGEMM shape");
    SB_ARG(A && B && C, "null pointer");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    const int m = row1 - row0;
    if (m == 0 || N == 0) return 0;
    CUdeviceptr a = DP(A + (size_t)row0 * K), b = DP(B), cc = DP(C + (size_t)row0 * N);
    /* one CTA per 128x128 tile (two resident per SM); the kernel's tile loop
     * covers the rest if the count ever exceeds the grid limit */
    const long tiles = (long)CEIL_DIV(m, 128) * CEIL_DIV(N, 128);
    if (tiles < c->sms && m % 128 == 0 && N % 128 == 0 && K % 32 == 0 && K > 0 && ALIGNED16(A) && ALIGNED16(B) &&
        ALIGNED16(C + (size_t)row0 * N) && ALIGNED16(A + (size_t)row0 * K))
        /* fewer tiles than SMs: the TMA-staged kernel, stream-K over one CTA
         * per SM (its 4-stage ring suits the short k-ranges: 1024^3 58.4
         * against 60.4 us for the register-staged stream-K) */
        return sb_sgemm_tma(A + (size_t)row0 * K, B, C + (size_t)row0 * N, m, N, K, stream);
    if (tiles < 2L * c->sms && m % 128 == 0 && N % 128 == 0 && K % 16 == 0 && K > 0 && ALIGNED16(A) &&
        ALIGNED16(B) && ALIGNED16(C + (size_t)row0 * N) && ALIGNED16(A + (size_t)row0 * K)) {
        /* small products: stream-K -- the tiles' k-chunks cut into equal
         * ranges, two CTAs per SM; partial tiles added in CTA order */
        const long units = tiles * (K / 16);
        int G = (int)(units < 2L * c->sms ? units : 2L * c->sms);
        CUdeviceptr ws;
        int rc = ws_reserve(c, (size_t)2 * G * 128 * 128 * 4, &ws);
        if (rc) return rc;
        void *args[] = {&a, &b, &cc, &ws, (void *)&m, &N, &K};
        rc = sb_launch(c, F_SGEMM_B200_STK, (unsigned)G, 1, 256, 0, (CUstream)stream, args, 0);
        if (rc) return rc;
        int bk = 16;
        void *fargs[] = {&ws, &cc, (void *)&m, &N, &K, &G, &bk};
        return sb_launch(c, F_SGEMM_STK_FIXUP, (unsigned)(tiles * 16), 1, 256, 0, (CUstream)stream, fargs, 0);
    }
    if (m % 128 == 0 && N % 128 == 0 && K % 16 == 0 && K > 0 && ALIGNED16(A + (size_t)row0 * K) && ALIGNED16(B) &&
        ALIGNED16(C + (size_t)row0 * N)) {
        /* whole tiles: the multi-destination kernel with one output -- the
         * same arithmetic, bit for bit, and without the partial-tile path
         * in its body it keeps fewer spills (16384^3: 151.5 against 153.5 ms) */
        float *out = C + (size_t)row0 * N;
        return sb_sgemm_multi(A + (size_t)row0 * K, B, &out, 1, m, N, K, stream);
    }
    const long grid = tiles < 0x7fffffffL ? tiles : 0x7fffffffL;
    void *args[] = {&a, &b, &cc, (void *)&m, &N, &K};
    return sb_launch(c, F_SGEMM_B200, (unsigned)grid, 1, 256, 0, (CUstream)stream, args, 0);
}

int sb_sgemm(const float *A, const float *B, float *C, int M, int N, int K, void *stream) {
    return sb_sgemm_rows(A, B, C, M, N, K, 0, M, stream);
}

int sb_sgemm_multi(const float *A, const float *B, float *const *C, int nc, int M, int N, int K, void *stream) {
    SB_ARG(A && B && C && nc >= 1 && nc <= SB_SGEMM_MAX_DST, "bad multi-destination SGEMM arguments");
    SB_ARG(M >= 0 && N >= 0 && K > 0 && M % 128 == 0 && N % 128 == 0 && K % 16 == 0 && ALIGNED16(A) &&
               ALIGNED16(B),
           "multi-destination SGEMM needs M, N % 128 == 0, K % 16 == 0 and 16-byte aligned operands");
    /* the kernel's parameter block: SgDst in csrc/switch_gpu.cu */
    struct {
        CUdeviceptr c[SB_SGEMM_MAX_DST];
        int n;
    } dst;
    memset(&dst, 0, sizeof dst);
    for (int d = 0; d < nc; d++) {
        SB_ARG(C[d] && ALIGNED16(C[d]), "multi-destination SGEMM needs 16-byte aligned outputs");
        dst.c[d] = DP(C[d]);
    }
    dst.n = nc;
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (M == 0 || N == 0) return 0;
    CUdeviceptr a = DP(A), b = DP(B);
    const long tiles = (long)(M / 128) * (N / 128);
    const long grid = tiles < 0x7fffffffL ? tiles : 0x7fffffffL;
    void *args[] = {&a, &b, &dst, &M, &N, &K};
    return sb_launch(c, F_SGEMM_B200_DST, (unsigned)grid, 1, 256, 0, (CUstream)stream, args, 0);
}

/* ------------------------------------------------------------------ probes */
int sb_membw_read4(const void *buf, float *out, int n4, int iters, int grid, void *stream) {
    SB_ARG(buf && out && n4 >= 0 && iters >= 0 && ALIGNED16(buf), "bad membw arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (grid <= 0) grid = 4 * c->sms;
    CUdeviceptr b = DP(buf), o = DP(out);
    void *args[] = {&b, &o, &n4, &iters};
    return sb_launch(c, F_MEMBW, (unsigned)grid, 1, 256, 0, (CUstream)stream, args, 0);
}

int sb_fma_peak(float *out, int iters, int grid, void *stream, double *flops) {
    SB_ARG(out && iters > 0, "bad fma_peak arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (grid <= 0) grid = 8 * c->sms;
    CUdeviceptr o = DP(out);
    float m = 0.999999f, a = 1e-6f;
    void *args[] = {&o, &iters, &m, &a};
    if (flops) *flops = (double)grid * 256.0 * iters * 16.0 * 8.0 * 2.0;
    return sb_launch(c, F_FMA_PEAK, (unsigned)grid, 1, 256, 0, (CUstream)stream, args, 0);
}

/* ------------------------------------------------------------------ GEMV */
static unsigned gemv_grid(sb_ctx *c, long tasks, int warps) {
    long g = CEIL_DIV(tasks, warps);
    long cap = 4L * c->sms;
    if (g > cap) g = cap;
    return (unsigned)(g < 1 ? 1 : g);
}

int sb_gemv_f32(const float *W, const float *x, const float *bias, float *y, int K, int N, void *stream) {
    SB_ARG(W && x && y && K > 0 && N >= 0, "bad GEMV arguments");
    SB_ARG(K % 4 == 0 && ALIGNED16(W) && ALIGNED16(x), "gemv_f32 needs K % 4 == 0 and 16-byte aligned W, x");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr w = DP(W), xx = DP(x), b = DP(bias), yy = DP(y);
    void *args[] = {&w, &xx, &b, &yy, &K, &N};
    const long tasks = CEIL_DIV(N, 4);
    if (tasks < 2L * c->sms) /* short output: split-K over a CTA per four-row task */
        return sb_launch(c, F_GEMV_F32_SK, (unsigned)(tasks < 1 ? 1 : tasks), 1, 256, 0, (CUstream)stream, args, 0);
    SB_ARG((size_t)K * 4 <= 200 * 1024, "gemv_f32: K too large for the shared x stage");
    return sb_launch(c, F_GEMV_F32_B200, gemv_grid(c, CEIL_DIV(N, 4), 8), 1, 256, (unsigned)K * 4,
                     (CUstream)stream, args, 0);
}

int sb_gemv_multi_f32(const float *W, const float *X, const float *bias, float *Y, int K, int N, int T,
                      void *stream) {
    SB_ARG(W && X && Y && K > 0 && N >= 0 && T >= 0, "bad gemv_multi arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr w = DP(W), xx = DP(X), b = DP(bias), yy = DP(Y);
    void *args[] = {&w, &xx, &b, &yy, &K, &N, &T};
    return sb_launch(c, F_GEMV_MULTI, (unsigned)CEIL_DIV(N, 8), (unsigned)CEIL_DIV(T, 16), 256, 0,
                     (CUstream)stream, args, 0);
}

int sb_gemv_h(const uint16_t *W, const float *x, const float *bias, float *y, int K, int N, void *stream) {
    SB_ARG(W && x && y && K > 0 && N >= 0, "bad GEMV arguments");
    SB_ARG(K % 8 == 0 && ALIGNED16(W) && ALIGNED16(x), "gemv_h needs K % 8 == 0 and 16-byte aligned W, x");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr w = DP(W), xx = DP(x), b = DP(bias), yy = DP(y);
    void *args[] = {&w, &xx, &b, &yy, &K, &N};
    const long tasks = CEIL_DIV(N, 4);
    if (tasks < 2L * c->sms) /* short output: split-K over a CTA per four-row task */
        return sb_launch(c, F_GEMV_H_SK, (unsigned)(tasks < 1 ? 1 : tasks), 1, 256, 0, (CUstream)stream, args, 0);
    SB_ARG((size_t)K * 4 <= 200 * 1024, "gemv_h: K too large for the shared x stage");
    return sb_launch(c, F_GEMV_H_B200, gemv_grid(c, CEIL_DIV(N, 4), 8), 1, 256, (unsigned)K * 4,
                     (CUstream)stream, args, 0);
}

int sb_gemv_hh(const uint16_t *W, const uint16_t *X, float *Y, int K, int N, int B, void *stream) {
    SB_ARG(W && X && Y && K > 0 && N >= 0 && B >= 1 && B <= 8, "bad gemv_hh arguments");
    SB_ARG(K % 8 == 0 && ALIGNED16(W) && ALIGNED16(X), "gemv_hh needs K % 8 == 0 and 16-byte aligned W, X");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    /* Fewer four-row tasks than two per SM: the split-K form (a CTA per
     * task, K split over its warps); else a warp per task. */
    const long tasks = CEIL_DIV(N, 4);
    const int split_k = tasks < 2L * c->sms;
    for (int b0 = 0; b0 < B;) {
        int nb = B - b0 >= 4 ? 4 : (B - b0 >= 2 ? 2 : 1);
        CUdeviceptr w = DP(W), xx = DP(X + (size_t)b0 * K), yy = DP(Y + (size_t)b0 * N);
        void *args[] = {&w, &xx, &yy, &K, &N};
        int rc;
        if (split_k) {
            sb_fn_id f = nb == 4 ? F_GEMV_HH_SK4 : (nb == 2 ? F_GEMV_HH_SK2 : F_GEMV_HH_SK1);
            rc = sb_launch(c, f, (unsigned)(tasks < 1 ? 1 : tasks), 1, 256, 0, (CUstream)stream, args, 0);
        } else {
            SB_ARG((size_t)nb * K * 4 <= 220 * 1024, "gemv_hh: batch x K too large for the shared x stage");
            sb_fn_id f = nb == 4 ? F_GEMV_HH4 : (nb == 2 ? F_GEMV_HH2 : F_GEMV_HH1);
            rc = sb_launch(c, f, gemv_grid(c, tasks, 8), 1, 256, (unsigned)(nb * K * 4), (CUstream)stream, args, 0);
        }
        if (rc) return rc;
        b0 += nb;
    }
    return 0;
}

/* ------------------------------------------------------------------ elementwise / norms */
int sb_rmsnorm(const float *x, const uint16_t *w, float *y, int n, float eps, int rows, void *stream) {
    SB_ARG(x && w && y && n > 0 && rows >= 0, "bad rmsnorm arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr a = DP(x), b = DP(w), d = DP(y);
    void *args[] = {&a, &b, &d, &n, &eps};
    return sb_launch(c, F_RMSNORM, (unsigned)rows, 1, 256, 0, (CUstream)stream, args, 0);
}

int sb_layernorm(const float *x, const float *w, const float *b, float *y, int n, float eps, int rows,
                 void *stream) {
    SB_ARG(x && w && b && y && n > 0 && rows >= 0, "bad layernorm arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr a = DP(x), ww = DP(w), bb = DP(b), d = DP(y);
    void *args[] = {&a, &ww, &bb, &d, &n, &eps};
    return sb_launch(c, F_LAYERNORM, (unsigned)rows, 1, 256, 0, (CUstream)stream, args, 0);
}

int sb_rope(float *x, const float *cosT, const float *sinT, int T, int H, int HD, int pos0, void *stream) {
    SB_ARG(x && cosT && sinT && T >= 0 && H > 0 && HD > 0 && HD % 2 == 0 && pos0 >= 0, "bad rope arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr a = DP(x), cc = DP(cosT), s = DP(sinT);
    void *args[] = {&a, &cc, &s, &T, &H, &HD, &pos0};
    long total = (long)T * H * (HD / 2);
    return sb_launch(c, F_ROPE, (unsigned)(total ? CEIL_DIV(total, 256) : 0), 1, 256, 0, (CUstream)stream, args, 0);
}

int sb_swiglu(const float *g, const float *u, float *y, int n, void *stream) {
    SB_ARG(g && u && y && n >= 0, "bad swiglu arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr a = DP(g), b = DP(u), d = DP(y);
    void *args[] = {&a, &b, &d, &n};
    return sb_launch(c, F_SWIGLU, (unsigned)CEIL_DIV(n, 256), 1, 256, 0, (CUstream)stream, args, 0);
}

int sb_gelu(const float *x, float *y, int n, void *stream) {
    SB_ARG(x && y && n >= 0, "bad gelu arguments");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr a = DP(x), d = DP(y);
    void *args[] = {&a, &d, &n};
    return sb_launch(c, F_GELU, (unsigned)CEIL_DIV(n, 256), 1, 256, 0, (CUstream)stream, args, 0);
}

/* ------------------------------------------------------------------ attention */
int sb_attn_decode(const float *q, const float *kc, const float *vc, float *out, int T, int NH, int NKV, int HD,
                   int kv_stride, float scale, float *part, unsigned *counters, void *stream) {
    SB_ARG(q && kc && vc && out && part && counters, "null pointer");
    SB_ARG(T >= 1 && HD == 64 && NKV > 0 && NH % NKV == 0 && kv_stride >= NKV * HD && kv_stride % 2 == 0,
           "attention: need T >= 1, HD == 64, NH % NKV == 0");
    const int G = NH / NKV;
    SB_ARG(G == 1 || G == 7, "attention: NH/NKV must be 1 (MHA) or 7 (Qwen GQA)");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    int max_splits = CEIL_DIV(T, 16);
    CUdeviceptr a = DP(q), k = DP(kc), v = DP(vc), o = DP(out), p = DP(part), cn = DP(counters);
    void *args[] = {&a, &k, &v, &T, &o, &p, &cn, &kv_stride, &scale, &max_splits};
    return sb_launch(c, G == 7 ? F_ATTN_G7 : F_ATTN_G1, (unsigned)NKV, (unsigned)max_splits, 128, 0,
                     (CUstream)stream, args, 0);
}

/* ------------------------------------------------------------------ tensor-core GEMM */
static int encode_kmajor_fp16(CUtensorMap *tm, const void *base, int K, int rows, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows}, estr[2] = {1, 1};
    SB_CK(cuTensorMapEncodeTiled(tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void *)base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
    return 0;
}

int sb_gemm_hh(const uint16_t *W, const uint16_t *X, float *Y, int K, int N, int B, void *stream) {
    SB_ARG(W && X && Y && K > 0 && N >= 0 && B >= 1 && B <= 256, "bad gemm_hh arguments");
    SB_ARG(K % 8 == 0 && ALIGNED16(W) && ALIGNED16(X), "gemm_hh needs K % 8 == 0 and 16-byte aligned W, X");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (N == 0) return 0;
    /* Small batches on outputs shorter than 128 rows per SM: the tcgen05
     * kernel would split K and need a second launch; gemm_hh_mma* (mma.sync,
     * same fp16-in / FP32-accumulate semantics, subnormals kept) does it in
     * one launch, one CTA per 8 rows of W. */
    if (B <= 16 && N < 128L * c->sms) {
        /* 16 warps per CTA while the tiles are fewer than two per SM, else 4
         * (four CTAs per SM) */
        const int wide = CEIL_DIV(N, 8) < 2L * c->sms;
        const sb_fn_id f = wide ? (B > 8 ? F_GEMM_HH_MMA16 : F_GEMM_HH_MMA8)
                                : (B > 8 ? F_GEMM_HH_MMA16_W4 : F_GEMM_HH_MMA8_W4);
        CUdeviceptr w = DP(W), xx = DP(X), yy = DP(Y);
        void *args[] = {&w, &xx, &yy, &K, &N, &B};
        return sb_launch(c, f, (unsigned)CEIL_DIV(N, 8), 1, wide ? 512 : 128, 0, (CUstream)stream, args, 0);
    }
    const int n_pad = CEIL_DIV(B, 16) * 16;
    CUtensorMap tw, tx;
    int rc = encode_kmajor_fp16(&tw, W, K, N, 128);
    if (!rc) rc = encode_kmajor_fp16(&tx, X, K, B, n_pad);
    if (rc) return rc;
    /* one CTA per 128-row tile; split K when there are too few tiles to
     * occupy the SMs */
    const int tiles = CEIL_DIV(N, 128), nchunks = CEIL_DIV(K, 64);
    int splits = 1;
    if (tiles < c->sms) {
        splits = CEIL_DIV(c->sms, tiles);
        if (splits > nchunks) splits = nchunks;
    }
    CUdeviceptr y = DP(Y), ws = 0;
    if (splits > 1) {
        const size_t need = (size_t)splits * B * N * 4;
        if (c->tc_ws_bytes < need) {
            if (c->tc_ws) cuMemFree(c->tc_ws);
            c->tc_ws = 0;
            c->tc_ws_bytes = 0;
            SB_CK(cuMemAlloc(&c->tc_ws, need));
            c->tc_ws_bytes = need;
        }
        ws = c->tc_ws;
    }
    const unsigned smem = 1024 + 4 * (16384 + n_pad * 128) + 256;
    void *args[] = {&tw, &tx, &y, &ws, &N, &K, &B, (void *)&n_pad, &splits};
    rc = sb_launch(c, F_GEMM_HH_TC, (unsigned)(tiles * splits), 1, 192, smem, (CUstream)stream, args, 0);
    if (rc || splits == 1) return rc;
    long total = (long)B * N;
    return splitk_reduce(c, ws, y, total, splits, stream);
}

/* rows x K fp32, K-major, box {32 k, 128 rows}, 128-byte swizzle */
static int encode_kmajor_f32(CUtensorMap *tm, const void *base, int K, int rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows}, strides[1] = {(cuuint64_t)K * 4};
    const cuuint32_t box[2] = {32, 128}, estr[2] = {1, 1};
    SB_CK(cuTensorMapEncodeTiled(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
    return 0;
}

/* B [K][N] fp32 row-major, box {128 n, 32 k}, dense (no swizzle) */
static int encode_rowmajor_f32_b(CUtensorMap *tm, const void *base, int K, int N) {
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K}, strides[1] = {(cuuint64_t)N * 4};
    const cuuint32_t box[2] = {128, 32}, estr[2] = {1, 1};
    SB_CK(cuTensorMapEncodeTiled(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
    return 0;
}

int sb_sgemm_tma(const float *A, const float *B, float *C, int M, int N, int K, void *stream) {
    SB_ARG(M >= 0 && N >= 0 && K >= 0, "bad SGEMM shape");
    SB_ARG(A && B && C, "null pointer");
    SB_ARG(K % 4 == 0 && N % 4 == 0 && ALIGNED16(A) && ALIGNED16(B) && ALIGNED16(C),
           "sb_sgemm_tma needs K % 4 == 0, N % 4 == 0 and 16-byte aligned pointers");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (M == 0 || N == 0) return 0;
    if (K == 0) {
        for (int r = 0; r < M; r++) SB_CK(cuMemsetD32Async(DP(C + (size_t)r * N), 0, (size_t)N, (CUstream)stream));
        return 0;
    }
    CUtensorMap ta, tb;
    int rc = encode_kmajor_f32(&ta, A, K, M);
    if (!rc) rc = encode_rowmajor_f32_b(&tb, B, K, N);
    if (rc) return rc;
    const long tiles = (long)CEIL_DIV(M, 128) * CEIL_DIV(N, 128);
    const unsigned smem = 1024 + 4 * 32768 + 128;
    CUdeviceptr cc = DP(C), ws = 0;
    if (tiles < c->sms && M % 128 == 0 && N % 128 == 0 && K % 32 == 0) {
        /* stream-K over one CTA per SM; pieces added by sgemm_stk_fixup */
        const long units = tiles * (K / 32);
        int G = (int)(units < c->sms ? units : c->sms);
        rc = ws_reserve(c, (size_t)2 * G * 128 * 128 * 4, &ws);
        if (rc) return rc;
        void *args[] = {&ta, &tb, &cc, &M, &N, &K, &ws};
        rc = sb_launch(c, F_SGEMM_TMA, (unsigned)G, 1, 288, smem, (CUstream)stream, args, 0);
        if (rc) return rc;
        int bk = 32;
        void *fargs[] = {&ws, &cc, &M, &N, &K, &G, &bk};
        return sb_launch(c, F_SGEMM_STK_FIXUP, (unsigned)(tiles * 16), 1, 256, 0, (CUstream)stream, fargs, 0);
    }
    const unsigned grid = (unsigned)(tiles < c->sms ? tiles : c->sms);
    void *args[] = {&ta, &tb, &cc, &M, &N, &K, &ws};
    return sb_launch(c, F_SGEMM_TMA, grid, 1, 288, smem, (CUstream)stream, args, 0);
}

/* C = A . Bt^T with A [M][K] and Bt [N][K] both K-major (the kernel's operand form). */
static int sgemm3x_launch(sb_ctx *c, const float *A, const float *Bt, float *C, int M, int N, int K, void *stream) {
    CUtensorMap ta, tb;
    int rc = encode_kmajor_f32(&ta, A, K, M);
    if (!rc) rc = encode_kmajor_f32(&tb, Bt, K, N);
    if (rc) return rc;
    const long tiles = (long)CEIL_DIV(M, 128) * CEIL_DIV(N, 128);
    /* short or narrow products (a prompt prefill) leave SMs idle: split K
     * over several CTAs per tile, partial tiles summed in split order */
    const int nk = CEIL_DIV(K, 32);
    int splits = 1;
    if (tiles < c->sms) {
        splits = (int)CEIL_DIV(c->sms, tiles);
        if (splits > nk / 2) splits = nk / 2 > 0 ? nk / 2 : 1; /* >= 2 k-slices per CTA */
    }
    CUdeviceptr cc = DP(C), ws = 0;
    if (splits > 1) {
        const size_t need = (size_t)splits * M * N * 4;
        if (c->tc_ws_bytes < need) {
            if (c->tc_ws) cuMemFree(c->tc_ws);
            c->tc_ws = 0;
            c->tc_ws_bytes = 0;
            SB_CK(cuMemAlloc(&c->tc_ws, need));
            c->tc_ws_bytes = need;
        }
        ws = c->tc_ws;
    }
    void *args[] = {&ta, &tb, &cc, &M, &N, &K, &ws, &splits};
    const unsigned smem = 1024 + 3 * 65536 + 256;
    rc = sb_launch(c, F_SGEMM_3XTF32, (unsigned)(tiles * splits), 1, 192, smem, (CUstream)stream, args, 0);
    if (rc || splits == 1) return rc;
    long total = (long)M * N;
    return splitk_reduce(c, ws, cc, total, splits, stream);
}

int sb_sgemm_3xtf32(const float *A, const float *B, float *C, int M, int N, int K, void *stream) {
    SB_ARG(A && B && C && M >= 0 && N >= 0 && K > 0, "bad sgemm_3xtf32 arguments");
    SB_ARG(K % 4 == 0 && N % 4 == 0 && ALIGNED16(A) && ALIGNED16(B) && ALIGNED16(C),
           "sgemm_3xtf32 needs K % 4 == 0, N % 4 == 0 and 16-byte aligned A, B, C");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (M == 0 || N == 0) return 0;
    const long tiles = (long)CEIL_DIV(M, 128) * CEIL_DIV(N, 128);
    SB_ARG(tiles < 0x7fffffffL / 148, "sgemm_3xtf32: too many tiles");
    /* Bt = B^T (K-major) in a library-owned workspace, grown on demand */
    const size_t need = (size_t)K * N * 4;
    if (c->tc_bt_bytes < need) {
        if (c->tc_bt) cuMemFree(c->tc_bt);
        c->tc_bt = 0;
        c->tc_bt_bytes = 0;
        SB_CK(cuMemAlloc(&c->tc_bt, need));
        c->tc_bt_bytes = need;
    }
    CUdeviceptr bsrc = DP(B), bt = c->tc_bt;
    void *targs[] = {&bsrc, &bt, &K, &N};
    int rc = sb_launch(c, F_TRANSPOSE_F32, (unsigned)CEIL_DIV(N, 32), (unsigned)CEIL_DIV(K, 32), 32 * 8, 0,
                       (CUstream)stream, targs, 0);
    if (rc) return rc;
    return sgemm3x_launch(c, A, (const float *)(uintptr_t)bt, C, M, N, K, stream);
}

int sb_sgemm_3xtf32_multi(const float *A, const float *B, float *const *C, int nc, int M, int N, int K,
                          void *stream) {
    SB_ARG(A && B && C && nc >= 1 && nc <= SB_SGEMM_MAX_DST, "bad multi-destination sgemm_3xtf32 arguments");
    SB_ARG(M >= 0 && N >= 0 && K > 0 && M % 128 == 0 && N % 128 == 0 && K % 4 == 0 && ALIGNED16(A) && ALIGNED16(B),
           "multi-destination sgemm_3xtf32 needs M, N % 128 == 0, K % 4 == 0 and 16-byte aligned operands");
    /* the kernel's parameter block: T3Dst in csrc/tc_kernels.cu */
    struct {
        CUdeviceptr c[SB_SGEMM_MAX_DST];
        int n;
    } dst;
    memset(&dst, 0, sizeof dst);
    for (int d = 0; d < nc; d++) {
        SB_ARG(C[d] && ALIGNED16(C[d]), "multi-destination sgemm_3xtf32 needs 16-byte aligned outputs");
        dst.c[d] = DP(C[d]);
    }
    dst.n = nc;
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (M == 0 || N == 0) return 0;
    const long tiles = (long)(M / 128) * (N / 128);
    SB_ARG(tiles < 0x7fffffffL, "multi-destination sgemm_3xtf32: too many tiles");
    const size_t need = (size_t)K * N * 4; /* Bt = B^T in the library-owned workspace */
    if (c->tc_bt_bytes < need) {
        if (c->tc_bt) cuMemFree(c->tc_bt);
        c->tc_bt = 0;
        c->tc_bt_bytes = 0;
        SB_CK(cuMemAlloc(&c->tc_bt, need));
        c->tc_bt_bytes = need;
    }
    CUdeviceptr bsrc = DP(B), bt = c->tc_bt;
    void *targs[] = {&bsrc, &bt, &K, &N};
    int rc = sb_launch(c, F_TRANSPOSE_F32, (unsigned)CEIL_DIV(N, 32), (unsigned)CEIL_DIV(K, 32), 32 * 8, 0,
                       (CUstream)stream, targs, 0);
    if (rc) return rc;
    CUtensorMap ta, tb;
    rc = encode_kmajor_f32(&ta, A, K, M);
    if (!rc) rc = encode_kmajor_f32(&tb, (const float *)(uintptr_t)bt, K, N);
    if (rc) return rc;
    void *args[] = {&ta, &tb, &dst, &M, &N, &K};
    const unsigned smem = 1024 + 3 * 65536 + 256;
    return sb_launch(c, F_SGEMM_3XTF32_DST, (unsigned)tiles, 1, 192, smem, (CUstream)stream, args, 0);
}

int sb_sgemm_nt_3xtf32(const float *A, const float *Bt, float *C, int M, int N, int K, void *stream) {
    SB_ARG(A && Bt && C && M >= 0 && N >= 0 && K > 0, "bad sgemm_nt_3xtf32 arguments");
    SB_ARG(K % 4 == 0 && N % 4 == 0 && ALIGNED16(A) && ALIGNED16(Bt) && ALIGNED16(C),
           "sgemm_nt_3xtf32 needs K % 4 == 0, N % 4 == 0 and 16-byte aligned A, Bt, C");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    if (M == 0 || N == 0) return 0;
    SB_ARG((long)CEIL_DIV(M, 128) * CEIL_DIV(N, 128) < 0x7fffffffL / 148, "sgemm_nt_3xtf32: too many tiles");
    return sgemm3x_launch(c, A, Bt, C, M, N, K, stream);
}

int sb_tc_set_test_skip(int chunk) {
    SB_ARG(chunk >= -1, "chunk must be >= -1");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr p;
    size_t bytes;
    SB_CK(cuCtxSynchronize());
    SB_CK(cuModuleGetGlobal(&p, &bytes, c->mod[M_TC], "tc_test_skip"));
    SB_CK(cuMemsetD32(p, (unsigned)(chunk + 1), 1));
    return 0;
}

int sb_tc_error(int *err) {
    SB_ARG(err, "null pointer");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr p;
    size_t bytes;
    SB_CK(cuCtxSynchronize());
    SB_CK(cuModuleGetGlobal(&p, &bytes, c->mod[M_TC], "tc_err"));
    SB_CK(cuMemcpyDtoH(err, p, 4));
    if (*err) SB_CK(cuMemsetD32(p, 0, 1));
    return 0;
}

/* ---------------------------------------------------------- token selection */
int sb_topk_penalized(const float *logits, int V, const int *ctx, int ctx_len, float temperature, float rep_penalty,
                      int top_k, int *idx_out, float *val_out, void *stream) {
    SB_ARG(logits && V > 0 && ctx_len >= 0 && (ctx || ctx_len == 0) && idx_out && val_out, "bad top-k arguments");
    SB_ARG(top_k >= 1 && top_k <= 64 && temperature > 0.0f && rep_penalty > 0.0f, "bad top-k settings");
    const long G = CEIL_DIV(V, 1024);
    SB_ARG(G * top_k <= 16384 && V <= (1 << 18), "V > 2^18, or ceil(V / 1024) x top_k exceeds 16384 candidates");
    sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    CUdeviceptr ws;
    int rc = ws_reserve(c, (size_t)G * top_k * 8, &ws);
    if (rc) return rc;
    CUdeviceptr lg = DP(logits), cx = DP(ctx), ci = ws, cv = ws + (size_t)G * top_k * 4;
    void *args[] = {&lg, &V, &cx, &ctx_len, &temperature, &rep_penalty, &top_k, &ci, &cv};
    rc = sb_launch(c, F_TOPK_PARTIAL, (unsigned)G, 1, 256, 0, (CUstream)stream, args, 0);
    if (rc) return rc;
    int ncand = (int)(G * top_k);
    CUdeviceptr oi = DP(idx_out), ov = DP(val_out);
    void *margs[] = {&ci, &cv, &ncand, &top_k, &oi, &ov};
    return sb_launch(c, F_TOPK_MERGE, 1, 1, 1024, 0, (CUstream)stream, margs, 0);
}

