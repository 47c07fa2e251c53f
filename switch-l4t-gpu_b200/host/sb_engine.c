/* sb_engine.c -- the decode engines (Qwen2.5-0.5B FP16 weights, GPT-2 124M
 * FP32) on the driver API.
 *
 * Compared with the reference's gpu_forward (qwen_engine.c:205-269,
 * gpt2_engine.c:174-264), which issues ~390 / ~218 driver calls per token,
 * uploads the embedding row from the host, copies all V logits back and
 * takes the argmax on the host, one step here is 1 + 5 per layer + 2 fused
 * kernels that read the step position from device memory (SbStep).  The
 * step is captured once as a CUDA graph (one with the LM head + argmax, one
 * without for prompt tokens) and replayed per token; kernels are chained
 * with programmatic dependent launch so each one's weight prefetch overlaps
 * the previous one's tail.
 *
 * Device memory: the weight file is uploaded verbatim as one allocation and
 * tensors are addressed at the reference's fixed offsets; KV cache FP32
 * [2][layers][max_ctx][kv_width]; activations, logits, attention scratch,
 * token ids and the SbStep are one further allocation.
 */
#define _GNU_SOURCE
#include <limits.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include "../csrc/sb_mk_params.h"
#include "../csrc/sb_step.h"
#include "sb_internal.h"
#include "sb_models.h"

#define CEIL_DIV(a, b) (((a) + (b)-1) / (b))

struct sb_engine {
    int model;
    int ctx_cap;
    unsigned flags;
    sb_ctx *c;
    CUstream stream;
    CUdeviceptr w;  /* weight file image */
    size_t wbytes;
    CUdeviceptr kv; /* [2][NL][ctx][kvw] */
    CUdeviceptr scratch;
    CUdeviceptr x, q, att, hid, logits, part, counters, step, tokens;
    CUdeviceptr tk; /* sampler candidates: 64 ids then 64 values */
    int max_splits;
    int V, NL, kvw;
    CUgraphExec gexec[2];
    int n_prompt, n_end;
    /* persistent whole-step kernel (qwen_decode_mk2 / qwen_decode_mk / gpt2_decode_mk) */
    int mk, mk2;
    CUdeviceptr wdt; /* mk2: W_down transposed per layer [NL][FC][C] fp16 */
    size_t ll_words;
    CUdeviceptr ll, sync, err; /* flagged exchange words; u32[2] seq / arrivals; error flag */
    int mk_splits, mk_score_cap;
    unsigned mk_smem;
    long mk_steps; /* launches since the flagged words were last cleared */
    CUdeviceptr trace;
    int test_stall; /* sb_engine_set_test_stall */
    /* batched prompt prefill: activations of up to PF_T tokens */
    CUdeviceptr pf_x, pf_xh, pf_y, pf_q, pf_att, pf_a;
    SbStep st_begin; /* the step state sb_engine_begin wrote */
};

#define MK_THREADS 512
#define MK_WARPS 16
static unsigned mk_smem_bytes(int model, int score_cap) {
    /* Qwen: x planes (FC floats) | 16 warp regions of (6 rows + 1/2 row) of 896 fp16
     * GPT-2: x (FC floats) | 16 warp regions of (3 rows + 1/2 row) of 768 fp32
     * both: | scores | red(32) opart(16x64) ksum(16) (m, l) of NH x SPLITS_MAX partials
     * Qwen: | fp16 hi / lo activation vectors (C halves each) */
    const unsigned head = model == SB_MODEL_QWEN ? QW_FC * 4 + MK_WARPS * (6 * QW_C * 2 + QW_C)
                                                 : G2_FC * 4 + MK_WARPS * (3 * G2_C * 4 + G2_C * 2);
    const unsigned hl = model == SB_MODEL_QWEN ? QW_C * 4 : 0; /* fp16 hi / lo activation vectors */
    return head + (unsigned)score_cap * 4 + (32 + MK_WARPS * 64 + MK_WARPS + QW_NH * SB_MK_SPLITS_MAX * 2) * 4 + hl;
}

/* qwen_decode_mk2: warp regions of 5 rows + an O half-row, the CTA's W_downT
 * rows (ceil(FC / CTAs) of them), scores, the attention scratch and the fp16
 * hi / lo activation vectors */
static unsigned mk2_smem_bytes(int score_cap, int ctas) {
    const unsigned dsmax = (unsigned)CEIL_DIV(QW_FC, ctas);
    return MK_WARPS * (5 * QW_C * 2 + QW_C) + dsmax * QW_C * 2 + (unsigned)((score_cap + 3) & ~3) * 4 +
           (32 + MK_WARPS * 64 + MK_WARPS + QW_NH * SB_MK_SPLITS_MAX * 2) * 4 + QW_C * 4;
}

/* ------------------------------------------------------------------ upload */
static int upload_file(sb_engine *e, const char *path, size_t want) {
    FILE *f = fopen(path, "rb");
    if (!f) return sb_fail(SB_ERR_FILE, "cannot open weight file", __FILE__, __LINE__);
    struct stat st;
    if (fstat(fileno(f), &st) != 0 || (size_t)st.st_size != want) {
        fclose(f);
        return sb_fail(SB_ERR_FILE, "weight file has the wrong size for this model", __FILE__, __LINE__);
    }
    const size_t CH = 64u << 20;
    void *buf[2] = {NULL, NULL};
    CUevent ev[2] = {NULL, NULL};
    int rc = 0;
    if (cuMemAllocHost(&buf[0], CH) || cuMemAllocHost(&buf[1], CH) || cuEventCreate(&ev[0], 0) ||
        cuEventCreate(&ev[1], 0)) {
        rc = sb_fail(SB_ERR_STATE, "pinned staging allocation failed", __FILE__, __LINE__);
        goto out;
    }
    for (size_t off = 0, i = 0; off < want; off += CH, i++) {
        const size_t n = want - off < CH ? want - off : CH;
        const int k = (int)(i & 1);
        if (i >= 2 && cuEventSynchronize(ev[k])) { rc = sb_fail(SB_ERR_STATE, "upload sync", __FILE__, __LINE__); goto out; }
        if (fread(buf[k], 1, n, f) != n) { rc = sb_fail(SB_ERR_FILE, "short read of weight file", __FILE__, __LINE__); goto out; }
        CUresult r = cuMemcpyHtoDAsync(e->w + off, buf[k], n, e->stream);
        if (r == CUDA_SUCCESS) r = cuEventRecord(ev[k], e->stream);
        if (r != CUDA_SUCCESS) { rc = sb_fail((int)r, "weight upload", __FILE__, __LINE__); goto out; }
    }
    if (cuStreamSynchronize(e->stream)) rc = sb_fail(SB_ERR_STATE, "upload sync", __FILE__, __LINE__);
out:
    cuStreamSynchronize(e->stream);
    for (int k = 0; k < 2; k++) {
        if (buf[k]) cuMemFreeHost(buf[k]);
        if (ev[k]) cuEventDestroy(ev[k]);
    }
    fclose(f);
    return rc;
}

/* ------------------------------------------------------------------ step recording */
static int pdl_on(const sb_engine *e) { return !(e->flags & SB_FLAG_NO_PDL); }

/* One kernel of a decode step: which = SBK_* for layer l. */
enum { SBK_EMBED = 0, SBK_QKV, SBK_ATTN, SBK_O, SBK_MLP_UP, SBK_MLP_DOWN, SBK_LMHEAD, SBK_FINALIZE, SBK_COUNT };

static int launch_qwen(sb_engine *e, int l, int which, int with_logits, int pdl) {
    sb_ctx *c = e->c;
    CUstream s = e->stream;
    int C = QW_C, NH = QW_NH, NKV = QW_NKV, HD = QW_HD, FC = QW_FC, V = QW_V, KVD = QW_KVD;
    float eps = 1e-6f, scale = 0.125f;
    CUdeviceptr emb = e->w, cosT = e->w + QW_OFF_COS, sinT = e->w + QW_OFF_SIN;
    CUdeviceptr lb = e->w + QW_LBASE + (size_t)l * QW_LSTRIDE;
    CUdeviceptr g_in = lb + QWL_INLN * 2, wqkv = lb + QWL_QKVW * 2, bqkv = lb + QWL_QKVB * 2;
    CUdeviceptr wo = lb + QWL_OW * 2, g_post = lb + QWL_POST * 2, wgu = lb + QWL_GATEUP * 2;
    CUdeviceptr wd = lb + QWL_DOWN * 2;
    CUdeviceptr kc = e->kv + (size_t)l * e->ctx_cap * KVD * 4;
    CUdeviceptr vc = e->kv + (size_t)(QW_NL + l) * e->ctx_cap * KVD * 4;
    switch (which) {
    case SBK_EMBED: {
        void *a[] = {&emb, &e->tokens, &e->step, &e->x, &C};
        return sb_launch(c, F_QWEN_EMBED, 1, 1, 256, 0, s, a, pdl);
    }
    case SBK_QKV: { /* 576 RoPE-pair tasks: 4 per CTA of 4 warps */
        void *a[] = {&wqkv, &bqkv, &g_in, &e->x, &cosT, &sinT, &e->step, &e->q, &kc, &vc, &C, &NH, &NKV, &HD, &eps};
        return sb_launch(c, F_QWEN_QKV, QW_QKV / 2 / 4, 1, 128, C * 4, s, a, pdl);
    }
    case SBK_ATTN: {
        void *a[] = {&e->q, &kc, &vc, &e->step, &e->att, &e->part, &e->counters, &KVD, &scale, &e->max_splits};
        return sb_launch(c, F_QWEN_ATTN, NKV, e->max_splits, 128, 0, s, a, pdl);
    }
    case SBK_O: { /* 8 warps, 2 per row: 4 rows per CTA */
        int K = C, N = C, ks = 2;
        void *a[] = {&wo, &e->att, &e->step, &e->x, &K, &N, &ks};
        return sb_launch(c, F_QWEN_RESID, N / (8 / ks), 1, 256, 0, s, a, pdl);
    }
    case SBK_MLP_UP: { /* 2432 (gate,up) row-pair tasks: 8 per CTA of 4 warps */
        void *a[] = {&wgu, &g_post, &e->x, &e->step, &e->hid, &C, &FC, &eps};
        return sb_launch(c, F_QWEN_GATEUP, CEIL_DIV(FC / 2, 8), 1, 128, C * 4, s, a, pdl);
    }
    case SBK_MLP_DOWN: { /* 8 warps, 4 per row: 2 rows per CTA */
        int K = FC, N = C, ks = 4;
        void *a[] = {&wd, &e->hid, &e->step, &e->x, &K, &N, &ks};
        return sb_launch(c, F_QWEN_RESID, N / (8 / ks), 1, 256, 0, s, a, pdl);
    }
    case SBK_LMHEAD: {
        CUdeviceptr g_f = e->w + QW_OFF_LNF;
        void *a[] = {&emb, &g_f, &e->x, &e->step, &e->logits, &C, &V, &eps};
        return sb_launch(c, F_QWEN_LMHEAD, 2 * c->sms, 1, 256, C * 4, s, a, pdl);
    }
    case SBK_FINALIZE: {
        int wl = with_logits;
        void *a[] = {&e->step, &e->tokens, &wl};
        return sb_launch(c, F_QWEN_FINALIZE, 1, 1, 32, 0, s, a, pdl);
    }
    }
    return sb_fail(SB_ERR_ARG, "unknown step kernel", __FILE__, __LINE__);
}

static int launch_gpt2(sb_engine *e, int l, int which, int with_logits, int pdl) {
    sb_ctx *c = e->c;
    CUstream s = e->stream;
    int C = G2_C, FC = G2_FC, V = G2_V;
    float eps = 1e-5f, scale = 0.125f;
    CUdeviceptr wte = e->w, wpe = e->w + G2_OFF_WPE * 4;
    CUdeviceptr lb = e->w + (G2_LBASE + (size_t)l * G2_LAYER) * 4;
    CUdeviceptr ln1w = lb + G2L_LN1W * 4, ln1b = lb + G2L_LN1B * 4, wqkv = lb + G2L_QKVW * 4;
    CUdeviceptr bqkv = lb + G2L_QKVB * 4, wo = lb + G2L_AOW * 4, bo = lb + G2L_AOB * 4;
    CUdeviceptr ln2w = lb + G2L_LN2W * 4, ln2b = lb + G2L_LN2B * 4, wfc = lb + G2L_FCW * 4;
    CUdeviceptr bfc = lb + G2L_FCB * 4, wp = lb + G2L_PROJW * 4, bp = lb + G2L_PROJB * 4;
    CUdeviceptr kc = e->kv + (size_t)l * e->ctx_cap * C * 4;
    CUdeviceptr vc = e->kv + (size_t)(G2_NL + l) * e->ctx_cap * C * 4;
    switch (which) {
    case SBK_EMBED: {
        void *a[] = {&wte, &wpe, &e->tokens, &e->step, &e->x, &C};
        return sb_launch(c, F_GPT2_EMBED, 1, 1, 256, 0, s, a, pdl);
    }
    case SBK_QKV: { /* 1152 two-row tasks: 4 per CTA of 4 warps */
        void *a[] = {&wqkv, &bqkv, &ln1w, &ln1b, &e->x, &e->step, &e->q, &kc, &vc, &C, &eps};
        return sb_launch(c, F_GPT2_LN_QKV, 3 * C / 2 / 4, 1, 128, C * 4, s, a, pdl);
    }
    case SBK_ATTN: {
        void *a[] = {&e->q, &kc, &vc, &e->step, &e->att, &e->part, &e->counters, &C, &scale, &e->max_splits};
        return sb_launch(c, F_GPT2_ATTN, G2_NH, e->max_splits, 128, 0, s, a, pdl);
    }
    case SBK_O: {
        int K = C, N = C, ks = 2;
        void *a[] = {&wo, &bo, &e->att, &e->step, &e->x, &K, &N, &ks};
        return sb_launch(c, F_GPT2_RESID, N / (8 / ks), 1, 256, 0, s, a, pdl);
    }
    case SBK_MLP_UP: { /* 768 four-row tasks: 4 per CTA of 4 warps */
        void *a[] = {&wfc, &bfc, &ln2w, &ln2b, &e->x, &e->step, &e->hid, &C, &FC, &eps};
        return sb_launch(c, F_GPT2_LN_FC, FC / 4 / 4, 1, 128, C * 4, s, a, pdl);
    }
    case SBK_MLP_DOWN: {
        int K = FC, N = C, ks = 4;
        void *a[] = {&wp, &bp, &e->hid, &e->step, &e->x, &K, &N, &ks};
        return sb_launch(c, F_GPT2_RESID, N / (8 / ks), 1, 256, 0, s, a, pdl);
    }
    case SBK_LMHEAD: {
        CUdeviceptr lnfw = e->w + G2_OFF_LNFW * 4, lnfb = e->w + G2_OFF_LNFB * 4;
        void *a[] = {&wte, &lnfw, &lnfb, &e->x, &e->step, &e->logits, &C, &V, &eps};
        return sb_launch(c, F_GPT2_LMHEAD, 2 * c->sms, 1, 256, C * 4, s, a, pdl);
    }
    case SBK_FINALIZE: {
        int wl = with_logits;
        void *a[] = {&e->step, &e->tokens, &wl};
        return sb_launch(c, F_GPT2_FINALIZE, 1, 1, 32, 0, s, a, pdl);
    }
    }
    return sb_fail(SB_ERR_ARG, "unknown step kernel", __FILE__, __LINE__);
}

static int launch_kernel(sb_engine *e, int l, int which, int with_logits, int pdl) {
    return e->model == SB_MODEL_QWEN ? launch_qwen(e, l, which, with_logits, pdl)
                                     : launch_gpt2(e, l, which, with_logits, pdl);
}

static int mk_fn(int model, int v2) { return model == SB_MODEL_QWEN ? (v2 ? F_QWEN_MK2 : F_QWEN_MK) : F_GPT2_MK; }

static int record_mk(sb_engine *e, int with_logits) {
    SbMkParams prm;
    memset(&prm, 0, sizeof prm);
    prm.w = e->w;
    prm.kv = e->kv;
    prm.ll = e->ll;
    prm.logits = e->logits;
    prm.st = e->step;
    prm.tokens = e->tokens;
    prm.sync = e->sync;
    prm.err = e->err;
    prm.trace = e->trace;
    prm.ctx_cap = e->ctx_cap;
    prm.with_logits = with_logits;
    prm.splits = e->mk_splits;
    prm.score_cap = e->mk_score_cap;
    prm.test_stall = e->test_stall;
    prm.aux = e->wdt;
    void *args[] = {&prm};
    return sb_launch_coop(e->c, mk_fn(e->model, e->mk2), (unsigned)e->c->sms, MK_THREADS, e->mk_smem, e->stream,
                          args);
}

static int record_model(sb_engine *e, int with_logits) {
    if (e->mk) return record_mk(e, with_logits);
    const int pdl = pdl_on(e);
    int rc = launch_kernel(e, 0, SBK_EMBED, with_logits, pdl);
    for (int l = 0; !rc && l < e->NL; l++)
        for (int k = SBK_QKV; !rc && k <= SBK_MLP_DOWN; k++) rc = launch_kernel(e, l, k, with_logits, pdl);
    if (!rc && with_logits) rc = launch_kernel(e, 0, SBK_LMHEAD, with_logits, pdl);
    if (!rc) rc = launch_kernel(e, 0, SBK_FINALIZE, with_logits, pdl);
    return rc;
}

static int record_step(sb_engine *e, int with_logits) { return record_model(e, with_logits); }

static int ensure_graph(sb_engine *e, int with_logits) {
    if (e->flags & SB_FLAG_NO_GRAPH) return 0;
    if (e->gexec[with_logits]) return 0;
    SB_CK(cuStreamBeginCapture(e->stream, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL));
    int rc = record_step(e, with_logits);
    CUgraph g = NULL;
    CUresult r = cuStreamEndCapture(e->stream, &g);
    if (rc) {
        if (g) cuGraphDestroy(g);
        return rc;
    }
    if (r != CUDA_SUCCESS) return sb_fail((int)r, "cuStreamEndCapture", __FILE__, __LINE__);
    r = cuGraphInstantiate(&e->gexec[with_logits], g, 0);
    cuGraphDestroy(g);
    if (r != CUDA_SUCCESS) return sb_fail((int)r, "cuGraphInstantiate", __FILE__, __LINE__);
    return 0;
}

static int run_step(sb_engine *e, int with_logits) {
    e->mk_steps++;
    if (e->flags & SB_FLAG_NO_GRAPH) return record_step(e, with_logits);
    int rc = ensure_graph(e, with_logits);
    if (rc) return rc;
    SB_CK(cuGraphLaunch(e->gexec[with_logits], e->stream));
    return 0;
}

/* ------------------------------------------------------------------ lifecycle */
sb_engine *sb_engine_create(int model, const char *weights_path, int max_ctx, unsigned flags) {
    if (model != SB_MODEL_QWEN && model != SB_MODEL_GPT2) {
        sb_fail(SB_ERR_ARG, "unknown model id", __FILE__, __LINE__);
        return NULL;
    }
    const int file_ctx = model == SB_MODEL_QWEN ? QW_CTX_FILE : G2_CTX;
    if (max_ctx <= 0 || max_ctx > file_ctx) {
        sb_fail(SB_ERR_ARG, "max_ctx out of range for this model", __FILE__, __LINE__);
        return NULL;
    }
    sb_ctx *c = sb_ctx_get();
    if (!c) return NULL;
    sb_engine *e = calloc(1, sizeof *e);
    e->model = model;
    e->ctx_cap = max_ctx;
    e->flags = flags;
    e->c = c;
    const int qw = model == SB_MODEL_QWEN;
    e->V = qw ? QW_V : G2_V;
    e->NL = qw ? QW_NL : G2_NL;
    e->kvw = qw ? QW_KVD : G2_C;
    e->wbytes = qw ? QW_FILE_BYTES : (size_t)G2_TOTAL_FLOATS * 4;
    e->max_splits = CEIL_DIV(max_ctx, 16);
    /* the persistent kernel needs >= 128 co-resident CTAs (its per-CTA row
     * shares are sized for that) and cooperative launch */
    if (!(flags & SB_FLAG_MULTI_KERNEL) && c->sms >= 128) {
        e->mk_splits = c->sms / (model == SB_MODEL_QWEN ? QW_NH : G2_NH);
        if (e->mk_splits > SB_MK_SPLITS_MAX) e->mk_splits = SB_MK_SPLITS_MAX;
        e->mk_score_cap = (CEIL_DIV(max_ctx, e->mk_splits) + 8 + 3) & ~3; /* multiple of 4 floats */
        int coop = 0;
        cuDeviceGetAttribute(&coop, CU_DEVICE_ATTRIBUTE_COOPERATIVE_LAUNCH, c->dev);
        /* Qwen: the split-K kernel unless asked for the earlier one (or it does not fit) */
        if (model == SB_MODEL_QWEN && !(flags & SB_FLAG_MK_V1) && c->sms <= 160) {
            e->mk_smem = mk2_smem_bytes(e->mk_score_cap, c->sms);
            e->mk2 = coop && sb_occupancy(c, F_QWEN_MK2, MK_THREADS, e->mk_smem) >= 1;
        }
        if (!e->mk2) e->mk_smem = mk_smem_bytes(model, e->mk_score_cap);
        e->mk = e->mk2 || (coop && sb_occupancy(c, mk_fn(model, 0), MK_THREADS, e->mk_smem) >= 1);
    }
    e->ll_words = e->mk2 ? (size_t)SB_MK2_LL_WORDS(c->sms) : (size_t)SB_MK_LL_WORDS;
    const int groups = qw ? QW_NKV : G2_NH, G = qw ? QW_NH / QW_NKV : 1;
    const int C = qw ? QW_C : G2_C, FC = qw ? QW_FC : G2_FC, NQ = qw ? QW_C : G2_C;

    if (cuStreamCreate(&e->stream, CU_STREAM_NON_BLOCKING)) { sb_fail(SB_ERR_STATE, "stream", __FILE__, __LINE__); goto fail; }
    if (cuMemAlloc(&e->w, e->wbytes)) { sb_fail(SB_ERR_STATE, "weight allocation", __FILE__, __LINE__); goto fail; }
    if (upload_file(e, weights_path, e->wbytes)) goto fail;
    if (qw) {
        /* fp16 regions (embedding; layers + final norm) -- not the fp32 RoPE
         * tables between them: subnormals -> 0 once, as the reference decodes */
        const size_t regions[2][2] = {{0, QW_OFF_COS}, {QW_LBASE, QW_FILE_BYTES}};
        for (int k = 0; k < 2; k++) {
            CUdeviceptr base = e->w + regions[k][0];
            long n16 = (long)((regions[k][1] - regions[k][0]) / 16);
            void *a[] = {&base, &n16};
            if (sb_launch(c, F_FP16_FLUSH, 4 * c->sms, 1, 256, 0, e->stream, a, 0)) goto fail;
        }
        if (cuStreamSynchronize(e->stream)) { sb_fail(SB_ERR_STATE, "weight flush", __FILE__, __LINE__); goto fail; }
        if (e->mk2) { /* W_downT [layer][FC][C]: W_down [C][FC] of every layer, transposed (flushed above) */
            const size_t bytes = (size_t)QW_NL * QW_FC * QW_C * 2;
            if (cuMemAlloc(&e->wdt, bytes)) { sb_fail(SB_ERR_STATE, "W_downT allocation", __FILE__, __LINE__); goto fail; }
            CUdeviceptr src = e->w + QW_LBASE + QWL_DOWN * 2, dst = e->wdt;
            int rows = QW_C, cols = QW_FC;
            long in_stride = (long)(QW_LSTRIDE / 2), out_stride = (long)QW_FC * QW_C;
            void *a[] = {&src, &dst, &rows, &cols, &in_stride, &out_stride};
            CUstream s = e->stream;
            if (sb_launch3(c, F_TRANSPOSE_U16, CEIL_DIV(QW_FC, 32), CEIL_DIV(QW_C, 32), QW_NL, 256, s, a) ||
                cuStreamSynchronize(s)) {
                sb_fail(SB_ERR_STATE, "W_downT transpose", __FILE__, __LINE__);
                goto fail;
            }
        }
    }
    const size_t kv_bytes = (size_t)2 * e->NL * max_ctx * e->kvw * 4;
    if (cuMemAlloc(&e->kv, kv_bytes)) { sb_fail(SB_ERR_STATE, "KV allocation", __FILE__, __LINE__); goto fail; }
    /* scratch: x[C] q[NQ] att[NQ] hid[FC] logits[V] part counters step tokens */
    size_t off = 0;
#define CARVE(field, bytes) do { e->field = (CUdeviceptr)off; off += ((size_t)(bytes) + 255) & ~(size_t)255; } while (0)
    CARVE(x, C * 4);
    CARVE(q, NQ * 4);
    CARVE(att, NQ * 4);
    CARVE(hid, FC * 4);
    CARVE(logits, (size_t)e->V * 4);
    {
        size_t pf = (size_t)groups * e->max_splits * G * 66;
        size_t pm = (size_t)QW_NH * (e->mk_splits > 0 ? e->mk_splits : 1) * 66;
        CARVE(part, (pf > pm ? pf : pm) * 4);
    }
    CARVE(counters, groups * 4);
    CARVE(step, sizeof(SbStep));
    CARVE(tokens, (size_t)(max_ctx + 2) * 4);
    CARVE(ll, e->ll_words * 8);
    CARVE(sync, 8);
    CARVE(err, 4);
    CARVE(tk, 64 * 8);
#undef CARVE
    if (cuMemAlloc(&e->scratch, off)) { sb_fail(SB_ERR_STATE, "scratch allocation", __FILE__, __LINE__); goto fail; }
    e->x += e->scratch; e->q += e->scratch; e->att += e->scratch; e->hid += e->scratch;
    e->logits += e->scratch; e->part += e->scratch; e->counters += e->scratch; e->step += e->scratch;
    e->tokens += e->scratch;
    e->ll += e->scratch;
    e->sync += e->scratch;
    e->err += e->scratch;
    e->tk += e->scratch;
    if (cuMemsetD8Async(e->scratch, 0, off, e->stream) || cuMemsetD8Async(e->kv, 0, kv_bytes, e->stream) ||
        cuStreamSynchronize(e->stream)) {
        sb_fail(SB_ERR_STATE, "initialisation", __FILE__, __LINE__);
        goto fail;
    }
    return e;
fail:
    sb_engine_destroy(e);
    return NULL;
}

void sb_engine_destroy(sb_engine *e) {
    if (!e) return;
    if (e->stream) cuStreamSynchronize(e->stream);
    CUdeviceptr pf[] = {e->pf_x, e->pf_xh, e->pf_y, e->pf_q, e->pf_att, e->pf_a};
    for (int i = 0; i < 6; i++)
        if (pf[i]) cuMemFree(pf[i]);
    for (int i = 0; i < 2; i++)
        if (e->gexec[i]) cuGraphExecDestroy(e->gexec[i]);
    if (e->scratch) cuMemFree(e->scratch);
    if (e->wdt) cuMemFree(e->wdt);
    if (e->kv) cuMemFree(e->kv);
    if (e->w) cuMemFree(e->w);
    if (e->stream) cuStreamDestroy(e->stream);
    free(e);
}

int sb_engine_reset(sb_engine *e) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_CK(cuMemsetD8Async(e->kv, 0, (size_t)2 * e->NL * e->ctx_cap * e->kvw * 4, e->stream));
    SB_CK(cuStreamSynchronize(e->stream));
    return 0;
}

void *sb_engine_stream(sb_engine *e) { return e ? (void *)e->stream : NULL; }

int sb_engine_logits(sb_engine *e, const float **dev_logits, int *vocab) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    if (dev_logits) *dev_logits = (const float *)(uintptr_t)e->logits;
    if (vocab) *vocab = e->V;
    return 0;
}

int sb_engine_kv_cache(sb_engine *e, void **dev_kv, size_t *bytes, int *layers, int *max_ctx, int *width) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    if (dev_kv) *dev_kv = (void *)(uintptr_t)e->kv;
    if (bytes) *bytes = (size_t)2 * e->NL * e->ctx_cap * e->kvw * 4;
    if (layers) *layers = e->NL;
    if (max_ctx) *max_ctx = e->ctx_cap;
    if (width) *width = e->kvw;
    return 0;
}

int sb_engine_launches_per_step(sb_engine *e, int with_logits) {
    if (!e) return 0;
    if (e->mk) return 1;
    return 1 + 5 * e->NL + (with_logits ? 1 : 0) + 1;
}

double sb_engine_step_bytes(sb_engine *e) {
    if (!e) return 0;
    if (e->model == SB_MODEL_QWEN) {
        /* every layer matrix + the tied LM head (embedding) */
        double layer = ((double)QW_QKV * QW_C + (double)QW_C * QW_C + 2.0 * QW_FC * QW_C + (double)QW_C * QW_FC) * 2;
        return QW_NL * layer + (double)QW_V * QW_C * 2;
    }
    double layer = ((double)3 * G2_C * G2_C + (double)G2_C * G2_C + 2.0 * G2_FC * G2_C) * 4;
    return G2_NL * layer + (double)G2_V * G2_C * 4;
}

/* ------------------------------------------------------------------ stepping */
/* A persistent-kernel barrier that timed out leaves *err set (the kernel
 * returned early instead of hanging); report it and clear the flag. */
/* Clear the flagged words and the sequence number (epoch 0 never matches). */
static int mk_clear_words(sb_engine *e) {
    SB_CK(cuMemsetD8Async(e->ll, 0, e->ll_words * 8, e->stream));
    SB_CK(cuMemsetD32Async(e->sync, 0, 2, e->stream));
    e->mk_steps = 0;
    return 0;
}

/* A persistent-kernel wait that timed out leaves *err set (the kernel
 * returned early instead of hanging); report it, and reset the exchange
 * words so the aborted step's stale words cannot match a later epoch. */
static int check_device_error(sb_engine *e) {
    if (!e->mk) return 0;
    int err = 0;
    SB_CK(cuMemcpyDtoHAsync(&err, e->err, 4, e->stream));
    SB_CK(cuStreamSynchronize(e->stream));
    if (err) {
        SB_CK(cuMemsetD32Async(e->err, 0, 1, e->stream));
        int rc = mk_clear_words(e);
        if (rc) return rc;
        SB_CK(cuStreamSynchronize(e->stream));
        return sb_fail(SB_ERR_STATE, "decode step aborted: a wait inside the persistent kernel timed out", __FILE__,
                       __LINE__);
    }
    return 0;
}

/* The epoch packs the step sequence number above 7 stage bits into 32 bits:
 * clear the words well before the sequence number could wrap. */
static int mk_epoch_guard(sb_engine *e) {
    if (!e->mk || e->mk_steps < (1L << 24)) return 0;
    return mk_clear_words(e);
}

static int put_step(sb_engine *e, const SbStep *st) {
    int rc = mk_epoch_guard(e);
    if (rc) return rc;
    SB_CK(cuMemcpyHtoDAsync(e->step, st, sizeof *st, e->stream));
    return 0;
}

int sb_engine_forward(sb_engine *e, int token, int pos, int want_logits, float *logits_host) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_ARG(pos >= 0 && pos < e->ctx_cap, "pos outside the KV cache");
    SB_ARG(token >= 0 && token < e->V, "token id out of range");
    SbStep st;
    memset(&st, 0, sizeof st);
    st.pos = pos;
    st.n_prompt = INT_MAX / 2; /* never write a next token */
    st.n_end = INT_MAX / 2;
    st.pos_limit = e->ctx_cap;
    int tok = token;
    SB_CK(cuMemcpyHtoDAsync(e->tokens + (size_t)pos * 4, &tok, 4, e->stream));
    int rc = put_step(e, &st);
    if (rc) return rc;
    if ((rc = run_step(e, want_logits ? 1 : 0))) return rc;
    if (want_logits && logits_host) SB_CK(cuMemcpyDtoHAsync(logits_host, e->logits, (size_t)e->V * 4, e->stream));
    SB_CK(cuStreamSynchronize(e->stream));
    return check_device_error(e);
}

int sb_engine_begin(sb_engine *e, const int *prompt, int n_prompt, int n_gen, unsigned gen_flags) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_ARG(prompt && n_prompt >= 1 && n_gen >= 0, "need at least one prompt token");
    SB_ARG(n_prompt + n_gen <= e->ctx_cap, "prompt + generation exceeds the KV cache");
    for (int i = 0; i < n_prompt; i++) SB_ARG(prompt[i] >= 0 && prompt[i] < e->V, "prompt id out of range");
    SB_CK(cuMemcpyHtoDAsync(e->tokens, prompt, (size_t)n_prompt * 4, e->stream));
    SbStep st;
    memset(&st, 0, sizeof st);
    st.pos = 0;
    st.n_prompt = n_prompt;
    st.n_end = n_prompt + n_gen + 1;
    st.pos_limit = e->ctx_cap;
    st.stop_on_eos = (gen_flags & SB_GEN_STOP_EOS) ? 1 : 0;
    st.eos0 = e->model == SB_MODEL_QWEN ? QW_EOT : G2_EOT;
    st.eos1 = e->model == SB_MODEL_QWEN ? QW_IM_END : -1;
    e->n_prompt = n_prompt;
    e->n_end = st.n_end;
    e->st_begin = st;
    /* graphs are built before the timed phases start */
    int rc = ensure_graph(e, 0);
    if (!rc) rc = ensure_graph(e, 1);
    if (rc) return rc;
    return put_step(e, &st);
}

int sb_engine_steps(sb_engine *e, int n, int with_logits) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    for (int i = 0; i < n; i++) {
        int rc = run_step(e, with_logits ? 1 : 0);
        if (rc) return rc;
    }
    return 0;
}

int sb_engine_finish(sb_engine *e, int *out_ids, int *n_out) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SbStep st;
    SB_CK(cuMemcpyDtoHAsync(&st, e->step, sizeof st, e->stream));
    SB_CK(cuStreamSynchronize(e->stream));
    int rc = check_device_error(e);
    if (rc) return rc;
    int n = e->n_prompt + st.n_generated;
    if (n > e->n_end) n = e->n_end;
    if (out_ids) {
        SB_CK(cuMemcpyDtoHAsync(out_ids, e->tokens, (size_t)n * 4, e->stream));
        SB_CK(cuStreamSynchronize(e->stream));
    }
    if (n_out) *n_out = n;
    return 0;
}

/* ------------------------------------------------------------------ prefill */
#define PF_T 128 /* prompt tokens per batch: 2 * PF_T hi/lo rows <= the GEMM's 256 */
/* element-wise prefill kernels: blocks per token row of n elements (256 threads each) */
#define PF_GY(n) ((unsigned)CEIL_DIV((n), 256))

/* GPT-2: LayerNorm rows -> 3xTF32 tensor-core products against the [out][in]
 * weights (FP32 accuracy) -> bias / GELU / residual kernels; causal attention
 * per (token, head) with the Qwen prefill kernel (12 KV heads = MHA). */
static int prefill_gpt2(sb_engine *e, int n) {
    sb_ctx *c = e->c;
    if (!e->pf_x) {
        SB_CK(cuMemAlloc(&e->pf_x, (size_t)PF_T * G2_C * 4));
        SB_CK(cuMemAlloc(&e->pf_a, (size_t)PF_T * G2_FC * 4));
        SB_CK(cuMemAlloc(&e->pf_y, (size_t)PF_T * G2_FC * 4));
        SB_CK(cuMemAlloc(&e->pf_q, (size_t)PF_T * G2_C * 4));
        SB_CK(cuMemAlloc(&e->pf_att, (size_t)PF_T * G2_C * 4));
    }
    CUstream s = e->stream;
    int C = G2_C, FC = G2_FC, NH = G2_NH, HD = G2_HD;
    float eps = 1e-5f, scale = 0.125f;
    const CUdeviceptr wte = e->w, wpe = e->w + G2_OFF_WPE * 4;
    const float *pa = (const float *)(uintptr_t)e->pf_a, *patt = (const float *)(uintptr_t)e->pf_att;
    float *py = (float *)(uintptr_t)e->pf_y;
    for (int p0 = 0; p0 < n; p0 += PF_T) {
        int T = n - p0 < PF_T ? n - p0 : PF_T;
        void *ea[] = {(void *)&wte, (void *)&wpe, &e->tokens, &e->pf_x, &p0, &C};
        int rc = sb_launch(c, F_G2PF_EMBED, (unsigned)T, PF_GY(G2_C), 256, 0, s, ea, 0);
        for (int l = 0; !rc && l < G2_NL; l++) {
            const CUdeviceptr lb = e->w + (G2_LBASE + (size_t)l * G2_LAYER) * 4;
            CUdeviceptr ln1w = lb + G2L_LN1W * 4, ln1b = lb + G2L_LN1B * 4, wqkv = lb + G2L_QKVW * 4;
            CUdeviceptr bqkv = lb + G2L_QKVB * 4, wo = lb + G2L_AOW * 4, bo = lb + G2L_AOB * 4;
            CUdeviceptr ln2w = lb + G2L_LN2W * 4, ln2b = lb + G2L_LN2B * 4, wfc = lb + G2L_FCW * 4;
            CUdeviceptr bfc = lb + G2L_FCB * 4, wp = lb + G2L_PROJW * 4, bp = lb + G2L_PROJB * 4;
            CUdeviceptr kc = e->kv + (size_t)l * e->ctx_cap * C * 4;
            CUdeviceptr vc = e->kv + (size_t)(G2_NL + l) * e->ctx_cap * C * 4;
            void *la[] = {&e->pf_x, &ln1w, &ln1b, &e->pf_a, &C, &eps};
            rc = sb_launch(c, F_G2_LAYERNORM_ROWS, (unsigned)T, 1, 256, 0, s, la, 0);
            if (!rc) rc = sb_sgemm_nt_3xtf32(pa, (const float *)(uintptr_t)wqkv, py, T, 3 * C, C, s);
            void *qa[] = {&e->pf_y, &bqkv, &e->pf_q, &kc, &vc, &p0, &C};
            if (!rc) rc = sb_launch(c, F_G2PF_QKV, (unsigned)T, PF_GY(G2_C), 256, 0, s, qa, 0);
            if (l == G2_NL - 1) break; /* the last layer's output feeds only logits */
            void *aa[] = {&e->pf_q, &kc, &vc, &e->pf_att, &p0, &C, &NH, &NH, &HD, &scale};
            if (!rc) rc = sb_launch(c, F_PF_ATTN, (unsigned)T, (unsigned)NH, 128, (unsigned)(p0 + T) * 4, s, aa, 0);
            if (!rc) rc = sb_sgemm_nt_3xtf32(patt, (const float *)(uintptr_t)wo, py, T, C, C, s);
            void *ra[] = {&e->pf_y, &bo, &e->pf_x, &C};
            if (!rc) rc = sb_launch(c, F_G2PF_BIAS_RESID, (unsigned)T, PF_GY(G2_C), 256, 0, s, ra, 0);
            void *l2[] = {&e->pf_x, &ln2w, &ln2b, &e->pf_a, &C, &eps};
            if (!rc) rc = sb_launch(c, F_G2_LAYERNORM_ROWS, (unsigned)T, 1, 256, 0, s, l2, 0);
            if (!rc) rc = sb_sgemm_nt_3xtf32(pa, (const float *)(uintptr_t)wfc, py, T, FC, C, s);
            void *ga[] = {&e->pf_y, &bfc, &e->pf_a, &FC};
            if (!rc) rc = sb_launch(c, F_G2PF_BIAS_GELU, (unsigned)T, PF_GY(G2_FC), 256, 0, s, ga, 0);
            if (!rc) rc = sb_sgemm_nt_3xtf32(pa, (const float *)(uintptr_t)wp, py, T, C, FC, s);
            void *pr[] = {&e->pf_y, &bp, &e->pf_x, &C};
            if (!rc) rc = sb_launch(c, F_G2PF_BIAS_RESID, (unsigned)T, PF_GY(G2_C), 256, 0, s, pr, 0);
        }
        if (rc) return rc;
    }
    SbStep st = e->st_begin;
    st.pos = n;
    return put_step(e, &st);
}

int sb_engine_prefill(sb_engine *e, int n) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_ARG(n >= 0 && n < e->n_prompt, "prefill covers prompt tokens before the last one");
    if (n == 0) return 0;
    if (e->model == SB_MODEL_GPT2) return prefill_gpt2(e, n);
    sb_ctx *c = e->c;
    if (!e->pf_x) {
        SB_CK(cuMemAlloc(&e->pf_x, (size_t)PF_T * QW_C * 4));
        SB_CK(cuMemAlloc(&e->pf_xh, (size_t)2 * PF_T * QW_FC * 2));
        SB_CK(cuMemAlloc(&e->pf_y, (size_t)2 * PF_T * 2 * QW_FC * 4));
        SB_CK(cuMemAlloc(&e->pf_q, (size_t)PF_T * QW_C * 4));
        SB_CK(cuMemAlloc(&e->pf_att, (size_t)PF_T * QW_C * 4));
    }
    CUstream s = e->stream;
    int C = QW_C, FC = QW_FC, NH = QW_NH, NKV = QW_NKV, HD = QW_HD;
    float eps = 1e-6f, scale = 0.125f;
    const CUdeviceptr cosT = e->w + QW_OFF_COS, sinT = e->w + QW_OFF_SIN;
    const uint16_t *xh = (const uint16_t *)(uintptr_t)e->pf_xh;
    float *y = (float *)(uintptr_t)e->pf_y;
    for (int p0 = 0; p0 < n; p0 += PF_T) {
        int T = n - p0 < PF_T ? n - p0 : PF_T;
        void *ea[] = {&e->w, &e->tokens, &e->pf_x, &p0, &C};
        int rc = sb_launch(c, F_PF_EMBED, (unsigned)T, PF_GY(QW_C), 256, 0, s, ea, 0);
        for (int l = 0; !rc && l < QW_NL; l++) {
            const CUdeviceptr L = e->w + QW_LBASE + (size_t)l * QW_LSTRIDE;
            CUdeviceptr g_in = L, wqkv = L + QW_C * 2, bqkv = wqkv + (size_t)QW_QKV * QW_C * 2;
            CUdeviceptr wo = bqkv + QW_QKV * 2, g_post = wo + (size_t)QW_C * QW_C * 2, wgu = g_post + QW_C * 2;
            CUdeviceptr wdown = wgu + (size_t)2 * QW_FC * QW_C * 2;
            CUdeviceptr kc = e->kv + (size_t)l * e->ctx_cap * QW_KVD * 4;
            CUdeviceptr vc = e->kv + (size_t)(QW_NL + l) * e->ctx_cap * QW_KVD * 4;
            int twoT = 2 * T;
            /* QKV of every token (RoPE, KV-cache rows) */
            void *ra[] = {&e->pf_x, &g_in, &e->pf_xh, &T, &C, &eps};
            rc = sb_launch(c, F_PF_RMS_SPLIT, (unsigned)T, 1, 256, 0, s, ra, 0);
            if (!rc) rc = sb_gemm_hh((const uint16_t *)(uintptr_t)wqkv, xh, y, C, QW_QKV, twoT, s);
            void *qa[] = {&e->pf_y, &bqkv, (void *)&cosT, (void *)&sinT, &e->pf_q, &kc, &vc, &T, &p0, &C, &NH, &NKV, &HD};
            if (!rc) rc = sb_launch(c, F_PF_QKV, (unsigned)T, PF_GY(QW_QKV / 2), 256, 0, s, qa, 0);
            if (l == QW_NL - 1) break; /* the last layer's output feeds only logits */
            /* causal attention, O projection + residual */
            void *aa[] = {&e->pf_q, &kc, &vc, &e->pf_att, &p0, &C, &NH, &NKV, &HD, &scale};
            if (!rc) rc = sb_launch(c, F_PF_ATTN, (unsigned)T, (unsigned)NH, 128, (unsigned)(p0 + T) * 4, s, aa, 0);
            void *sa[] = {&e->pf_att, &e->pf_xh, &T, &C};
            if (!rc) rc = sb_launch(c, F_PF_SPLIT, (unsigned)T, PF_GY(QW_C), 256, 0, s, sa, 0);
            if (!rc) rc = sb_gemm_hh((const uint16_t *)(uintptr_t)wo, xh, y, C, QW_C, twoT, s);
            void *xa[] = {&e->pf_y, &e->pf_x, &T, &C};
            if (!rc) rc = sb_launch(c, F_PF_RESID, (unsigned)T, PF_GY(QW_C), 256, 0, s, xa, 0);
            /* MLP: RMSNorm -> gate|up -> SwiGLU -> down + residual */
            void *pa[] = {&e->pf_x, &g_post, &e->pf_xh, &T, &C, &eps};
            if (!rc) rc = sb_launch(c, F_PF_RMS_SPLIT, (unsigned)T, 1, 256, 0, s, pa, 0);
            if (!rc) rc = sb_gemm_hh((const uint16_t *)(uintptr_t)wgu, xh, y, C, 2 * QW_FC, twoT, s);
            void *wa[] = {&e->pf_y, &e->pf_xh, &T, &FC};
            if (!rc) rc = sb_launch(c, F_PF_SWIGLU_SPLIT, (unsigned)T, PF_GY(QW_FC), 256, 0, s, wa, 0);
            if (!rc) rc = sb_gemm_hh((const uint16_t *)(uintptr_t)wdown, xh, y, FC, QW_C, twoT, s);
            if (!rc) rc = sb_launch(c, F_PF_RESID, (unsigned)T, PF_GY(QW_C), 256, 0, s, xa, 0);
        }
        if (rc) return rc;
    }
    /* the decode steps continue at position n */
    SbStep st = e->st_begin;
    st.pos = n;
    return put_step(e, &st);
}

int sb_engine_generate(sb_engine *e, const int *prompt, int n_prompt, int n_gen, int *out_ids, int *n_out,
                       unsigned gen_flags) {
    int rc = sb_engine_begin(e, prompt, n_prompt, n_gen, gen_flags);
    if (!rc && !(e->flags & SB_FLAG_NO_PREFILL) && n_prompt > 1) {
        rc = sb_engine_prefill(e, n_prompt - 1); /* prompt tokens batched on the tensor cores */
        if (!rc) rc = sb_engine_steps(e, n_gen + 1, 1); /* last prompt token + n_gen */
        if (!rc) rc = sb_engine_finish(e, out_ids, n_out);
        return rc;
    }
    if (!rc) rc = sb_engine_steps(e, n_prompt - 1, 0); /* prompt tokens: no LM head */
    if (!rc) rc = sb_engine_steps(e, n_gen + 1, 1);    /* last prompt token + n_gen */
    if (!rc) rc = sb_engine_finish(e, out_ids, n_out);
    return rc;
}

/* ------------------------------------------------------------------ profiling */
/* Algorithmic DRAM bytes of one launch of a step kernel (weights streamed
 * plus activations read/written), the numerator of its roofline figure. */
static double kernel_bytes(const sb_engine *e, int which) {
    const int qw = e->model == SB_MODEL_QWEN;
    const double C = qw ? QW_C : G2_C, FC = qw ? QW_FC : G2_FC, V = qw ? QW_V : G2_V;
    const double wb = qw ? 2.0 : 4.0; /* weight element bytes */
    const double NQKV = qw ? QW_QKV : 3.0 * G2_C;
    switch (which) {
    case SBK_QKV: return NQKV * C * wb + NQKV * wb + C * 4 + C * wb + NQKV * 4;
    case SBK_O: return C * C * wb + C * 4 + 2 * C * 4;
    case SBK_MLP_UP: return (qw ? 2 * FC : FC) * C * wb + C * 4 + C * wb + FC * 4;
    case SBK_MLP_DOWN: return C * FC * wb + FC * 4 + 2 * C * 4;
    case SBK_LMHEAD: return V * C * wb + C * 4 + C * wb + V * 4;
    default: return 0;
    }
}

int sb_engine_profile(sb_engine *e, int which, int reps, void *flush, size_t flush_bytes, float *avg_ms,
                      double *bytes) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_ARG(which >= 0 && which < SBK_COUNT && reps > 0, "bad profile request");
    SbStep st;
    memset(&st, 0, sizeof st);
    st.pos = 0;
    st.n_prompt = INT_MAX / 2;
    st.n_end = INT_MAX / 2;
    st.pos_limit = e->ctx_cap;
    int rc = put_step(e, &st);
    if (rc) return rc;
    CUevent e0, e1;
    SB_CK(cuEventCreate(&e0, 0));
    SB_CK(cuEventCreate(&e1, 0));
    double total = 0;
    /* The flush READS the buffer (membw_read4) so L2 ends up full of clean
     * lines: a memset would leave ~126 MB of dirty lines whose write-back
     * would be charged to the timed kernel. */
    CUdeviceptr fb = (CUdeviceptr)(uintptr_t)flush;
    int fn4 = (int)(flush_bytes / 16), fiters = 1;
    for (int r = 0; r < reps && !rc; r++) {
        if (flush && fn4 > 0) {
            void *fa[] = {&fb, &e->logits, &fn4, &fiters};
            rc = sb_launch(e->c, F_MEMBW, (unsigned)(4 * e->c->sms), 1, 256, 0, e->stream, fa, 0);
        }
        if (!rc) rc = cuEventRecord(e0, e->stream);
        if (!rc) rc = launch_kernel(e, 0, which, 1, 0);
        if (!rc) rc = cuEventRecord(e1, e->stream);
        if (!rc) rc = cuEventSynchronize(e1);
        float ms = 0;
        if (!rc) rc = cuEventElapsedTime(&ms, e0, e1);
        total += ms;
    }
    cuEventDestroy(e0);
    cuEventDestroy(e1);
    if (rc) return sb_fail(rc, "profile launch", __FILE__, __LINE__);
    if (avg_ms) *avg_ms = (float)(total / reps);
    if (bytes) *bytes = kernel_bytes(e, which);
    return 0;
}

const char *sb_engine_step_kernel(sb_engine *e) {
    if (!e) return "";
    if (!e->mk) return e->model == SB_MODEL_QWEN ? "qwen per-stage kernels" : "gpt2 per-stage kernels";
    return e->model == SB_MODEL_QWEN ? (e->mk2 ? "qwen_decode_mk2" : "qwen_decode_mk") : "gpt2_decode_mk";
}

int sb_engine_uses_persistent_kernel(sb_engine *e) { return e && e->mk; }

int sb_engine_sample(sb_engine *e, int ctx_len, float temperature, int top_k, float top_p, float rep_penalty,
                     uint32_t *rng_state) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_ARG(ctx_len >= 0 && ctx_len <= e->ctx_cap && rng_state, "bad sampling arguments");
    SB_ARG(top_k >= 1 && top_k <= 64, "top_k must be in 1..64");
    /* the device picks the k candidates of the reference's steps 1-3 from
     * the step's logits and the token ids in the KV order; the host draws */
    CUdeviceptr ci = e->tk, cv = e->tk + 64 * 4;
    int rc = sb_topk_penalized((const float *)(uintptr_t)e->logits, e->V, (const int *)(uintptr_t)e->tokens, ctx_len,
                               temperature, rep_penalty, top_k, (int *)(uintptr_t)ci, (float *)(uintptr_t)cv,
                               e->stream);
    if (rc) return -rc;
    int idx[64];
    float val[64];
    SB_CK(cuMemcpyDtoHAsync(idx, ci, (size_t)top_k * 4, e->stream));
    SB_CK(cuMemcpyDtoHAsync(val, cv, (size_t)top_k * 4, e->stream));
    SB_CK(cuStreamSynchronize(e->stream));
    return sb_sample_topk(idx, val, top_k, top_p, rng_state);
}

int sb_engine_set_test_stall(sb_engine *e, int cta) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    SB_ARG(e->mk, "the test stall applies to the persistent step kernel only");
    SB_ARG(cta >= -1 && cta < e->c->sms, "cta out of range");
    e->test_stall = cta + 1;
    for (int i = 0; i < 2; i++)
        if (e->gexec[i]) {
            cuGraphExecDestroy(e->gexec[i]);
            e->gexec[i] = NULL;
        }
    return 0;
}

int sb_engine_set_trace(sb_engine *e, void *dev_buf) {
    if (!e) return sb_fail(SB_ERR_ARG, "null engine", __FILE__, __LINE__);
    e->trace = (CUdeviceptr)(uintptr_t)dev_buf;
    for (int i = 0; i < 2; i++)
        if (e->gexec[i]) {
            cuGraphExecDestroy(e->gexec[i]);
            e->gexec[i] = NULL;
        }
    return 0;
}
