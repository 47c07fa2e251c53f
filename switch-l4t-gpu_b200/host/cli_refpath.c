/* cli_refpath.c -- per-stage decode through a module image's drop-in
 * kernels (the reference's gpu_forward) and the serial CPU forward (the
 * reference's cpu_forward), for the command-line hosts; see cli_refpath.h.
 *
 * Both follow the reference's stage order and launch geometry so that an
 * operator's own module, passed with --ptx, runs exactly as it would under
 * the reference host, and so that --selftest means what it means there:
 * device logits against an independent FP32 CPU computation. */
#define _GNU_SOURCE
#include "cli_refpath.h"

#include <cuda.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/switch_b200.h"
#include "sb_models.h"

#define RP_BLOCK 256
#define RP_CK(x)                                                                                        \
    do {                                                                                                \
        CUresult r_ = (x);                                                                              \
        if (r_ != CUDA_SUCCESS) {                                                                       \
            const char *s_ = NULL;                                                                      \
            cuGetErrorString(r_, &s_);                                                                  \
            fprintf(stderr, "CUDA error %d (%s) at %s:%d\n", (int)r_, s_ ? s_ : "?", __FILE__, __LINE__); \
            exit(1);                                                                                    \
        }                                                                                               \
    } while (0)

enum { F_GEMV, F_GEMVB, F_NORM, F_ROPE, F_SWIGLU, F_GELU, F_ABIAS, F_ADD2, F_ASCORES, F_ASOFTMAX, F_AMIX, F_N };

struct refpath {
    int model, ctx, V, C, NL, kvw, fused;
    float *trace;
    char module_name[512];
    unsigned char *hw; /* the weight file, host copy */
    size_t wbytes;
    CUmodule mod;
    CUfunction f[F_N];
    CUdeviceptr w;       /* the weight file, device copy (tensors at the file's byte offsets) */
    CUdeviceptr qkvb32;  /* Qwen: q/k/v biases decoded to FP32 per layer (the kernel reads float bias) */
    CUdeviceptr kc, vc;  /* [NL][ctx][kvw] */
    CUdeviceptr x, ln, qkv, att, y, ln2, hid, hid2, scores, probs, logits, x2;
    /* CPU forward */
    float *kch, *vch, *sc, *rx, *rln, *rqkv, *ratt, *ry, *rln2, *rhid, *rhid2;
};

const char *rp_module_name(const refpath *r) { return r->module_name; }

/* the reference's fp16 decode (qwen_engine.c:90-98): exponent 0 reads as 0 */
static float h2f_ref(unsigned short h) {
    const unsigned e = (h >> 10) & 0x1fu;
    if (e == 0) return 0.0f;
    const unsigned u = ((unsigned)(h & 0x8000u) << 16) | ((e + 112u) << 23) | ((unsigned)(h & 0x3ffu) << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static CUdeviceptr dalloc(size_t bytes) {
    CUdeviceptr p = 0;
    RP_CK(cuMemAlloc(&p, bytes));
    RP_CK(cuMemsetD8(p, 0, bytes));
    return p;
}

static void gdump(const char *tag, CUdeviceptr d, int n) {
    float *tmp = malloc((size_t)n * 4);
    RP_CK(cuCtxSynchronize());
    RP_CK(cuMemcpyDtoH(tmp, d, (size_t)n * 4));
    float s = 0;
    for (int i = 0; i < n; i++) s += tmp[i];
    printf("    g.%-8s first4=%.3f %.3f %.3f %.3f sum=%.3f\n", tag, tmp[0], tmp[1], tmp[2], tmp[3], s);
    free(tmp);
}
static void cdump(const char *tag, const float *v, int n) {
    float s = 0;
    for (int i = 0; i < n; i++) s += v[i];
    printf("    c.%-8s first4=%.3f %.3f %.3f %.3f sum=%.3f\n", tag, v[0], v[1], v[2], v[3], s);
}

static void launch(refpath *r, int fn, unsigned grid, unsigned block, void **args) {
    RP_CK(cuLaunchKernel(r->f[fn], grid, 1, 1, block, 1, 1, 0, NULL, args, NULL));
}

refpath *rp_open(int model, const char *weights, const char *module_path, int ctx) {
    refpath *r = calloc(1, sizeof *r);
    const int qw = model == SB_MODEL_QWEN;
    r->model = model;
    r->ctx = ctx;
    r->V = qw ? QW_V : G2_V;
    r->C = qw ? QW_C : G2_C;
    r->NL = qw ? QW_NL : G2_NL;
    r->kvw = qw ? QW_KVD : G2_C;
    r->wbytes = qw ? QW_FILE_BYTES : (size_t)G2_TOTAL_FLOATS * 4;
    FILE *f = fopen(weights, "rb");
    if (!f) { fprintf(stderr, "cannot open %s\n", weights); exit(2); }
    r->hw = malloc(r->wbytes);
    if (fread(r->hw, 1, r->wbytes, f) != r->wbytes || fgetc(f) != EOF) {
        fprintf(stderr, "weight file %s has the wrong size\n", weights);
        exit(2);
    }
    fclose(f);
    if (sb_init(0)) { fprintf(stderr, "%s\n", sb_last_error()); exit(1); }
    /* the module: the operator's file, or this package's built-in image */
    if (module_path) {
        FILE *m = fopen(module_path, "rb");
        if (!m) { fprintf(stderr, "cannot open ptx\n"); exit(2); }
        fseek(m, 0, SEEK_END);
        const long n = ftell(m);
        fseek(m, 0, SEEK_SET);
        char *img = malloc((size_t)n + 1);
        if (fread(img, 1, (size_t)n, m) != (size_t)n) exit(2);
        img[n] = 0;
        fclose(m);
        RP_CK(cuModuleLoadData(&r->mod, img));
        free(img);
        snprintf(r->module_name, sizeof r->module_name, "%s", module_path);
    } else {
        const void *img = NULL;
        size_t n = 0;
        if (sb_module_image(qw ? "qwen" : "gpt2", &img, &n)) { fprintf(stderr, "no built-in module\n"); exit(1); }
        RP_CK(cuModuleLoadData(&r->mod, img));
        snprintf(r->module_name, sizeof r->module_name, "built-in %s.cubin", qw ? "qwen" : "gpt2");
    }
    /* the names each reference engine requires (qwen_engine.c:148-155, gpt2_engine.c:119-128) */
    if (qw) {
        const char *names[] = {"gemv_h", "rmsnorm", "rope", "swiglu", "add2", "attn_scores_gqa", "attn_softmax",
                               "attn_mix_gqa"};
        const int ids[] = {F_GEMV, F_NORM, F_ROPE, F_SWIGLU, F_ADD2, F_ASCORES, F_ASOFTMAX, F_AMIX};
        for (int i = 0; i < 8; i++) RP_CK(cuModuleGetFunction(&r->f[ids[i]], r->mod, names[i]));
    } else {
        const char *names[] = {"gemv_warp", "gemv_warp_b", "layernorm", "gelu", "add_bias", "add2", "attn_scores",
                               "attn_softmax", "attn_mix"};
        const int ids[] = {F_GEMV, F_GEMVB, F_NORM, F_GELU, F_ABIAS, F_ADD2, F_ASCORES, F_ASOFTMAX, F_AMIX};
        for (int i = 0; i < 9; i++) RP_CK(cuModuleGetFunction(&r->f[ids[i]], r->mod, names[i]));
    }
    return r;
}

/* device copies and buffers, on the first GPU forward (a CPU-only selftest
 * needs none of them) */
static void rp_device(refpath *r) {
    if (r->w) return;
    const int qw = r->model == SB_MODEL_QWEN, ctx = r->ctx;
    r->w = dalloc(r->wbytes);
    RP_CK(cuMemcpyHtoD(r->w, r->hw, r->wbytes));
    if (qw) {
        float *b = malloc((size_t)QW_NL * QW_QKV * 4);
        for (int l = 0; l < QW_NL; l++) {
            const unsigned short *src = (const unsigned short *)(r->hw + QW_LBASE + (size_t)l * QW_LSTRIDE) + QWL_QKVB;
            for (int i = 0; i < QW_QKV; i++) b[(size_t)l * QW_QKV + i] = h2f_ref(src[i]);
        }
        r->qkvb32 = dalloc((size_t)QW_NL * QW_QKV * 4);
        RP_CK(cuMemcpyHtoD(r->qkvb32, b, (size_t)QW_NL * QW_QKV * 4));
        free(b);
    }
    const size_t kv = (size_t)r->NL * ctx * r->kvw * 4;
    r->kc = dalloc(kv);
    r->vc = dalloc(kv);
    const int C = r->C, FC = qw ? QW_FC : G2_FC, NH = qw ? QW_NH : G2_NH;
    r->x = dalloc((size_t)C * 4);
    r->ln = dalloc((size_t)C * 4);
    r->qkv = dalloc((size_t)(qw ? QW_QKV : 3 * C) * 4);
    r->att = dalloc((size_t)C * 4);
    r->y = dalloc((size_t)C * 4);
    r->ln2 = dalloc((size_t)C * 4);
    r->hid = dalloc((size_t)2 * FC * 4);
    r->hid2 = dalloc((size_t)FC * 4);
    r->scores = dalloc((size_t)ctx * NH * 4);
    r->probs = dalloc((size_t)ctx * NH * 4);
    r->logits = dalloc((size_t)r->V * 4);
    r->x2 = dalloc((size_t)C * 4);
}

static void rp_host_buffers(refpath *r) {
    const int qw = r->model == SB_MODEL_QWEN, ctx = r->ctx, C = r->C, FC = qw ? QW_FC : G2_FC;
    r->kch = calloc((size_t)r->NL * ctx * r->kvw, 4);
    r->vch = calloc((size_t)r->NL * ctx * r->kvw, 4);
    r->sc = calloc((size_t)ctx, 4);
    r->rx = calloc(C, 4);
    r->rln = calloc(C, 4);
    r->rqkv = calloc(qw ? QW_QKV : 3 * C, 4);
    r->ratt = calloc(C, 4);
    r->ry = calloc(C, 4);
    r->rln2 = calloc(C, 4);
    r->rhid = calloc(2 * FC, 4);
    r->rhid2 = calloc(FC, 4);
}

void rp_close(refpath *r) {
    if (!r) return;
    CUdeviceptr d[] = {r->w, r->qkvb32, r->kc, r->vc, r->x, r->ln, r->qkv, r->att, r->y, r->ln2, r->hid, r->hid2,
                       r->scores, r->probs, r->logits, r->x2};
    for (size_t i = 0; i < sizeof d / sizeof d[0]; i++)
        if (d[i]) cuMemFree(d[i]);
    cuModuleUnload(r->mod);
    float *h[] = {r->kch, r->vch, r->sc, r->rx, r->rln, r->rqkv, r->ratt, r->ry, r->rln2, r->rhid, r->rhid2};
    for (size_t i = 0; i < sizeof h / sizeof h[0]; i++) free(h[i]);
    free(r->hw);
    free(r);
}

/* ------------------------------------------------------------------ Qwen (qwen_engine.c:205-269) */
static void qwen_forward(refpath *r, int token, int pos, int want_logits, float *logits, int debug) {
    const int gtrace = debug && pos == 0;
    int cC = QW_C, cQKV = QW_QKV, cFC = QW_FC, c2FC = 2 * QW_FC, cNH = QW_NH, cKV = QW_KVD, cHD = QW_HD, cV = QW_V;
    int cNKV = QW_NKV, one = 1, Tp = pos + 1, pos0 = pos;
    float eps = 1e-6f, scale = 0.125f;
    const unsigned short *emb = (const unsigned short *)r->hw;
    float *xb = malloc(QW_C * 4);
    for (int i = 0; i < QW_C; i++) xb[i] = h2f_ref(emb[(size_t)token * QW_C + i]);
    RP_CK(cuMemcpyHtoD(r->x, xb, QW_C * 4));
    free(xb);
    CUdeviceptr cosT = r->w + QW_OFF_COS, sinT = r->w + QW_OFF_SIN, lnf = r->w + QW_OFF_LNF;
    for (int l = 0; l < QW_NL; l++) {
        const CUdeviceptr L = r->w + QW_LBASE + (size_t)l * QW_LSTRIDE;
        CUdeviceptr inln = L + QWL_INLN * 2, qkvw = L + QWL_QKVW * 2, ow = L + QWL_OW * 2, post = L + QWL_POST * 2;
        CUdeviceptr gu = L + QWL_GATEUP * 2, down = L + QWL_DOWN * 2, qkvb = r->qkvb32 + (size_t)l * QW_QKV * 4;
        CUdeviceptr kcl = r->kc + (size_t)l * r->ctx * QW_KVD * 4, vcl = r->vc + (size_t)l * r->ctx * QW_KVD * 4;
        CUdeviceptr nullb = 0;
        launch(r, F_NORM, 1, RP_BLOCK, (void *[]){&r->x, &inln, &r->ln, &cC, &eps});
        if (gtrace && l == 0) gdump("ln1", r->ln, QW_C);
        launch(r, F_GEMV, (QW_QKV + 7) / 8, RP_BLOCK, (void *[]){&qkvw, &r->ln, &qkvb, &r->qkv, &cC, &cQKV});
        launch(r, F_ROPE, (QW_NH * (QW_HD / 2) + 255) / 256, RP_BLOCK,
               (void *[]){&r->qkv, &cosT, &sinT, &one, &cNH, &cHD, &pos0});
        CUdeviceptr dk = r->qkv + (size_t)QW_NH * QW_HD * 4;
        launch(r, F_ROPE, (QW_NKV * (QW_HD / 2) + 255) / 256, RP_BLOCK,
               (void *[]){&dk, &cosT, &sinT, &one, &cNKV, &cHD, &pos0});
        if (gtrace && l == 0) gdump("qkv", r->qkv, QW_QKV);
        RP_CK(cuMemcpyDtoD(kcl + (size_t)pos * QW_KVD * 4, r->qkv + (size_t)QW_NH * QW_HD * 4, QW_KVD * 4));
        RP_CK(cuMemcpyDtoD(vcl + (size_t)pos * QW_KVD * 4, r->qkv + (size_t)(QW_NH * QW_HD + QW_KVD) * 4, QW_KVD * 4));
        launch(r, F_ASCORES, (Tp * QW_NH + 255) / 256, RP_BLOCK,
               (void *[]){&r->qkv, &kcl, &r->scores, &Tp, &scale, &cNH, &cKV, &cHD});
        launch(r, F_ASOFTMAX, 1, QW_NH, (void *[]){&r->scores, &r->probs, &Tp, &cNH});
        launch(r, F_AMIX, (QW_NH * QW_HD + 255) / 256, RP_BLOCK,
               (void *[]){&r->probs, &vcl, &r->att, &Tp, &cNH, &cKV, &cHD});
        if (gtrace && l == 0) {
            gdump("scores", r->scores, Tp * QW_NH);
            gdump("probs", r->probs, Tp * QW_NH);
            gdump("attnout", r->att, QW_C);
        }
        launch(r, F_GEMV, (QW_C + 7) / 8, RP_BLOCK, (void *[]){&ow, &r->att, &nullb, &r->y, &cC, &cC});
        launch(r, F_ADD2, (QW_C + 255) / 256, RP_BLOCK, (void *[]){&r->x, &r->y, &r->x, &cC});
        if (gtrace && l == 0) gdump("res1", r->x, QW_C);
        launch(r, F_NORM, 1, RP_BLOCK, (void *[]){&r->x, &post, &r->ln2, &cC, &eps});
        launch(r, F_GEMV, (2 * QW_FC + 7) / 8, RP_BLOCK, (void *[]){&gu, &r->ln2, &nullb, &r->hid, &cC, &c2FC});
        if (gtrace && l == 0) gdump("gate", r->hid, QW_FC);
        CUdeviceptr up = r->hid + (size_t)QW_FC * 4;
        launch(r, F_SWIGLU, (QW_FC + 255) / 256, RP_BLOCK, (void *[]){&r->hid, &up, &r->hid2, &cFC});
        if (gtrace && l == 0) gdump("swiglu", r->hid2, QW_FC);
        launch(r, F_GEMV, (QW_C + 7) / 8, RP_BLOCK, (void *[]){&down, &r->hid2, &nullb, &r->y, &cFC, &cC});
        launch(r, F_ADD2, (QW_C + 255) / 256, RP_BLOCK, (void *[]){&r->x, &r->y, &r->x, &cC});
        if (gtrace && l == 0) gdump("res2", r->x, QW_C);
        if (r->trace) RP_CK(cuMemcpyDtoH(r->trace + (size_t)l * QW_C, r->x, QW_C * 4));
    }
    if (!want_logits) return;
    CUdeviceptr nullb = 0, embd = r->w;
    launch(r, F_NORM, 1, RP_BLOCK, (void *[]){&r->x, &lnf, &r->x2, &cC, &eps});
    launch(r, F_GEMV, (QW_V + 7) / 8, RP_BLOCK, (void *[]){&embd, &r->x2, &nullb, &r->logits, &cC, &cV});
    RP_CK(cuCtxSynchronize());
    if (logits) RP_CK(cuMemcpyDtoH(logits, r->logits, (size_t)QW_V * 4));
}

/* qwen_engine.c:276-289 */
static void cpu_gemv_h(const unsigned short *W, const float *x, const unsigned short *bias, float *y, int K, int N) {
    for (int o = 0; o < N; o++) {
        const unsigned short *row = W + (size_t)o * K;
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc += h2f_ref(row[k]) * x[k];
        y[o] = acc + (bias ? h2f_ref(bias[o]) : 0.0f);
    }
}
static void cpu_rms(const float *x, const unsigned short *w, float *y, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / n + 1e-6f);
    for (int i = 0; i < n; i++) y[i] = x[i] * inv * h2f_ref(w[i]);
}

/* qwen_engine.c:292-358 */
static void qwen_cpu(refpath *r, int token, int pos, int want_logits, float *logits, int debug) {
    const int C = QW_C, HD = QW_HD, KVD = QW_KVD, NH = QW_NH, NKV = QW_NKV, FC = QW_FC, ctx = r->ctx;
    const int dump = debug && pos == 0;
    const unsigned short *emb = (const unsigned short *)r->hw;
    const float *cosT = (const float *)(r->hw + QW_OFF_COS), *sinT = (const float *)(r->hw + QW_OFF_SIN);
    float *x = r->rx, *ln = r->rln, *qkv = r->rqkv, *att = r->ratt, *y = r->ry, *ln2 = r->rln2, *g = r->rhid;
    float *dn = r->rhid2, *sc = r->sc;
    for (int i = 0; i < C; i++) x[i] = h2f_ref(emb[(size_t)token * C + i]);
    for (int l = 0; l < QW_NL; l++) {
        const unsigned short *b = (const unsigned short *)(r->hw + QW_LBASE + (size_t)l * QW_LSTRIDE);
        if (dump && l == 0) cdump("embed", x, C);
        cpu_rms(x, b + QWL_INLN, ln, C);
        if (dump && l == 0) cdump("ln1", ln, C);
        cpu_gemv_h(b + QWL_QKVW, ln, b + QWL_QKVB, qkv, C, QW_QKV);
        if (dump && l == 0) cdump("qkv", qkv, QW_QKV);
        for (int h = 0; h < NH + NKV; h++) { /* RoPE: the q heads, then the k heads */
            float *v = h < NH ? qkv + h * HD : qkv + C + (h - NH) * HD;
            for (int i = 0; i < HD / 2; i++) {
                const float a = v[i], b2 = v[HD / 2 + i];
                const float c = cosT[(size_t)pos * (HD / 2) + i], s = sinT[(size_t)pos * (HD / 2) + i];
                v[i] = a * c - b2 * s;
                v[HD / 2 + i] = a * s + b2 * c;
            }
        }
        float *kc = r->kch + (size_t)l * ctx * KVD, *vc = r->vch + (size_t)l * ctx * KVD;
        for (int i = 0; i < KVD; i++) {
            kc[(size_t)pos * KVD + i] = qkv[C + i];
            vc[(size_t)pos * KVD + i] = qkv[C + KVD + i];
        }
        for (int h = 0; h < NH; h++) {
            const int g2 = h / (NH / NKV);
            float maxv = -1e30f;
            for (int t = 0; t <= pos; t++) {
                float acc = 0.0f;
                for (int d = 0; d < HD; d++) acc += qkv[h * HD + d] * kc[(size_t)t * KVD + g2 * HD + d];
                sc[t] = acc * 0.125f;
                if (sc[t] > maxv) maxv = sc[t];
            }
            float sum = 0.0f;
            for (int t = 0; t <= pos; t++) {
                sc[t] = expf(sc[t] - maxv);
                sum += sc[t];
            }
            for (int d = 0; d < HD; d++) {
                float acc = 0.0f;
                for (int t = 0; t <= pos; t++) acc += (sc[t] / sum) * vc[(size_t)t * KVD + g2 * HD + d];
                att[h * HD + d] = acc;
            }
        }
        cpu_gemv_h(b + QWL_OW, att, NULL, y, C, C);
        if (dump && l == 0) cdump("ao", y, C);
        for (int i = 0; i < C; i++) x[i] += y[i];
        if (dump && l == 0) cdump("res1", x, C);
        cpu_rms(x, b + QWL_POST, ln2, C);
        cpu_gemv_h(b + QWL_GATEUP, ln2, NULL, g, C, 2 * FC);
        for (int i = 0; i < FC; i++) dn[i] = (g[i] / (1.0f + expf(-g[i]))) * g[FC + i];
        cpu_gemv_h(b + QWL_DOWN, dn, NULL, y, FC, C);
        for (int i = 0; i < C; i++) x[i] += y[i];
        if (r->trace) memcpy(r->trace + (size_t)l * C, x, (size_t)C * 4);
    }
    if (!want_logits) return;
    cpu_rms(x, (const unsigned short *)(r->hw + QW_OFF_LNF), ln, C);
    cpu_gemv_h(emb, ln, NULL, logits, C, QW_V);
}

/* ------------------------------------------------------------------ GPT-2 (gpt2_engine.c:174-264) */
static void gpt2_forward(refpath *r, int token, int pos, int want_logits, float *logits, int debug) {
    const int gtrace = debug && pos == 0;
    const int C = G2_C, FC = G2_FC;
    int cC = C, c3C = 3 * C, cFC = FC, cV = G2_V, T = pos + 1;
    float eps = 1e-5f, scale = 0.125f;
    const float *hw = (const float *)r->hw;
    float *xh = malloc(C * 4);
    for (int i = 0; i < C; i++) xh[i] = hw[(size_t)token * C + i] + hw[G2_OFF_WPE + (size_t)pos * C + i];
    RP_CK(cuMemcpyHtoD(r->x, xh, C * 4));
    free(xh);
    for (int l = 0; l < G2_NL; l++) {
        const CUdeviceptr L = r->w + (G2_LBASE + (size_t)l * G2_LAYER) * 4;
        CUdeviceptr ln1w = L + G2L_LN1W * 4, ln1b = L + G2L_LN1B * 4, qkvw = L + G2L_QKVW * 4, qkvb = L + G2L_QKVB * 4;
        CUdeviceptr aow = L + G2L_AOW * 4, aob = L + G2L_AOB * 4, ln2w = L + G2L_LN2W * 4, ln2b = L + G2L_LN2B * 4;
        CUdeviceptr fcw = L + G2L_FCW * 4, fcb = L + G2L_FCB * 4, pw = L + G2L_PROJW * 4, pb = L + G2L_PROJB * 4;
        CUdeviceptr kcl = r->kc + (size_t)l * r->ctx * C * 4, vcl = r->vc + (size_t)l * r->ctx * C * 4;
        launch(r, F_NORM, 1, RP_BLOCK, (void *[]){&r->x, &ln1w, &ln1b, &r->ln, &cC, &eps});
        if (gtrace && l == 0) gdump("ln1", r->ln, C);
        if (r->fused) {
            launch(r, F_GEMVB, (3 * C + 7) / 8, RP_BLOCK, (void *[]){&qkvw, &r->ln, &qkvb, &r->qkv, &cC, &c3C});
        } else {
            launch(r, F_GEMV, (3 * C + 7) / 8, RP_BLOCK, (void *[]){&qkvw, &r->ln, &r->qkv, &cC, &c3C});
            launch(r, F_ABIAS, (3 * C + 255) / 256, RP_BLOCK, (void *[]){&r->qkv, &qkvb, &c3C});
        }
        if (gtrace && l == 0) gdump("qkv", r->qkv, 3 * C);
        RP_CK(cuMemcpyDtoD(kcl + (size_t)pos * C * 4, r->qkv + (size_t)C * 4, C * 4));
        RP_CK(cuMemcpyDtoD(vcl + (size_t)pos * C * 4, r->qkv + (size_t)2 * C * 4, C * 4));
        launch(r, F_ASCORES, (T * G2_NH + 255) / 256, RP_BLOCK, (void *[]){&r->qkv, &kcl, &r->scores, &T, &scale});
        launch(r, F_ASOFTMAX, 1, G2_NH, (void *[]){&r->scores, &r->probs, &T});
        launch(r, F_AMIX, 3, RP_BLOCK, (void *[]){&r->probs, &vcl, &r->att, &T});
        if (gtrace && l == 0) {
            gdump("scores", r->scores, T * G2_NH);
            gdump("probs", r->probs, T * G2_NH);
            gdump("attnout", r->att, C);
        }
        if (r->fused) {
            launch(r, F_GEMVB, (C + 7) / 8, RP_BLOCK, (void *[]){&aow, &r->att, &aob, &r->y, &cC, &cC});
        } else {
            launch(r, F_GEMV, (C + 7) / 8, RP_BLOCK, (void *[]){&aow, &r->att, &r->y, &cC, &cC});
            launch(r, F_ABIAS, (C + 255) / 256, RP_BLOCK, (void *[]){&r->y, &aob, &cC});
        }
        if (gtrace && l == 0) gdump("ao", r->y, C);
        launch(r, F_ADD2, 3, RP_BLOCK, (void *[]){&r->x, &r->y, &r->x, &cC});
        if (gtrace && l == 0) gdump("res1", r->x, C);
        launch(r, F_NORM, 1, RP_BLOCK, (void *[]){&r->x, &ln2w, &ln2b, &r->ln2, &cC, &eps});
        if (gtrace && l == 0) gdump("ln2", r->ln2, C);
        if (r->fused) {
            launch(r, F_GEMVB, (FC + 7) / 8, RP_BLOCK, (void *[]){&fcw, &r->ln2, &fcb, &r->hid, &cC, &cFC});
        } else {
            launch(r, F_GEMV, (FC + 7) / 8, RP_BLOCK, (void *[]){&fcw, &r->ln2, &r->hid, &cC, &cFC});
            launch(r, F_ABIAS, (FC + 255) / 256, RP_BLOCK, (void *[]){&r->hid, &fcb, &cFC});
        }
        if (gtrace && l == 0) gdump("fc", r->hid, FC);
        launch(r, F_GELU, (FC + 255) / 256, RP_BLOCK, (void *[]){&r->hid, &r->hid, &cFC});
        if (gtrace && l == 0) gdump("gelu", r->hid, FC);
        if (r->fused) {
            launch(r, F_GEMVB, (C + 7) / 8, RP_BLOCK, (void *[]){&pw, &r->hid, &pb, &r->y, &cFC, &cC});
        } else {
            launch(r, F_GEMV, (C + 7) / 8, RP_BLOCK, (void *[]){&pw, &r->hid, &r->y, &cFC, &cC});
            launch(r, F_ABIAS, (C + 255) / 256, RP_BLOCK, (void *[]){&r->y, &pb, &cC});
        }
        if (gtrace && l == 0) gdump("proj", r->y, C);
        launch(r, F_ADD2, 3, RP_BLOCK, (void *[]){&r->x, &r->y, &r->x, &cC});
        if (gtrace && l == 0) gdump("res2", r->x, C);
        if (r->trace) RP_CK(cuMemcpyDtoH(r->trace + (size_t)l * C, r->x, C * 4));
    }
    if (!want_logits) return;
    CUdeviceptr lnfw = r->w + G2_OFF_LNFW * 4, lnfb = r->w + G2_OFF_LNFB * 4, wte = r->w;
    launch(r, F_NORM, 1, RP_BLOCK, (void *[]){&r->x, &lnfw, &lnfb, &r->x2, &cC, &eps});
    launch(r, F_GEMV, (G2_V + 7) / 8, RP_BLOCK, (void *[]){&wte, &r->x2, &r->logits, &cC, &cV});
    RP_CK(cuCtxSynchronize());
    if (logits) RP_CK(cuMemcpyDtoH(logits, r->logits, (size_t)G2_V * 4));
}

/* gpt2_engine.c:333-349 */
static void cpu_ln(const float *x, const float *w, const float *b, float *y) {
    float mean = 0.0f, var = 0.0f;
    for (int i = 0; i < G2_C; i++) mean += x[i];
    mean /= G2_C;
    for (int i = 0; i < G2_C; i++) {
        const float d = x[i] - mean;
        var += d * d;
    }
    var /= G2_C;
    const float inv = 1.0f / sqrtf(var + 1e-5f);
    for (int i = 0; i < G2_C; i++) y[i] = (x[i] - mean) * inv * w[i] + b[i];
}
static void cpu_gemv(const float *W, const float *x, const float *bias, float *y, int K, int N) {
    for (int o = 0; o < N; o++) {
        const float *row = W + (size_t)o * K;
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc += row[k] * x[k];
        y[o] = acc + (bias ? bias[o] : 0.0f);
    }
}

/* gpt2_engine.c:363-421 */
static void gpt2_cpu(refpath *r, int token, int pos, int want_logits, float *logits, int debug) {
    const int C = G2_C, HD = G2_HD, FC = G2_FC, ctx = r->ctx;
    const int dump = debug && pos == 0;
    const float *hw = (const float *)r->hw;
    float *x = r->rx, *ln = r->rln, *qkv = r->rqkv, *att = r->ratt, *y = r->ry, *ln2 = r->rln2, *fc = r->rhid;
    float *sc = r->sc;
    for (int i = 0; i < C; i++) x[i] = hw[(size_t)token * C + i] + hw[G2_OFF_WPE + (size_t)pos * C + i];
    for (int l = 0; l < G2_NL; l++) {
        const float *b = hw + G2_LBASE + (size_t)l * G2_LAYER;
        if (dump && l == 0) cdump("embed", x, C);
        cpu_ln(x, b + G2L_LN1W, b + G2L_LN1B, ln);
        if (dump && l == 0) cdump("ln1", ln, C);
        cpu_gemv(b + G2L_QKVW, ln, b + G2L_QKVB, qkv, C, 3 * C);
        if (dump && l == 0) cdump("qkv", qkv, 3 * C);
        float *kc = r->kch + (size_t)l * ctx * C, *vc = r->vch + (size_t)l * ctx * C;
        for (int i = 0; i < C; i++) {
            kc[(size_t)pos * C + i] = qkv[C + i];
            vc[(size_t)pos * C + i] = qkv[2 * C + i];
        }
        for (int h = 0; h < G2_NH; h++) {
            float maxv = -1e30f, sum = 0.0f;
            for (int t = 0; t <= pos; t++) {
                const float *kh = kc + (size_t)t * C + h * HD, *qh = qkv + h * HD;
                float acc = 0.0f;
                for (int d = 0; d < HD; d++) acc += qh[d] * kh[d];
                sc[t] = acc * 0.125f;
                if (sc[t] > maxv) maxv = sc[t];
            }
            for (int t = 0; t <= pos; t++) {
                sc[t] = expf(sc[t] - maxv);
                sum += sc[t];
            }
            for (int d = 0; d < HD; d++) {
                float acc = 0.0f;
                for (int t = 0; t <= pos; t++) acc += sc[t] * vc[(size_t)t * C + h * HD + d];
                att[h * HD + d] = acc / sum;
            }
        }
        cpu_gemv(b + G2L_AOW, att, b + G2L_AOB, y, C, C);
        if (dump && l == 0) cdump("ao", y, C);
        for (int i = 0; i < C; i++) x[i] += y[i];
        if (dump && l == 0) cdump("res1", x, C);
        cpu_ln(x, b + G2L_LN2W, b + G2L_LN2B, ln2);
        if (dump && l == 0) cdump("ln2", ln2, C);
        cpu_gemv(b + G2L_FCW, ln2, b + G2L_FCB, fc, C, FC);
        if (dump && l == 0) cdump("fc", fc, FC);
        for (int i = 0; i < FC; i++) {
            const float v = fc[i], t = 0.7978845608f * (v + 0.044715f * v * v * v);
            fc[i] = 0.5f * v * (1.0f + tanhf(t));
        }
        if (dump && l == 0) cdump("gelu", fc, FC);
        cpu_gemv(b + G2L_PROJW, fc, b + G2L_PROJB, y, FC, C);
        if (dump && l == 0) cdump("proj", y, C);
        for (int i = 0; i < C; i++) x[i] += y[i];
        if (dump && l == 0) cdump("res2", x, C);
        if (r->trace) memcpy(r->trace + (size_t)l * C, x, (size_t)C * 4);
    }
    if (!want_logits) return;
    cpu_ln(x, hw + G2_OFF_LNFW, hw + G2_OFF_LNFB, ln);
    cpu_gemv(hw, ln, NULL, logits, C, G2_V);
}

void rp_forward(refpath *r, int token, int pos, int want_logits, float *logits, int debug) {
    if (pos < 0 || pos >= r->ctx || token < 0 || token >= r->V) {
        fprintf(stderr, "token %d / position %d out of range\n", token, pos);
        exit(1);
    }
    rp_device(r);
    if (r->model == SB_MODEL_QWEN) qwen_forward(r, token, pos, want_logits, logits, debug);
    else gpt2_forward(r, token, pos, want_logits, logits, debug);
}

void rp_cpu_forward(refpath *r, int token, int pos, int want_logits, float *logits, int debug) {
    if (pos < 0 || pos >= r->ctx || token < 0 || token >= r->V) {
        fprintf(stderr, "token %d / position %d out of range\n", token, pos);
        exit(1);
    }
    if (!r->kch) rp_host_buffers(r);
    if (r->model == SB_MODEL_QWEN) qwen_cpu(r, token, pos, want_logits, logits, debug);
    else gpt2_cpu(r, token, pos, want_logits, logits, debug);
}

void rp_set_fused(refpath *r, int fused) { r->fused = fused; }
void rp_set_trace(refpath *r, float *buf) { r->trace = buf; }
