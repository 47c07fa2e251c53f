/* oracle.c -- CPU restatement of the reference golden models.  TEST
 * INFRASTRUCTURE ONLY (see oracle.h).  Build with -O2 -ffp-contract=off. */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <fcntl.h>
#include <unistd.h>

/* ------------------------------------------------------------------ util */
float orc_h2f(uint16_t h) {
    /* qwen_engine.c:90-98: exponent 0 -> 0 (subnormals flushed). */
    uint32_t e = (h >> 10) & 0x1fu;
    if (e == 0) return 0.0f;
    union { uint32_t u; float f; } cvt;
    cvt.u = ((uint32_t)(h & 0x8000u) << 16) | ((e - 15u + 127u) << 23) |
            ((uint32_t)(h & 0x3ffu) << 13);
    return cvt.f;
}

int orc_argmax(const float *v, int n) {
    int b = 0;
    float m = v[0];
    for (int i = 1; i < n; i++)
        if (v[i] > m) { m = v[i]; b = i; }
    return b;
}

/* Generic row-range thread pool: fn(ctx, r0, r1) over [0,n). */
typedef void (*row_fn)(void *ctx, int r0, int r1);
typedef struct { row_fn fn; void *ctx; int r0, r1; } row_job;
static void *row_thread(void *p) {
    row_job *j = (row_job *)p;
    j->fn(j->ctx, j->r0, j->r1);
    return NULL;
}
static void parallel_rows(row_fn fn, void *ctx, int n, int nthreads) {
    if (nthreads <= 1 || n < 2 * nthreads) { fn(ctx, 0, n); return; }
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    row_job jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].r0 = (int)((long)n * t / nthreads);
        jobs[t].r1 = (int)((long)n * (t + 1) / nthreads);
        pthread_create(&th[t], NULL, row_thread, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------ SGEMM */
typedef struct { const float *A, *B; float *C; int N, K, row0; } sg_ctx;
static void sg_rows(void *p, int r0, int r1) {
    sg_ctx *c = (sg_ctx *)p;
    int N = c->N, K = c->K;
    for (int i = c->row0 + r0; i < c->row0 + r1; i++)
        for (int j = 0; j < N; j++) {
            /* gpu_workload.c:97-98 */
            float ref = 0;
            for (int k = 0; k < K; k++) ref += c->A[(size_t)i * K + k] * c->B[(size_t)k * N + j];
            c->C[(size_t)i * N + j] = ref;
        }
}
void orc_sgemm_rows(const float *A, const float *B, float *C, int M, int N, int K,
                    int row0, int row1, int nthreads) {
    (void)M;
    sg_ctx c = {A, B, C, N, K, row0};
    parallel_rows(sg_rows, &c, row1 - row0, nthreads);
}

int orc_sgemm_bad_cells(const float *got, const float *ref, size_t n) {
    int bad = 0;
    for (size_t i = 0; i < n; i++) {
        float d = got[i] - ref[i];
        if (d < 0) d = -d;
        float r = ref[i] < 0 ? -ref[i] : ref[i];
        if (d > 0.05f * r + 1e-3f) bad++;
    }
    return bad;
}

static uint64_t sm64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct { const float *X; const double *v; double *out; int cols; } mv_ctx;
static void mv_rows(void *p, int r0, int r1) {
    mv_ctx *c = (mv_ctx *)p;
    for (int i = r0; i < r1; i++) {
        double s = 0;
        const float *row = c->X + (size_t)i * c->cols;
        for (int k = 0; k < c->cols; k++) s += (double)row[k] * c->v[k];
        c->out[i] = s;
    }
}
double orc_freivalds(const float *A, const float *B, const float *C, int M, int N, int K,
                     uint64_t seed, int nthreads) {
    double *r = malloc(sizeof(double) * N), *br = malloc(sizeof(double) * K);
    double *abr = malloc(sizeof(double) * M), *cr = malloc(sizeof(double) * M);
    uint64_t s = seed;
    for (int j = 0; j < N; j++) r[j] = (sm64(&s) >> 63) ? 1.0 : -1.0;
    mv_ctx c1 = {B, r, br, N};
    parallel_rows(mv_rows, &c1, K, nthreads);
    mv_ctx c2 = {A, br, abr, K};
    parallel_rows(mv_rows, &c2, M, nthreads);
    mv_ctx c3 = {C, r, cr, N};
    parallel_rows(mv_rows, &c3, M, nthreads);
    double num = 0, den = 0;
    for (int i = 0; i < M; i++) {
        num += (cr[i] - abr[i]) * (cr[i] - abr[i]);
        den += abr[i] * abr[i];
    }
    free(r); free(br); free(abr); free(cr);
    return sqrt(num) / fmax(sqrt(den), 1e-300);
}

/* ------------------------------------------------------------------ GEMV */
typedef struct { const float *W, *x, *bias; float *y; int K; } gf_ctx;
static void gf_rows(void *p, int r0, int r1) {
    gf_ctx *c = (gf_ctx *)p;
    for (int o = r0; o < r1; o++) {
        const float *row = c->W + (size_t)o * c->K;
        float acc = 0.0f;
        for (int k = 0; k < c->K; k++) acc += row[k] * c->x[k];
        c->y[o] = acc + (c->bias ? c->bias[o] : 0.0f);
    }
}
void orc_gemv_f32(const float *W, const float *x, const float *bias, float *y, int K, int N,
                  int nthreads) {
    gf_ctx c = {W, x, bias, y, K};
    parallel_rows(gf_rows, &c, N, nthreads);
}
void orc_gemv_multi_f32(const float *W, const float *X, const float *bias, float *Y, int K,
                        int N, int T, int nthreads) {
    for (int t = 0; t < T; t++)
        orc_gemv_f32(W, X + (size_t)t * K, bias, Y + (size_t)t * N, K, N, nthreads);
}

typedef struct { const uint16_t *W; const float *x, *bias; float *y; int K; } gh_ctx;
static void gh_rows(void *p, int r0, int r1) {
    gh_ctx *c = (gh_ctx *)p;
    for (int o = r0; o < r1; o++) {
        const uint16_t *row = c->W + (size_t)o * c->K;
        float acc = 0.0f;
        for (int k = 0; k < c->K; k++) acc += orc_h2f(row[k]) * c->x[k];
        c->y[o] = acc + (c->bias ? c->bias[o] : 0.0f);
    }
}
void orc_gemv_h(const uint16_t *W, const float *x, const float *bias, float *y, int K, int N,
                int nthreads) {
    gh_ctx c = {W, x, bias, y, K};
    parallel_rows(gh_rows, &c, N, nthreads);
}

/* ------------------------------------------------------------------ elementwise */
void orc_rmsnorm(const float *x, const uint16_t *w, float *y, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * inv * orc_h2f(w[i]);
}

void orc_layernorm(const float *x, const float *w, const float *b, float *y, int n, float eps) {
    float mean = 0.0f, var = 0.0f;
    for (int i = 0; i < n; i++) mean += x[i];
    mean /= n;
    for (int i = 0; i < n; i++) { float d = x[i] - mean; var += d * d; }
    var /= n;
    float inv = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < n; i++) y[i] = (x[i] - mean) * inv * w[i] + b[i];
}

void orc_rope(float *x, const float *cosT, const float *sinT, int T, int H, int HD, int pos0) {
    int hd2 = HD / 2;
    for (int t = 0; t < T; t++) {
        float *row = x + (size_t)t * H * HD;
        for (int h = 0; h < H; h++)
            for (int i = 0; i < hd2; i++) {
                float a = row[h * HD + i], b2 = row[h * HD + hd2 + i];
                float c = cosT[(size_t)(pos0 + t) * hd2 + i], s = sinT[(size_t)(pos0 + t) * hd2 + i];
                row[h * HD + i] = a * c - b2 * s;
                row[h * HD + hd2 + i] = a * s + b2 * c;
            }
    }
}

void orc_swiglu(const float *g, const float *u, float *y, int n) {
    for (int i = 0; i < n; i++) y[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

void orc_gelu(const float *x, float *y, int n) {
    for (int i = 0; i < n; i++) {
        float v = x[i];
        float t = 0.7978845608f * (v + 0.044715f * v * v * v);
        y[i] = 0.5f * v * (1.0f + tanhf(t));
    }
}

void orc_attn_qwen(const float *q, const float *kc, const float *vc, float *out, int T, int NH,
                   int NKV, int HD, int kv_stride, float scale) {
    float *sc = malloc(sizeof(float) * (T > 0 ? T : 1));
    for (int h = 0; h < NH; h++) {
        int g = h / (NH / NKV);
        float maxv = -1e30f;
        for (int t = 0; t < T; t++) {
            float acc = 0.0f;
            for (int d = 0; d < HD; d++) acc += q[h * HD + d] * kc[(size_t)t * kv_stride + g * HD + d];
            sc[t] = acc * scale;
            if (sc[t] > maxv) maxv = sc[t];
        }
        float sum = 0.0f;
        for (int t = 0; t < T; t++) { sc[t] = expf(sc[t] - maxv); sum += sc[t]; }
        for (int d = 0; d < HD; d++) {
            float acc = 0.0f;
            for (int t = 0; t < T; t++) acc += (sc[t] / sum) * vc[(size_t)t * kv_stride + g * HD + d];
            out[h * HD + d] = acc;
        }
    }
    free(sc);
}

void orc_attn_gpt2(const float *q, const float *kc, const float *vc, float *out, int T, int NH,
                   int HD, int kv_stride, float scale) {
    float *sc = malloc(sizeof(float) * (T > 0 ? T : 1));
    for (int h = 0; h < NH; h++) {
        float maxv = -1e30f, sum = 0.0f;
        for (int t = 0; t < T; t++) {
            const float *kh = kc + (size_t)t * kv_stride + h * HD;
            const float *qh = q + h * HD;
            float acc = 0.0f;
            for (int d = 0; d < HD; d++) acc += qh[d] * kh[d];
            sc[t] = acc * scale;
            if (sc[t] > maxv) maxv = sc[t];
        }
        for (int t = 0; t < T; t++) { sc[t] = expf(sc[t] - maxv); sum += sc[t]; }
        for (int d = 0; d < HD; d++) {
            float acc = 0.0f;
            for (int t = 0; t < T; t++) acc += sc[t] * vc[(size_t)t * kv_stride + h * HD + d];
            out[h * HD + d] = acc / sum;
        }
    }
    free(sc);
}

/* ------------------------------------------------------------------ file map */
static void *map_file(const char *path, size_t want, size_t *got) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st) != 0 || (want && (size_t)st.st_size != want)) { close(fd); return NULL; }
    void *p = mmap(NULL, st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return NULL;
    *got = st.st_size;
    return p;
}

/* ------------------------------------------------------------------ Qwen */
/* Dims and byte layout restated from qwen_engine.c:43-75 (conv_qwen.py:63-99). */
#define QV 151936
#define QC 896
#define QNL 24
#define QNH 14
#define QNKV 2
#define QHD 64
#define QKVD (QNKV * QHD)
#define QQKV (QC + 2 * QKVD)
#define QFC 4864
#define QCTXF 8192
#define Q_OFF_COS ((size_t)QV * QC * 2)
#define Q_OFF_SIN (Q_OFF_COS + (size_t)QCTXF * (QHD / 2) * 4)
#define Q_LBASE (Q_OFF_SIN + (size_t)QCTXF * (QHD / 2) * 4)
#define Q_LSTRIDE ((size_t)(QC + QQKV * QC + QQKV + QC * QC + QC + 2 * QFC * QC + QC * QFC) * 2)
#define Q_OFF_LNF (Q_LBASE + (size_t)QNL * Q_LSTRIDE)
#define Q_FILE (Q_OFF_LNF + (size_t)QC * 2)
/* per-layer fp16 element offsets (qwen_engine.c:69-75) */
#define QI_INLN 0
#define QI_QKVW ((size_t)QC)
#define QI_QKVB ((size_t)QC + (size_t)QQKV * QC)
#define QI_OW (QI_QKVB + QQKV)
#define QI_POST (QI_OW + (size_t)QC * QC)
#define QI_GATEUP (QI_POST + QC)
#define QI_DOWN (QI_GATEUP + (size_t)2 * QFC * QC)

struct orc_qwen {
    const uint8_t *file;
    size_t size;
    int ctx;
    float *kc, *vc; /* [NL][ctx][KVD] */
    float x[QC], ln[QC], qkv[QQKV], att[QC], y[QC], ln2[QC], gate[2 * QFC], down[QFC];
    float qkvb[QNL][QQKV];
};

orc_qwen *orc_qwen_open(const char *path, int ctx) {
    size_t got = 0;
    const uint8_t *f = map_file(path, Q_FILE, &got);
    if (!f) return NULL;
    orc_qwen *m = calloc(1, sizeof(*m));
    m->file = f; m->size = got; m->ctx = ctx;
    m->kc = calloc((size_t)QNL * ctx * QKVD, sizeof(float));
    m->vc = calloc((size_t)QNL * ctx * QKVD, sizeof(float));
    for (int l = 0; l < QNL; l++) {
        const uint16_t *b = (const uint16_t *)(f + Q_LBASE + (size_t)l * Q_LSTRIDE);
        for (int i = 0; i < QQKV; i++) m->qkvb[l][i] = orc_h2f(b[QI_QKVB + i]);
    }
    return m;
}
void orc_qwen_reset(orc_qwen *m) {
    memset(m->kc, 0, sizeof(float) * (size_t)QNL * m->ctx * QKVD);
    memset(m->vc, 0, sizeof(float) * (size_t)QNL * m->ctx * QKVD);
}
const float *orc_qwen_residual(const orc_qwen *m) { return m->x; }
float *orc_qwen_kv(orc_qwen *m, int which) { return which ? m->vc : m->kc; }
void orc_qwen_close(orc_qwen *m) {
    if (!m) return;
    munmap((void *)m->file, m->size);
    free(m->kc); free(m->vc); free(m);
}

void orc_qwen_forward(orc_qwen *m, int token, int pos, int want_logits, float *logits,
                      int nthreads) {
    const uint16_t *emb = (const uint16_t *)m->file;
    const float *cosT = (const float *)(m->file + Q_OFF_COS);
    const float *sinT = (const float *)(m->file + Q_OFF_SIN);
    const float EPS = 1e-6f, SCALE = 0.125f;
    for (int i = 0; i < QC; i++) m->x[i] = orc_h2f(emb[(size_t)token * QC + i]);
    for (int l = 0; l < QNL; l++) {
        const uint16_t *b = (const uint16_t *)(m->file + Q_LBASE + (size_t)l * Q_LSTRIDE);
        float *kc = m->kc + (size_t)l * m->ctx * QKVD, *vc = m->vc + (size_t)l * m->ctx * QKVD;
        orc_rmsnorm(m->x, b + QI_INLN, m->ln, QC, EPS);
        orc_gemv_h(b + QI_QKVW, m->ln, m->qkvb[l], m->qkv, QC, QQKV, nthreads);
        orc_rope(m->qkv, cosT, sinT, 1, QNH, QHD, pos);        /* q heads */
        orc_rope(m->qkv + QC, cosT, sinT, 1, QNKV, QHD, pos);  /* k heads */
        for (int i = 0; i < QKVD; i++) {
            kc[(size_t)pos * QKVD + i] = m->qkv[QC + i];
            vc[(size_t)pos * QKVD + i] = m->qkv[QC + QKVD + i];
        }
        orc_attn_qwen(m->qkv, kc, vc, m->att, pos + 1, QNH, QNKV, QHD, QKVD, SCALE);
        orc_gemv_h(b + QI_OW, m->att, NULL, m->y, QC, QC, nthreads);
        for (int i = 0; i < QC; i++) m->x[i] += m->y[i];
        orc_rmsnorm(m->x, b + QI_POST, m->ln2, QC, EPS);
        orc_gemv_h(b + QI_GATEUP, m->ln2, NULL, m->gate, QC, 2 * QFC, nthreads);
        orc_swiglu(m->gate, m->gate + QFC, m->down, QFC);
        orc_gemv_h(b + QI_DOWN, m->down, NULL, m->y, QFC, QC, nthreads);
        for (int i = 0; i < QC; i++) m->x[i] += m->y[i];
    }
    if (!want_logits) return;
    orc_rmsnorm(m->x, (const uint16_t *)(m->file + Q_OFF_LNF), m->ln, QC, EPS);
    orc_gemv_h(emb, m->ln, NULL, logits, QC, QV, nthreads);
}

/* ------------------------------------------------------------------ GPT-2 */
/* Dims and float layout restated from gpt2_engine.c:40-70 (conv_gpt2.py:150-155). */
#define GV 50257
#define GC 768
#define GNH 12
#define GHD 64
#define GNL 12
#define GCTX 1024
#define GFC 3072
#define G_LAYER (2 * GC + 3 * GC * GC + 3 * GC + GC * GC + GC + 2 * GC + GFC * GC + GFC + GFC * GC + GC)
#define G_OFF_WPE ((size_t)GV * GC)
#define G_LBASE (G_OFF_WPE + (size_t)GCTX * GC)
#define G_OFF_LNFW (G_LBASE + (size_t)GNL * G_LAYER)
#define G_OFF_LNFB (G_OFF_LNFW + GC)
#define G_TOTAL (G_OFF_LNFB + GC)
#define GL_LN1W 0
#define GL_LN1B (GL_LN1W + GC)
#define GL_QKVW (GL_LN1B + GC)
#define GL_QKVB (GL_QKVW + 3 * GC * GC)
#define GL_AOW (GL_QKVB + 3 * GC)
#define GL_AOB (GL_AOW + GC * GC)
#define GL_LN2W (GL_AOB + GC)
#define GL_LN2B (GL_LN2W + GC)
#define GL_FCW (GL_LN2B + GC)
#define GL_FCB (GL_FCW + GFC * GC)
#define GL_PROJW (GL_FCB + GFC)
#define GL_PROJB (GL_PROJW + GFC * GC)

struct orc_gpt2 {
    const float *w;
    size_t size;
    int ctx;
    float *kc, *vc; /* [NL][ctx][C] */
    float x[GC], ln[GC], qkv[3 * GC], att[GC], y[GC], ln2[GC], fc[GFC];
};

orc_gpt2 *orc_gpt2_open(const char *path, int ctx) {
    size_t got = 0;
    const float *f = map_file(path, (size_t)G_TOTAL * 4, &got);
    if (!f) return NULL;
    orc_gpt2 *m = calloc(1, sizeof(*m));
    m->w = f; m->size = got; m->ctx = ctx;
    m->kc = calloc((size_t)GNL * ctx * GC, sizeof(float));
    m->vc = calloc((size_t)GNL * ctx * GC, sizeof(float));
    return m;
}
void orc_gpt2_reset(orc_gpt2 *m) {
    memset(m->kc, 0, sizeof(float) * (size_t)GNL * m->ctx * GC);
    memset(m->vc, 0, sizeof(float) * (size_t)GNL * m->ctx * GC);
}
const float *orc_gpt2_residual(const orc_gpt2 *m) { return m->x; }
float *orc_gpt2_kv(orc_gpt2 *m, int which) { return which ? m->vc : m->kc; }
void orc_gpt2_close(orc_gpt2 *m) {
    if (!m) return;
    munmap((void *)m->w, m->size);
    free(m->kc); free(m->vc); free(m);
}

void orc_gpt2_forward(orc_gpt2 *m, int token, int pos, int want_logits, float *logits,
                      int nthreads) {
    const float *w = m->w;
    for (int i = 0; i < GC; i++)
        m->x[i] = w[(size_t)token * GC + i] + w[G_OFF_WPE + (size_t)pos * GC + i];
    for (int l = 0; l < GNL; l++) {
        const float *b = w + G_LBASE + (size_t)l * G_LAYER;
        float *kc = m->kc + (size_t)l * m->ctx * GC, *vc = m->vc + (size_t)l * m->ctx * GC;
        orc_layernorm(m->x, b + GL_LN1W, b + GL_LN1B, m->ln, GC, 1e-5f);
        orc_gemv_f32(b + GL_QKVW, m->ln, b + GL_QKVB, m->qkv, GC, 3 * GC, nthreads);
        for (int i = 0; i < GC; i++) {
            kc[(size_t)pos * GC + i] = m->qkv[GC + i];
            vc[(size_t)pos * GC + i] = m->qkv[2 * GC + i];
        }
        orc_attn_gpt2(m->qkv, kc, vc, m->att, pos + 1, GNH, GHD, GC, 0.125f);
        orc_gemv_f32(b + GL_AOW, m->att, b + GL_AOB, m->y, GC, GC, nthreads);
        for (int i = 0; i < GC; i++) m->x[i] += m->y[i];
        orc_layernorm(m->x, b + GL_LN2W, b + GL_LN2B, m->ln2, GC, 1e-5f);
        orc_gemv_f32(b + GL_FCW, m->ln2, b + GL_FCB, m->fc, GC, GFC, nthreads);
        orc_gelu(m->fc, m->fc, GFC);
        orc_gemv_f32(b + GL_PROJW, m->fc, b + GL_PROJB, m->y, GFC, GC, nthreads);
        for (int i = 0; i < GC; i++) m->x[i] += m->y[i];
    }
    if (!want_logits) return;
    orc_layernorm(m->x, w + G_OFF_LNFW, w + G_OFF_LNFB, m->ln, GC, 1e-5f);
    orc_gemv_f32(w, m->ln, NULL, logits, GC, GV, nthreads);
}
