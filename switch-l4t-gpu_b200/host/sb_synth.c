/* sb_synth.c -- deterministic synthetic inputs in the reference's formats.
 *
 * Real checkpoints are not used; weights are N(0, 0.02) with unit norm
 * gains and zero LayerNorm betas, written in exactly the flat layouts the
 * reference's converters produce (conv_qwen.py:63-99, conv_gpt2.py:150-168),
 * so the reference engines and this package read the same files.
 *
 * Every tensor is generated in 1 Mi-element blocks; block b of tensor t uses
 * its own splitmix64 stream seeded from (seed, t, b), so the bytes do not
 * depend on the number of threads.  Normals use Box-Muller in double. */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "../../include/switch_b200.h"
#include "sb_models.h"

static uint64_t sm64_next(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static double u01(uint64_t *s) { return ((sm64_next(s) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
static uint64_t mix(uint64_t a, uint64_t b) {
    uint64_t s = a ^ (b * 0xD1B54A32D192ED03ull);
    return sm64_next(&s);
}

static uint16_t f2h(float f) {
    _Float16 h = (_Float16)f; /* IEEE round-to-nearest-even */
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

enum { K_NORMAL_F32, K_NORMAL_F16, K_CONST_F32, K_CONST_F16 };
typedef struct {
    int kind;
    float stdv;
    float cval;
    uint64_t stream; /* per-tensor seed */
    size_t n;
    void *out;
} gen_job;

#define BLK ((size_t)1 << 20)

static void gen_block(const gen_job *j, size_t b) {
    size_t lo = b * BLK, hi = lo + BLK < j->n ? lo + BLK : j->n;
    if (j->kind == K_CONST_F32) {
        for (size_t i = lo; i < hi; i++) ((float *)j->out)[i] = j->cval;
        return;
    }
    if (j->kind == K_CONST_F16) {
        uint16_t h = f2h(j->cval);
        for (size_t i = lo; i < hi; i++) ((uint16_t *)j->out)[i] = h;
        return;
    }
    uint64_t s = mix(j->stream, b);
    for (size_t i = lo; i < hi; i += 2) {
        double r = sqrt(-2.0 * log(u01(&s))), t = 6.283185307179586 * u01(&s);
        float z0 = (float)(r * cos(t) * j->stdv), z1 = (float)(r * sin(t) * j->stdv);
        if (j->kind == K_NORMAL_F32) {
            ((float *)j->out)[i] = z0;
            if (i + 1 < hi) ((float *)j->out)[i + 1] = z1;
        } else {
            ((uint16_t *)j->out)[i] = f2h(z0);
            if (i + 1 < hi) ((uint16_t *)j->out)[i + 1] = f2h(z1);
        }
    }
}

typedef struct {
    const gen_job *j;
    size_t nblk;
    int tid, nth;
} gen_thread_arg;
static void *gen_thread(void *p) {
    gen_thread_arg *a = p;
    for (size_t b = a->tid; b < a->nblk; b += a->nth) gen_block(a->j, b);
    return NULL;
}

static void run_job(const gen_job *j) {
    size_t nblk = (j->n + BLK - 1) / BLK;
    int nth = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nth < 1) nth = 1;
    if (nth > 64) nth = 64;
    if ((size_t)nth > nblk) nth = (int)nblk;
    if (nth <= 1) {
        for (size_t b = 0; b < nblk; b++) gen_block(j, b);
        return;
    }
    pthread_t th[64];
    gen_thread_arg args[64];
    for (int t = 0; t < nth; t++) {
        args[t] = (gen_thread_arg){j, nblk, t, nth};
        pthread_create(&th[t], NULL, gen_thread, &args[t]);
    }
    for (int t = 0; t < nth; t++) pthread_join(th[t], NULL);
}

/* write one tensor; `tensor_id` distinguishes streams within a file */
static int emit(FILE *f, void *buf, int kind, size_t n, float stdv, float cval, uint64_t seed, uint64_t tensor_id) {
    gen_job j = {kind, stdv, cval, mix(seed, tensor_id), n, buf};
    run_job(&j);
    size_t esz = (kind == K_NORMAL_F16 || kind == K_CONST_F16) ? 2 : 4;
    return fwrite(buf, esz, n, f) == n ? 0 : -1;
}

static long synth_qwen(FILE *f, uint64_t seed) {
    const size_t big = (size_t)QW_V * QW_C; /* largest tensor (embedding) */
    void *buf = malloc(big * 2);
    if (!buf) return -1;
    long rc = 0;
    uint64_t tid = 0;
    rc |= emit(f, buf, K_NORMAL_F16, big, 0.02f, 0, seed, tid++);
    /* RoPE tables: freq_d = theta^(-2d/HD), angle = pos * freq_d (conv_qwen.py:75-80) */
    float *cs = malloc((size_t)QW_CTX_FILE * (QW_HD / 2) * 4);
    for (int which = 0; which < 2 && cs; which++) {
        for (int p = 0; p < QW_CTX_FILE; p++)
            for (int d = 0; d < QW_HD / 2; d++) {
                double freq = pow(1000000.0, -2.0 * d / QW_HD);
                double ang = (double)p * freq;
                cs[(size_t)p * (QW_HD / 2) + d] = (float)(which == 0 ? cos(ang) : sin(ang));
            }
        if (fwrite(cs, 4, (size_t)QW_CTX_FILE * (QW_HD / 2), f) != (size_t)QW_CTX_FILE * (QW_HD / 2)) rc = -1;
    }
    free(cs);
    for (int l = 0; l < QW_NL; l++) {
        rc |= emit(f, buf, K_CONST_F16, QW_C, 0, 1.0f, seed, tid++);                          /* in_ln */
        rc |= emit(f, buf, K_NORMAL_F16, (size_t)QW_QKV * QW_C, 0.02f, 0, seed, tid++);       /* qkv_w */
        rc |= emit(f, buf, K_NORMAL_F16, QW_QKV, 0.02f, 0, seed, tid++);                      /* qkv_b */
        rc |= emit(f, buf, K_NORMAL_F16, (size_t)QW_C * QW_C, 0.02f, 0, seed, tid++);         /* o_w */
        rc |= emit(f, buf, K_CONST_F16, QW_C, 0, 1.0f, seed, tid++);                          /* post_ln */
        rc |= emit(f, buf, K_NORMAL_F16, (size_t)2 * QW_FC * QW_C, 0.02f, 0, seed, tid++);    /* gate|up */
        rc |= emit(f, buf, K_NORMAL_F16, (size_t)QW_C * QW_FC, 0.02f, 0, seed, tid++);        /* down */
    }
    rc |= emit(f, buf, K_CONST_F16, QW_C, 0, 1.0f, seed, tid++); /* final norm */
    free(buf);
    return rc ? -1 : (long)QW_FILE_BYTES;
}

static long synth_gpt2(FILE *f, uint64_t seed) {
    const size_t big = (size_t)G2_V * G2_C;
    float *buf = malloc(big * 4);
    if (!buf) return -1;
    long rc = 0;
    uint64_t tid = 0;
    rc |= emit(f, buf, K_NORMAL_F32, big, 0.02f, 0, seed, tid++);                        /* wte */
    rc |= emit(f, buf, K_NORMAL_F32, (size_t)G2_CTX * G2_C, 0.02f, 0, seed, tid++);      /* wpe */
    for (int l = 0; l < G2_NL; l++) {
        rc |= emit(f, buf, K_CONST_F32, G2_C, 0, 1.0f, seed, tid++);                     /* ln1_w */
        rc |= emit(f, buf, K_CONST_F32, G2_C, 0, 0.0f, seed, tid++);                     /* ln1_b */
        rc |= emit(f, buf, K_NORMAL_F32, (size_t)3 * G2_C * G2_C, 0.02f, 0, seed, tid++);/* qkv_w */
        rc |= emit(f, buf, K_NORMAL_F32, 3 * G2_C, 0.02f, 0, seed, tid++);              /* qkv_b */
        rc |= emit(f, buf, K_NORMAL_F32, (size_t)G2_C * G2_C, 0.02f, 0, seed, tid++);    /* ao_w */
        rc |= emit(f, buf, K_NORMAL_F32, G2_C, 0.02f, 0, seed, tid++);                   /* ao_b */
        rc |= emit(f, buf, K_CONST_F32, G2_C, 0, 1.0f, seed, tid++);                     /* ln2_w */
        rc |= emit(f, buf, K_CONST_F32, G2_C, 0, 0.0f, seed, tid++);                     /* ln2_b */
        rc |= emit(f, buf, K_NORMAL_F32, (size_t)G2_FC * G2_C, 0.02f, 0, seed, tid++);   /* fc_w */
        rc |= emit(f, buf, K_NORMAL_F32, G2_FC, 0.02f, 0, seed, tid++);                  /* fc_b */
        rc |= emit(f, buf, K_NORMAL_F32, (size_t)G2_FC * G2_C, 0.02f, 0, seed, tid++);   /* proj_w */
        rc |= emit(f, buf, K_NORMAL_F32, G2_C, 0.02f, 0, seed, tid++);                   /* proj_b */
    }
    rc |= emit(f, buf, K_CONST_F32, G2_C, 0, 1.0f, seed, tid++); /* ln_f w */
    rc |= emit(f, buf, K_CONST_F32, G2_C, 0, 0.0f, seed, tid++); /* ln_f b */
    free(buf);
    return rc ? -1 : (long)G2_TOTAL_FLOATS * 4;
}

long sb_synth_weights(int model, const char *path, uint64_t seed) {
    if (model != SB_MODEL_QWEN && model != SB_MODEL_GPT2) return -1;
    FILE *f = fopen(path, "wb");
    if (!f) return -1;
    long n = model == SB_MODEL_QWEN ? synth_qwen(f, seed) : synth_gpt2(f, seed);
    if (fclose(f) != 0) n = -1;
    return n;
}

void sb_synth_ids(int *ids, int n, int vocab, uint64_t seed) {
    uint64_t s = mix(seed, 0x1d5);
    for (int i = 0; i < n; i++) ids[i] = (int)(sm64_next(&s) % (uint64_t)vocab);
}

void sb_synth_uniform(float *out, size_t n, float lo, float hi, uint64_t seed) {
    uint64_t s = mix(seed, 0xa11);
    for (size_t i = 0; i < n; i++) out[i] = (float)(lo + (hi - lo) * ((sm64_next(&s) >> 40) * (1.0 / 16777216.0)));
}

void sb_synth_normal_h(uint16_t *out, size_t n, float stdv, uint64_t seed) {
    gen_job j = {K_NORMAL_F16, stdv, 0, mix(seed, 0x4e), n, out};
    run_job(&j);
}
