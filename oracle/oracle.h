/* oracle.h -- CPU restatement of pkia/switch-l4t-gpu's golden models.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA kernels, the
 * C-ABI library, the C hosts, bench.py's GPU arms) links or calls this code.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it,
 * and only as the checker.
 *
 * Every function restates the reference's serial C arithmetic in the same
 * order (float accumulation, left-to-right products, libm expf/tanhf/sqrtf),
 * compiled with -ffp-contract=off so no multiply-add is fused.  The threaded
 * variants split OUTPUT ROWS (or heads) across threads; each output is still
 * computed by exactly the serial loop, so results are bit-identical to the
 * single-thread call.
 *
 * Parity pin: the restatement is checked against the reference's own C
 * (gpu-llm/engine/{qwen,gpt2}_engine.c compiled unmodified into oracle/_ref
 * with stubbed driver calls) and against fixtures in tests/golden/ that were
 * generated from it.
 */
#ifndef SB_ORACLE_H
#define SB_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp16 bits -> float with exponent-0 flushed to zero and no inf/NaN handling
 * (gpu-llm/engine/qwen_engine.c:90-98). */
float orc_h2f(uint16_t h);

/* SGEMM triple loop, C[i][j] = sum_k A[i][k]*B[k][j], float accumulation in k
 * order (gpu_workload.c:96-98).  Rows [row0,row1) only; nthreads<=1 = serial. */
void orc_sgemm_rows(const float *A, const float *B, float *C, int M, int N, int K,
                    int row0, int row1, int nthreads);

/* Harness tolerance check of gpu_workload.c:99-101: |d| > 0.05|ref| + 1e-3. */
int orc_sgemm_bad_cells(const float *got, const float *ref, size_t n);

/* Freivalds in double: returns ||C r - A (B r)||_2 / ||A (B r)||_2 for a
 * +-1 vector r from `seed` (about 1e-6 for a correct FP32 product; O(1) for
 * a wrong tile). */
double orc_freivalds(const float *A, const float *B, const float *C, int M, int N, int K,
                     uint64_t seed, int nthreads);

/* FP32 GEMV y[n] = sum_k W[n][k] x[k] (+bias[n]); gemv_test.c:85-90 and
 * cpu_gemv gpt2_engine.c:342-349 (bias may be NULL). */
void orc_gemv_f32(const float *W, const float *x, const float *bias, float *y,
                  int K, int N, int nthreads);

/* Batched FP32 GEMV, Y[t][n] = sum_k W[n][k] X[t][k] + bias[n]: the per-token
 * cpu_gemv of gpt2_engine.c:342-349 applied to each row of X (the arithmetic
 * gemv_multi, gpt2_kernels.cu:115-155, must reproduce). */
void orc_gemv_multi_f32(const float *W, const float *X, const float *bias, float *Y,
                        int K, int N, int T, int nthreads);

/* FP16-weight GEMV, cpu_gemv_h (qwen_engine.c:276-284).  `bias` is the fp16
 * bias already decoded to float (qwen_engine.c:170-175) or NULL. */
void orc_gemv_h(const uint16_t *W, const float *x, const float *bias, float *y,
                int K, int N, int nthreads);

/* cpu_rms (qwen_engine.c:285-290) with fp16 weight. */
void orc_rmsnorm(const float *x, const uint16_t *w, float *y, int n, float eps);
/* cpu_ln (gpt2_engine.c:333-341), centred two-pass variance, eps given. */
void orc_layernorm(const float *x, const float *w, const float *b, float *y, int n, float eps);
/* RoPE half-split rotation of rows [T][H*HD] at positions pos0.. using the
 * [CTX][HD/2] tables (qwen_engine.c:302-317; qwen_kernels.cu:97-116). */
void orc_rope(float *x, const float *cosT, const float *sinT, int T, int H, int HD, int pos0);
/* SiLU-gated product (qwen_engine.c:349-350). */
void orc_swiglu(const float *g, const float *u, float *y, int n);
/* tanh-GELU (gpt2_engine.c:406-410). */
void orc_gelu(const float *x, float *y, int n);

/* Decode attention over cached positions 0..T-1, one query token.
 * Qwen form (qwen_engine.c:324-342): out = sum_t (p_t/sum) v_t, GQA groups.
 * kc/vc rows have stride `kv_stride` floats; head h reads group h/(NH/NKV). */
void orc_attn_qwen(const float *q, const float *kc, const float *vc, float *out,
                   int T, int NH, int NKV, int HD, int kv_stride, float scale);
/* GPT-2 form (gpt2_engine.c:379-397): out = (sum_t p_t v_t)/sum, MHA. */
void orc_attn_gpt2(const float *q, const float *kc, const float *vc, float *out,
                   int T, int NH, int HD, int kv_stride, float scale);

/* Engine-level golden forwards over a weight FILE in the reference layout. */
typedef struct orc_qwen orc_qwen;
orc_qwen *orc_qwen_open(const char *path, int ctx);
void orc_qwen_reset(orc_qwen *m);
/* One decode step (token at pos; cache gains pos).  logits (V floats) written
 * when want_logits.  Restates cpu_forward, qwen_engine.c:292-358. */
void orc_qwen_forward(orc_qwen *m, int token, int pos, int want_logits, float *logits,
                      int nthreads);
/* Residual stream after the last forward's layers (C floats). */
const float *orc_qwen_residual(const orc_qwen *m);
/* The model's KV cache, which 0: keys, 1: values, each [NL][ctx][KVD] FP32
 * (the reference's kc_h / vc_h), writable so a test can plant a long
 * cached context without priming it token by token. */
float *orc_qwen_kv(orc_qwen *m, int which);
void orc_qwen_close(orc_qwen *m);

typedef struct orc_gpt2 orc_gpt2;
orc_gpt2 *orc_gpt2_open(const char *path, int ctx);
void orc_gpt2_reset(orc_gpt2 *m);
/* Restates cpu_forward, gpt2_engine.c:363-421. */
void orc_gpt2_forward(orc_gpt2 *m, int token, int pos, int want_logits, float *logits,
                      int nthreads);
const float *orc_gpt2_residual(const orc_gpt2 *m);
/* which 0: keys, 1: values, each [NL][ctx][C] FP32. */
float *orc_gpt2_kv(orc_gpt2 *m, int which);
void orc_gpt2_close(orc_gpt2 *m);

/* First index of the maximum (strict >), qwen_engine.c:360-364. */
int orc_argmax(const float *v, int n);

#ifdef __cplusplus
}
#endif
#endif
