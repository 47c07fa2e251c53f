/* sb_models.h -- dimensions and weight-file layouts of the two decode
 * models, identical to the reference engines' compile-time constants so the
 * same weight files load in both:
 *   Qwen2.5-0.5B, FP16: qwen_engine.c:43-75 (written by conv_qwen.py:63-99)
 *   GPT-2 124M, FP32:   gpt2_engine.c:40-70 (written by conv_gpt2.py:150-155)
 */
#ifndef SB_MODELS_H
#define SB_MODELS_H
#include <stddef.h>

/* ---- Qwen2.5-0.5B (byte offsets; fp16 unless noted) */
#define QW_V 151936
#define QW_C 896
#define QW_NL 24
#define QW_NH 14
#define QW_NKV 2
#define QW_HD 64
#define QW_KVD (QW_NKV * QW_HD)       /* 128 */
#define QW_QKV (QW_C + 2 * QW_KVD)    /* 1152 */
#define QW_FC 4864
#define QW_CTX_FILE 8192              /* RoPE table rows in the file */
#define QW_EOT 151643                 /* <|endoftext|> */
#define QW_IM_END 151645              /* <|im_end|> */
#define QW_OFF_COS ((size_t)QW_V * QW_C * 2)
#define QW_OFF_SIN (QW_OFF_COS + (size_t)QW_CTX_FILE * (QW_HD / 2) * 4)
#define QW_LBASE (QW_OFF_SIN + (size_t)QW_CTX_FILE * (QW_HD / 2) * 4)
/* per layer: in_ln[C] | qkv_w[QKV][C] | qkv_b[QKV] | o_w[C][C] | post_ln[C] |
 * gateup_w[2FC][C] (gate rows then up rows) | down_w[C][FC] */
#define QW_LSTRIDE ((size_t)(QW_C + QW_QKV * QW_C + QW_QKV + QW_C * QW_C + QW_C + 2 * QW_FC * QW_C + QW_C * QW_FC) * 2)
#define QW_OFF_LNF (QW_LBASE + (size_t)QW_NL * QW_LSTRIDE)
#define QW_FILE_BYTES (QW_OFF_LNF + (size_t)QW_C * 2)
/* element (fp16) offsets inside a layer */
#define QWL_INLN ((size_t)0)
#define QWL_QKVW ((size_t)QW_C)
#define QWL_QKVB (QWL_QKVW + (size_t)QW_QKV * QW_C)
#define QWL_OW (QWL_QKVB + QW_QKV)
#define QWL_POST (QWL_OW + (size_t)QW_C * QW_C)
#define QWL_GATEUP (QWL_POST + QW_C)
#define QWL_DOWN (QWL_GATEUP + (size_t)2 * QW_FC * QW_C)

/* ---- GPT-2 124M (float offsets) */
#define G2_V 50257
#define G2_C 768
#define G2_NH 12
#define G2_HD 64
#define G2_NL 12
#define G2_CTX 1024
#define G2_FC 3072
#define G2_EOT 50256
#define G2_LAYER ((size_t)2 * G2_C + 3 * G2_C * G2_C + 3 * G2_C + G2_C * G2_C + G2_C + 2 * G2_C + \
                  (size_t)G2_FC * G2_C + G2_FC + (size_t)G2_FC * G2_C + G2_C)
#define G2_OFF_WPE ((size_t)G2_V * G2_C)
#define G2_LBASE (G2_OFF_WPE + (size_t)G2_CTX * G2_C)
#define G2_OFF_LNFW (G2_LBASE + (size_t)G2_NL * G2_LAYER)
#define G2_OFF_LNFB (G2_OFF_LNFW + G2_C)
#define G2_TOTAL_FLOATS (G2_OFF_LNFB + G2_C) /* 124,439,808 */
#define G2L_LN1W ((size_t)0)
#define G2L_LN1B (G2L_LN1W + G2_C)
#define G2L_QKVW (G2L_LN1B + G2_C)
#define G2L_QKVB (G2L_QKVW + (size_t)3 * G2_C * G2_C)
#define G2L_AOW (G2L_QKVB + 3 * G2_C)
#define G2L_AOB (G2L_AOW + (size_t)G2_C * G2_C)
#define G2L_LN2W (G2L_AOB + G2_C)
#define G2L_LN2B (G2L_LN2W + G2_C)
#define G2L_FCW (G2L_LN2B + G2_C)
#define G2L_FCB (G2L_FCW + (size_t)G2_FC * G2_C)
#define G2L_PROJW (G2L_FCB + G2_FC)
#define G2L_PROJB (G2L_PROJW + (size_t)G2_FC * G2_C)

#endif
