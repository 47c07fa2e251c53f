/* sb_mk_params.h -- parameter block of the persistent decode kernel
 * (qwen_decode_mk), shared by the C host and the device code.  Device
 * addresses are carried as 64-bit integers so the layout is identical in
 * both languages. */
#ifndef SB_MK_PARAMS_H
#define SB_MK_PARAMS_H

/* Flagged exchange words (u64 = float bits | epoch << 32) between the
 * kernel's stages, in this order: residual x[896] | q k v[1152] |
 * MLP hidden[4864] | attention partials [14 heads][8 splits][66]. */
#define SB_MK_LL_WORDS (896 + 1152 + 4864 + 14 * 8 * 66)
#define SB_MK_SPLITS_MAX 8
/* qwen_decode_mk2: x (a 16-word line per CTA, up to 160 CTAs) | q k v |
 * attention partials (80 words each) | down partials [CTA][896] */
#define SB_MK2_LL_DP (160 * 16 + 1152 + 14 * 8 * 80)
#define SB_MK2_LL_WORDS(ctas) (SB_MK2_LL_DP + (ctas) * 896)

typedef struct SbMkParams {
    unsigned long long w;      /* weight file image                              */
    unsigned long long kv;     /* KV cache [2][layers][ctx][kv_width]            */
    unsigned long long ll;     /* SB_MK_LL_WORDS flagged words, zero at creation */
    unsigned long long logits; /* [V]                                            */
    unsigned long long st;     /* SbStep                                         */
    unsigned long long tokens; /* token ids                                      */
    unsigned long long sync;   /* u32[2]: step sequence number, LM-head arrivals */
    unsigned long long err;    /* set nonzero when a wait timed out              */
    unsigned long long trace;  /* 0, or u64 [ctas][256] globaltimer stamps:
                                * slot 0 start, 1 + 2k / 2 + 2k inputs ready /
                                * outputs written of stage k = layer * 5 + s  */
    int ctx_cap;
    int with_logits;
    int splits;                /* attention T-splits per head (<= SPLITS_MAX)    */
    int score_cap;             /* positions one split's score buffer holds       */
    int test_stall;            /* test hook: 0, or k > 0 -- CTA k-1 withholds its
                                * layer-0 outputs, so every other CTA's bounded
                                * wait runs out and the step reports an error */
    unsigned long long aux;    /* qwen_decode_mk2: W_down transposed per layer,
                                * [layers][4864][896] fp16                       */
} SbMkParams;

#endif
