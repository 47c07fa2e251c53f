/* sb_mk_params.h -- parameter block of the persistent decode kernel
 * (qwen_decode_mk), shared by the C host and the device code.  Device
 * addresses are carried as 64-bit integers so the layout is identical in
 * both languages. */
#ifndef SB_MK_PARAMS_H
#define SB_MK_PARAMS_H

typedef struct SbMkParams {
    unsigned long long w;      /* weight file image                        */
    unsigned long long kv;     /* KV cache [2][layers][ctx][kv_width]      */
    unsigned long long x;      /* residual                                 */
    unsigned long long q;      /* query                                    */
    unsigned long long part;   /* attention partials                       */
    unsigned long long hid;    /* MLP hidden                               */
    unsigned long long logits; /* [V]                                      */
    unsigned long long st;     /* SbStep                                   */
    unsigned long long tokens; /* token ids                                */
    unsigned long long bar;    /* grid-barrier counter, zeroed per launch  */
    unsigned long long err;    /* set to 1 when a barrier wait times out   */
    unsigned long long trace;  /* 0, or u64 [ctas][128][2] globaltimer stamps:
                                * (arrive, release) of every grid barrier    */
    int ctx_cap;
    int with_logits;
    int splits;                /* attention T-splits per head              */
    int score_cap;             /* positions one split's score buffer holds */
} SbMkParams;

#endif
