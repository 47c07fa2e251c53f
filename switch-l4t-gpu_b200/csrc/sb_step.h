/* sb_step.h -- the device-resident decode-step state shared by the fused
 * kernels and the C engine hosts.  Keeping the step position, the stop flag
 * and the argmax accumulator in device memory is what lets one captured CUDA
 * graph replay every token without host round-trips. */
#ifndef SB_STEP_H
#define SB_STEP_H

typedef struct SbStep {
    int pos;                /* position of the token being processed            */
    int n_prompt;           /* tokens [0, n_prompt) are given (teacher-forced)  */
    int n_end;              /* token buffer capacity: writes stop at n_end-1    */
    int done;               /* set once a stop token was generated              */
    int stop_on_eos;        /* 1: generation stops at eos0 / eos1               */
    int eos0, eos1;
    int n_generated;        /* tokens written by sb_finalize                    */
    int pos_limit;          /* KV-cache rows: a step with pos >= pos_limit is a no-op */
    unsigned long long key; /* argmax key of this step's logits (value|~index)  */
} SbStep;

#endif
