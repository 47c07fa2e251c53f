// sb_finalize.cuh -- the one-thread step-finalize kernel every decode
// module image carries (module images are loaded independently, so each
// needs its own copy of the symbol).
#pragma once
#include "sb_common.cuh"
#include "sb_step.h"

// A step is skipped once generation stopped or when its position would
// fall outside the KV cache (host misuse cannot write past the cache).
SB_DEV bool sb_step_idle(const SbStep *st) { return st->done || st->pos < 0 || st->pos >= st->pos_limit; }

// End of a step: once past the prompt, tokens[pos+1] = argmax; stop-token
// handling; pos += 1.  One thread.  with_logits == 0 for prompt steps that
// skip the LM head (qwen_engine.c:262, want_logits).
extern "C" __global__ void sb_finalize(SbStep *__restrict__ st, int *__restrict__ tokens, int with_logits) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    if (sb_step_idle(st)) return;
    const int p = st->pos;
    if (with_logits) {
        const int nxt = argmax_key_index(st->key);
        st->key = 0ull;
        if (p + 1 >= st->n_prompt && p + 1 < st->n_end) {
            tokens[p + 1] = nxt;
            st->n_generated += 1;
            if (st->stop_on_eos && (nxt == st->eos0 || nxt == st->eos1)) st->done = 1;
        }
    }
    st->pos = p + 1;
    if (st->pos >= st->n_end - 1) st->done = 1;  // last position of this generation was processed
}
