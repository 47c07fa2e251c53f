/* sb_sampler.c -- next-token sampling with the reference Qwen engine's
 * generation settings (qwen_engine.c:366-404, after Qwen2.5's
 * generation_config: temperature 0.7, top_k 20, top_p 0.8, repetition
 * penalty 1.1).  The steps are kept in the reference's order so that, given
 * the same logits, context and RNG state, the same token is drawn:
 *   1. repetition penalty for every context id (divide positive logits,
 *      multiply negative ones; repeated ids are penalised repeatedly);
 *   2. divide all logits by the temperature;
 *   3. top-k by k passes of first-index argmax, removing each winner;
 *   4. softmax over the k values (exp clamped to 0 below -87);
 *   5. keep the shortest prefix whose cumulative mass reaches top_p;
 *   6. draw r = u * min(mass kept, top_p) with a 32-bit xorshift (13/17/5)
 *      uniform u = (state & 0xffffff) / 2^24, and take the first index whose
 *      running sum reaches r (else the top token). */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/switch_b200.h"

static float clamped_exp(float x) {
    if (x > 88.0f) x = 88.0f;
    if (x < -87.0f) return 0.0f;
    return expf(x);
}

static float xorshift_uniform(uint32_t *s) {
    *s ^= *s << 13;
    *s ^= *s >> 17;
    *s ^= *s << 5;
    return (*s & 0xffffff) / 16777216.0f;
}

int sb_sample_token(const float *logits, int V, const int *ctx, int ctx_len, float temperature, int top_k,
                    float top_p, float rep_penalty, uint32_t *rng_state, float *scratch) {
    if (!logits || V <= 0 || top_k <= 0 || top_k > 64 || !rng_state) return -1;
    float *w = scratch ? scratch : malloc(sizeof(float) * (size_t)V);
    if (!w) return -1;
    memcpy(w, logits, sizeof(float) * (size_t)V);
    for (int i = 0; i < ctx_len; i++) {
        const int t = ctx[i];
        if (t < 0 || t >= V) continue;
        if (w[t] > 0) w[t] /= rep_penalty;
        else w[t] *= rep_penalty;
    }
    for (int i = 0; i < V; i++) w[i] /= temperature;
    int idx[64];
    float val[64];
    for (int k = 0; k < top_k; k++) {
        int b = 0;
        for (int i = 1; i < V; i++)
            if (w[i] > w[b]) b = i;
        idx[k] = b;
        val[k] = w[b];
        w[b] = -1e30f;
    }
    if (!scratch) free(w);
    return sb_sample_topk(idx, val, top_k, top_p, rng_state);
}

/* steps 4-6 on the k candidates (idx, value) of steps 1-3, in order */
int sb_sample_topk(const int *idx, const float *topv, int top_k, float top_p, uint32_t *rng_state) {
    if (!idx || !topv || top_k <= 0 || top_k > 64 || !rng_state) return -1;
    float val[64];
    const float mx = topv[0];
    float sum = 0.0f;
    for (int k = 0; k < top_k; k++) {
        val[k] = clamped_exp(topv[k] - mx);
        sum += val[k];
    }
    for (int k = 0; k < top_k; k++) val[k] /= sum;
    float cum = 0.0f;
    int keep = top_k;
    for (int k = 0; k < top_k; k++) {
        cum += val[k];
        if (cum >= top_p) {
            keep = k + 1;
            break;
        }
    }
    const float r = xorshift_uniform(rng_state) * ((cum < top_p) ? cum : top_p);
    int out = idx[0];
    cum = 0.0f;
    for (int k = 0; k < keep; k++) {
        cum += val[k];
        if (r <= cum) {
            out = idx[k];
            break;
        }
    }
    return out;
}
