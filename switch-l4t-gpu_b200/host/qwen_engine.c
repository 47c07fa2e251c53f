/* qwen_engine.c -- Qwen2.5-0.5B FP16-weight decode on B200 with the
 * reference engine's command line (gpu-llm/engine/qwen_engine.c:446-558):
 *
 *   qwen_engine --weights W.bin [--ptx M] [--ids F] [--gen N] [--selftest N]
 *               [--debug] [--greedy] [--serve] [--ctx N]
 *
 * The weight file is the reference's flat layout.  --ptx is accepted for
 * command-line compatibility; the sm_100a module images are linked into
 * libswitch_b200.  Generation follows the reference: prime the prompt
 * (logits on the last token only), then pick tokens greedily (--greedy) or
 * by the reference's sampler (temperature 0.7, top-k 20, top-p 0.8,
 * repetition penalty 1.1, xorshift seed 1234), stopping at <|endoftext|> or
 * <|im_end|>; out.ids receives prompt + generated ids; ENGINE_DONE last.
 *
 * Greedy generation runs entirely on the device (graph-replayed steps with
 * the argmax and next-token write fused); sampled generation copies the
 * logits back each token and samples on the host, as the reference does.
 *
 * --serve: per request read u32 T, T x u32 ids, u32 max_gen from stdin and
 * write u32 M, M x u32 ids (prompt echo + generation) to stdout; banners go
 * to stderr only (qwen_engine.c:406-444).
 * --selftest N: decode ids[0..N-1] through the graph-replayed fused step and
 * through direct launches without programmatic dependent launch, and compare
 * the last logits (top-5, max |diff|, argmax); the independent CPU golden
 * comparison is the parity test suite's job. */
#define _GNU_SOURCE
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "sb_cli.h"

#define V 151936
#define EOT 151643
#define IM_END 151645

static int greedy_mode = 0;
static uint32_t rng_state = 1234;
static float *scratch_logits, *sample_scratch;

static int next_token(sb_engine *e, const int *ids, int n) {
    (void)e;
    if (greedy_mode) return cli_argmax(scratch_logits, V);
    return sb_sample_token(scratch_logits, V, ids, n, 0.7f, 20, 0.8f, 1.1f, &rng_state, sample_scratch);
}

/* Sampled generation: forward per token with host logits. Returns total. */
static int generate_sampled(sb_engine *e, int *ids, int total, int n_gen, int cap, int *emitted) {
    for (int p = 0; p < total; p++)
        if (sb_engine_forward(e, ids[p], p, p == total - 1, p == total - 1 ? scratch_logits : NULL)) cli_die("forward");
    int nxt = next_token(e, ids, total);
    ids[total++] = nxt;
    *emitted = 0;
    for (int g = 0; g < n_gen && total < cap; g++) {
        if (nxt == EOT || nxt == IM_END) break;
        if (sb_engine_forward(e, nxt, total - 1, 1, scratch_logits)) cli_die("forward");
        nxt = next_token(e, ids, total);
        ids[total++] = nxt;
        (*emitted)++;
    }
    return total;
}

static int generate(sb_engine *e, int *ids, int total, int n_gen, int cap, int *emitted) {
    if (!greedy_mode) return generate_sampled(e, ids, total, n_gen, cap, emitted);
    if (total + n_gen > cap) n_gen = cap - total;
    int n = 0;
    if (sb_engine_generate(e, ids, total, n_gen, ids, &n, SB_GEN_STOP_EOS)) cli_die("generate");
    *emitted = n - total - 1 > 0 ? n - total - 1 : 0;
    return n;
}

static void serve_loop(sb_engine *e, int ctx) {
    int *buf = malloc(sizeof(int) * (size_t)(ctx + 2));
    for (;;) {
        uint32_t T = 0;
        if (fread(&T, 4, 1, stdin) != 1) break;
        uint32_t keep = (uint32_t)(ctx - 16);
        if (T > keep) { /* keep the tail (latest context) */
            uint32_t drop = T - keep;
            int *tmp = malloc(sizeof(int) * T);
            if (fread(tmp, 4, T, stdin) != T) { free(tmp); break; }
            memcpy(buf, tmp + drop, sizeof(int) * keep);
            free(tmp);
            T = keep;
        } else if (T > 0 && fread(buf, 4, T, stdin) != T) {
            break;
        }
        uint32_t maxg = 0;
        if (fread(&maxg, 4, 1, stdin) != 1) break;
        if (T == 0) { /* nothing to condition on: echo nothing */
            uint32_t z = 0;
            fwrite(&z, 4, 1, stdout);
            fflush(stdout);
            continue;
        }
        if ((int)maxg > ctx - (int)T - 2) maxg = (uint32_t)(ctx - (int)T - 2);
        int emitted = 0;
        int total = generate(e, buf, (int)T, (int)maxg, ctx, &emitted);
        uint32_t outn = (uint32_t)total;
        fwrite(&outn, 4, 1, stdout);
        fwrite(buf, 4, outn, stdout);
        fflush(stdout);
        fprintf(stderr, "serve: T=%u emitted=%d\n", T, emitted);
    }
    free(buf);
}

int main(int argc, char **argv) {
    setvbuf(stdout, NULL, _IONBF, 0);
    const char *weights = NULL, *ids_file = NULL;
    int n_gen = 24, selftest = 0, serve = 0, ctx = 2048, debug = 0;
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "--weights") && i + 1 < argc) weights = argv[++i];
        else if (!strcmp(argv[i], "--ptx") && i + 1 < argc) ++i; /* images are built in */
        else if (!strcmp(argv[i], "--ids") && i + 1 < argc) ids_file = argv[++i];
        else if (!strcmp(argv[i], "--gen") && i + 1 < argc) n_gen = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--selftest") && i + 1 < argc) selftest = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--ctx") && i + 1 < argc) ctx = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--debug")) debug = 1;
        else if (!strcmp(argv[i], "--greedy")) greedy_mode = 1;
        else if (!strcmp(argv[i], "--serve")) serve = 1;
        else { fprintf(stderr, "unknown arg %s\n", argv[i]); return 2; }
    }
    if (!weights) { fprintf(stderr, "--weights required\n"); return 2; }
    if (ctx < 32 || ctx > 8192) { fprintf(stderr, "--ctx must be in [32, 8192]\n"); return 2; }
    if (n_gen > ctx) n_gen = ctx;
    (void)debug;
    FILE *log = serve ? stderr : stdout;
    double t0 = cli_now();
    sb_engine *e = sb_engine_create(SB_MODEL_QWEN, weights, ctx, 0);
    if (!e) cli_die("engine");
    fprintf(log, "weights: %.1f MiB (24-layer Qwen2.5-0.5B, fp16); gpu ready in %.1f s (ctx %d)\n",
            990162688 / 1048576.0, cli_now() - t0, ctx);
    scratch_logits = malloc(sizeof(float) * V);
    sample_scratch = malloc(sizeof(float) * V);
    if (serve) {
        fprintf(stderr, "serve mode: reading requests from stdin\n");
        serve_loop(e, ctx);
        sb_engine_destroy(e);
        return 0;
    }
    int *ids = malloc(sizeof(int) * (size_t)(2 * ctx + 2));
    int total = 0;
    if (ids_file) {
        total = cli_read_ids(ids_file, ids, ctx);
        if (total < 0) { fprintf(stderr, "cannot open ids\n"); return 2; }
        printf("prompt: %d token(s)\n", total);
    } else {
        for (int i = 0; i < 8; i++) ids[i] = (i * 7919 + 42) % V;
        total = 8;
        printf("no --ids file; using %d deterministic ids\n", total);
    }
    if (total == 0) { fprintf(stderr, "empty prompt\n"); return 2; }
    if (selftest > total) selftest = total;
    if (selftest > 0) {
        float *a = malloc(sizeof(float) * V), *b = malloc(sizeof(float) * V), *tmp = malloc(sizeof(float) * V);
        sb_engine *d = sb_engine_create(SB_MODEL_QWEN, weights, ctx, SB_FLAG_NO_GRAPH | SB_FLAG_NO_PDL);
        if (!d) cli_die("engine");
        for (int p = 0; p < selftest; p++) {
            if (sb_engine_forward(e, ids[p], p, p == selftest - 1, p == selftest - 1 ? a : NULL)) cli_die("forward");
            if (sb_engine_forward(d, ids[p], p, p == selftest - 1, p == selftest - 1 ? b : NULL)) cli_die("forward");
        }
        double maxerr = 0;
        for (int i = 0; i < V; i++) maxerr = fmax(maxerr, fabs((double)a[i] - (double)b[i]));
        int ta[5], tb[5];
        cli_top5(a, V, ta, tmp);
        cli_top5(b, V, tb, tmp);
        printf("selftest at position %d: graph top-5 %d %d %d %d %d | direct top-5 %d %d %d %d %d\n", selftest - 1,
               ta[0], ta[1], ta[2], ta[3], ta[4], tb[0], tb[1], tb[2], tb[3], tb[4]);
        printf("  max |graph-direct| logit diff: %.6f  argmax %s\n", maxerr, ta[0] == tb[0] ? "MATCH" : "MISMATCH");
        printf(ta[0] == tb[0] && maxerr < 1e-3 ? "  SELFTEST: PASS\n" : "  SELFTEST: FAIL\n");
        sb_engine_destroy(d);
        free(a); free(b); free(tmp);
    }
    double ts = cli_now();
    int emitted = 0;
    int n = generate(e, ids, total, n_gen, ctx, &emitted);
    double dt = cli_now() - ts;
    printf("generated %d token(s) in %.3fs -> %.1f tok/s (fp16 weights, 24-layer Qwen2.5-0.5B on B200, %s; "
           "includes priming %d prompt tokens)\n", n - total, dt, (n - total) / dt, greedy_mode ? "greedy" : "sampled",
           total);
    cli_write_ids("out.ids", ids, n);
    printf("wrote out.ids (%d ids)\n", n);
    printf("ENGINE_DONE\n");
    sb_engine_destroy(e);
    return 0;
}
