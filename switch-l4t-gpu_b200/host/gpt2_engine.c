/* gpt2_engine.c -- GPT-2 124M FP32 greedy decode on B200 with the reference
 * engine's command line (gpu-llm/engine/gpt2_engine.c:430-573):
 *
 *   gpt2_engine --weights W.bin [--ptx M] [--ids F] [--gen N] [--selftest N]
 *               [--fused] [--batch-prefill] [--debug] [--ctx N]
 *
 * The weight file is the reference's flat FP32 layout (124,439,808 floats).
 * --ptx, --fused and --batch-prefill are accepted for compatibility: the
 * module images are built in, every step is fused (bias epilogues included)
 * and the prompt is primed with the same device steps.  Greedy generation
 * stops at <|endoftext|> (50256); out.ids receives prompt + generated ids.
 * --selftest N compares graph-replayed and directly launched steps (see
 * qwen_engine.c). */
#define _GNU_SOURCE
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "sb_cli.h"

#define V 50257

int main(int argc, char **argv) {
    setvbuf(stdout, NULL, _IONBF, 0);
    const char *weights = NULL, *ids_file = NULL;
    int n_gen = 24, selftest = 0, ctx = 1024;
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "--weights") && i + 1 < argc) weights = argv[++i];
        else if (!strcmp(argv[i], "--ptx") && i + 1 < argc) ++i;
        else if (!strcmp(argv[i], "--ids") && i + 1 < argc) ids_file = argv[++i];
        else if (!strcmp(argv[i], "--gen") && i + 1 < argc) n_gen = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--selftest") && i + 1 < argc) selftest = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--ctx") && i + 1 < argc) ctx = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--fused") || !strcmp(argv[i], "--batch-prefill") || !strcmp(argv[i], "--debug")) {
        } else { fprintf(stderr, "unknown arg %s\n", argv[i]); return 2; }
    }
    if (!weights) { fprintf(stderr, "--weights required\n"); return 2; }
    if (ctx < 16 || ctx > 1024) { fprintf(stderr, "--ctx must be in [16, 1024]\n"); return 2; }
    double t0 = cli_now();
    sb_engine *e = sb_engine_create(SB_MODEL_GPT2, weights, ctx, 0);
    if (!e) cli_die("engine");
    printf("weights: %.1f MiB (124.44M params); gpu ready in %.1f s\n", 124439808.0 * 4 / 1048576.0, cli_now() - t0);
    int *ids = malloc(sizeof(int) * (size_t)(ctx + 2));
    int total = 0;
    if (ids_file) {
        total = cli_read_ids(ids_file, ids, ctx);
        if (total < 0) { fprintf(stderr, "bad ids file\n"); return 1; }
        printf("prompt: %d token(s)\n", total);
    } else {
        for (int i = 0; i < 8; i++) ids[i] = (i * 7919 + 42) % V;
        total = 8;
        printf("no --ids file; using %d deterministic ids\n", total);
    }
    if (total == 0) { fprintf(stderr, "empty prompt\n"); return 1; }
    if (total + n_gen > ctx) n_gen = ctx - total;
    if (selftest > total) selftest = total;
    if (selftest > 0) {
        float *a = malloc(sizeof(float) * V), *b = malloc(sizeof(float) * V), *tmp = malloc(sizeof(float) * V);
        sb_engine *d = sb_engine_create(SB_MODEL_GPT2, weights, ctx, SB_FLAG_NO_GRAPH | SB_FLAG_NO_PDL);
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
    int n = 0;
    if (sb_engine_generate(e, ids, total, n_gen, ids, &n, SB_GEN_STOP_EOS)) cli_die("generate");
    double dt = cli_now() - ts;
    printf("generated %d token(s) in %.3fs -> %.1f tok/s (fp32, 12-layer GPT-2 on B200; includes priming %d "
           "prompt tokens)\n", n - total, dt, (n - total) / dt, total);
    cli_write_ids("out.ids", ids, n);
    printf("wrote out.ids (%d ids)\n", n);
    printf("ENGINE_DONE\n");
    sb_engine_destroy(e);
    return 0;
}
