/* qwen_engine.c -- Qwen2.5-0.5B FP16-weight decode on B200 with the
 * reference engine's command line (gpu-llm/engine/qwen_engine.c:446-558):
 *
 *   qwen_engine --weights W.bin [--ptx M] [--ids F] [--gen N] [--selftest N]
 *               [--debug] [--greedy] [--serve] [--ctx N]
 *
 * The weight file is the reference's flat layout.  Generation follows the
 * reference: prime the prompt (logits on the last token only), then pick
 * tokens greedily (--greedy) or by the reference's sampler (temperature 0.7,
 * top-k 20, top-p 0.8, repetition penalty 1.1, xorshift seed 1234),
 * stopping at <|endoftext|> or <|im_end|>; out.ids receives prompt +
 * generated ids; ENGINE_DONE last.
 *
 * Without --ptx every step is this package's fused engine: greedy generation
 * runs entirely on the device (graph-replayed persistent step with the
 * argmax and next-token write fused); sampled generation copies the logits
 * back each token and samples on the host, as the reference does.
 * --ptx M loads module image M and decodes through ITS drop-in kernels
 * (gemv_h, rmsnorm, rope, swiglu, attn_*, add2) with the reference's
 * per-stage launches (cli_refpath.c), as the reference host does.
 *
 * --selftest N: decode ids[0..N-1] on the GPU (the engine, or module M) and
 * with the serial CPU forward written in this host (cli_refpath.c), and
 * compare the logits at position N-1: top-5 of each, max |gpu - cpu|,
 * argmax MATCH -> "SELFTEST: PASS" (qwen_engine.c:494-521).
 * --debug: the reference's layer-0 stage dumps at position 0 ("g.*" from a
 * per-stage GPU pass, "c.*" from the CPU forward during --selftest).
 * --serve: per request read u32 T, T x u32 ids, u32 max_gen from stdin and
 * write u32 M, M x u32 ids (prompt echo + generation) to stdout; banners go
 * to stderr only (qwen_engine.c:406-444). */
#define _GNU_SOURCE
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cli_refpath.h"
#include "sb_cli.h"

#define V 151936
#define EOT 151643
#define IM_END 151645

static int greedy_mode = 0;
static uint32_t rng_state = 1234;
static float *scratch_logits, *sample_scratch;
static refpath *modpath; /* --ptx: decode through the given module's kernels */

/* one decode step with the reference's gpu_forward contract */
static void gpu_forward(sb_engine *e, int token, int pos, int want_logits, float *logits) {
    if (modpath) rp_forward(modpath, token, pos, want_logits, logits, 0);
    else if (sb_engine_forward(e, token, pos, want_logits, logits)) cli_die("forward");
}

/* The next token after a step whose logits are on the device (the engine
 * path: the top-20 candidates are picked there, the draw is on the host)
 * or in scratch_logits (the --ptx module path). */
static int next_token(sb_engine *e, const int *ids, int n) {
    if (greedy_mode) return cli_argmax(scratch_logits, V); /* only reached on the --ptx path */
    if (!modpath) {
        const int t = sb_engine_sample(e, n, 0.7f, 20, 0.8f, 1.1f, &rng_state);
        if (t < 0) cli_die("sample");
        return t;
    }
    return sb_sample_token(scratch_logits, V, ids, n, 0.7f, 20, 0.8f, 1.1f, &rng_state, sample_scratch);
}

/* Sampled generation: one forward per token; the engine keeps the logits
 * on the device. Returns total. */
static int generate_sampled(sb_engine *e, int *ids, int total, int n_gen, int cap, int *emitted) {
    float *host_logits = modpath ? scratch_logits : NULL;
    for (int p = 0; p < total; p++) gpu_forward(e, ids[p], p, p == total - 1, p == total - 1 ? host_logits : NULL);
    int nxt = next_token(e, ids, total);
    ids[total++] = nxt;
    *emitted = 0;
    for (int g = 0; g < n_gen && total < cap; g++) {
        if (nxt == EOT || nxt == IM_END) break;
        gpu_forward(e, nxt, total - 1, 1, host_logits);
        nxt = next_token(e, ids, total);
        ids[total++] = nxt;
        (*emitted)++;
    }
    return total;
}

static int generate(sb_engine *e, int *ids, int total, int n_gen, int cap, int *emitted) {
    if (!greedy_mode || modpath) return generate_sampled(e, ids, total, n_gen, cap, emitted);
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
    const char *weights = NULL, *ids_file = NULL, *ptx = NULL;
    int n_gen = 24, selftest = 0, serve = 0, ctx = 2048, debug = 0;
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "--weights") && i + 1 < argc) weights = argv[++i];
        else if (!strcmp(argv[i], "--ptx") && i + 1 < argc) ptx = argv[++i];
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
    FILE *log = serve ? stderr : stdout;
    double t0 = cli_now();
    sb_engine *e = NULL;
    if (ptx) {
        modpath = rp_open(SB_MODEL_QWEN, weights, ptx, ctx);
        fprintf(log, "weights: %.1f MiB (24-layer Qwen2.5-0.5B, fp16); module %s, per-stage launches (ctx %d)\n",
                990162688 / 1048576.0, rp_module_name(modpath), ctx);
    } else {
        e = sb_engine_create(SB_MODEL_QWEN, weights, ctx, 0);
        if (!e) cli_die("engine");
        fprintf(log, "weights: %.1f MiB (24-layer Qwen2.5-0.5B, fp16); gpu ready in %.1f s (ctx %d)\n",
                990162688 / 1048576.0, cli_now() - t0, ctx);
    }
    scratch_logits = malloc(sizeof(float) * V);
    sample_scratch = malloc(sizeof(float) * V);
    if (serve) {
        fprintf(stderr, "serve mode: reading requests from stdin\n");
        serve_loop(e, ctx);
        if (e) sb_engine_destroy(e);
        rp_close(modpath);
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
    if (debug) { /* layer-0 stage dumps of position 0 from a per-stage GPU pass */
        refpath *dbg = modpath ? modpath : rp_open(SB_MODEL_QWEN, weights, NULL, ctx);
        printf("debug: stage dumps of layer 0 at position 0 (%s)\n", rp_module_name(dbg));
        rp_forward(dbg, ids[0], 0, 0, NULL, 1);
        if (dbg != modpath) rp_close(dbg);
    }
    if (selftest > total) selftest = total;
    if (selftest > 0) {
        printf("selftest: comparing GPU vs serial-CPU logits at position %d...\n", selftest - 1);
        float *g = malloc(sizeof(float) * V), *c = malloc(sizeof(float) * V), *tmp = malloc(sizeof(float) * V);
        double ts = cli_now();
        for (int p = 0; p < selftest; p++) gpu_forward(e, ids[p], p, p == selftest - 1, p == selftest - 1 ? g : NULL);
        printf("  gpu forward x%d: %.1fs\n", selftest, cli_now() - ts);
        refpath *cpu = modpath ? modpath : rp_open(SB_MODEL_QWEN, weights, NULL, ctx);
        ts = cli_now();
        for (int p = 0; p < selftest; p++)
            rp_cpu_forward(cpu, ids[p], p, p == selftest - 1, p == selftest - 1 ? c : NULL, debug);
        printf("  cpu reference x%d: %.1fs\n", selftest, cli_now() - ts);
        double maxerr = 0;
        for (int i = 0; i < V; i++) maxerr = fmax(maxerr, fabs((double)g[i] - (double)c[i]));
        int tg[5], tc[5];
        cli_top5(g, V, tg, tmp);
        cli_top5(c, V, tc, tmp);
        printf("  gpu top-5 ids: %d %d %d %d %d\n", tg[0], tg[1], tg[2], tg[3], tg[4]);
        printf("  cpu top-5 ids: %d %d %d %d %d\n", tc[0], tc[1], tc[2], tc[3], tc[4]);
        printf("  max |gpu-cpu| logit err: %.4f  argmax gpu=%d cpu=%d %s\n", maxerr, tg[0], tc[0],
               tg[0] == tc[0] ? "MATCH" : "MISMATCH");
        printf(tg[0] == tc[0] ? "  SELFTEST: PASS\n" : "  SELFTEST: FAIL\n");
        if (cpu != modpath) rp_close(cpu);
        free(g); free(c); free(tmp);
    }
    double ts = cli_now();
    int emitted = 0;
    int n = generate(e, ids, total, n_gen, ctx, &emitted);
    double dt = cli_now() - ts;
    printf("generated %d token(s) in %.3fs -> %.1f tok/s (fp16 weights, 24-layer Qwen2.5-0.5B on B200, %s, %s; "
           "includes priming %d prompt tokens)\n", n - total, dt, (n - total) / dt, greedy_mode ? "greedy" : "sampled",
           modpath ? "per-stage module kernels" : "fused engine", total);
    cli_write_ids("out.ids", ids, n);
    printf("wrote out.ids (%d ids)\n", n);
    printf("ENGINE_DONE\n");
    if (e) sb_engine_destroy(e);
    rp_close(modpath);
    return 0;
}
