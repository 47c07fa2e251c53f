/* gpt2_engine.c -- GPT-2 124M FP32 greedy decode on B200 with the reference
 * engine's command line (gpu-llm/engine/gpt2_engine.c:430-573):
 *
 *   gpt2_engine --weights W.bin [--ptx M] [--ids F] [--gen N] [--selftest N]
 *               [--fused] [--batch-prefill] [--debug] [--ctx N]
 *
 * The weight file is the reference's flat FP32 layout (124,439,808 floats).
 * Without --ptx every step is this package's fused engine (graph-replayed
 * persistent step, argmax on the device; the prompt is primed with the
 * batched tensor-core prefill).  --ptx M loads module image M and decodes
 * through ITS drop-in kernels (gemv_warp, add_bias, layernorm, attn_*,
 * gelu, add2; gemv_warp_b under --fused) with the reference's per-stage
 * launches (cli_refpath.c).  --batch-prefill is accepted: the fused engine
 * always batches the prompt.  Greedy generation stops at <|endoftext|>
 * (50256); out.ids receives prompt + generated ids; ENGINE_DONE last.
 *
 * --selftest N (gpt2_engine.c:475-537): first the per-layer residual trace
 * of position 0, a per-stage GPU pass against the serial CPU forward
 * written in this host ("trace p0 Lxx: max|d|=..."); then ids[0..N-1] on
 * the GPU (engine, or module M) and on the CPU, and the logits at position
 * N-1 compared (top-5, max |gpu - cpu|, argmax MATCH -> "SELFTEST: PASS").
 * --debug: the reference's layer-0 stage dumps at position 0 ("g.*" from
 * the per-stage GPU pass, "c.*" from the CPU forward). */
#define _GNU_SOURCE
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cli_refpath.h"
#include "sb_cli.h"

#define V 50257
#define NL 12
#define C 768
#define EOT 50256

int main(int argc, char **argv) {
    setvbuf(stdout, NULL, _IONBF, 0);
    const char *weights = NULL, *ids_file = NULL, *ptx = NULL;
    int n_gen = 24, selftest = 0, ctx = 1024, debug = 0, fused = 0;
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "--weights") && i + 1 < argc) weights = argv[++i];
        else if (!strcmp(argv[i], "--ptx") && i + 1 < argc) ptx = argv[++i];
        else if (!strcmp(argv[i], "--ids") && i + 1 < argc) ids_file = argv[++i];
        else if (!strcmp(argv[i], "--gen") && i + 1 < argc) n_gen = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--selftest") && i + 1 < argc) selftest = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--ctx") && i + 1 < argc) ctx = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--fused")) fused = 1;
        else if (!strcmp(argv[i], "--debug")) debug = 1;
        else if (!strcmp(argv[i], "--batch-prefill")) {
        } else { fprintf(stderr, "unknown arg %s\n", argv[i]); return 2; }
    }
    if (!weights) { fprintf(stderr, "--weights required\n"); return 2; }
    if (ctx < 16 || ctx > 1024) { fprintf(stderr, "--ctx must be in [16, 1024]\n"); return 2; }
    double t0 = cli_now();
    sb_engine *e = NULL;
    refpath *mp = NULL; /* --ptx: the operator's module, per-stage launches */
    if (ptx) {
        mp = rp_open(SB_MODEL_GPT2, weights, ptx, ctx);
        rp_set_fused(mp, fused);
        printf("weights: %.1f MiB (124.44M params); module %s, per-stage launches\n", 124439808.0 * 4 / 1048576.0,
               rp_module_name(mp));
    } else {
        e = sb_engine_create(SB_MODEL_GPT2, weights, ctx, 0);
        if (!e) cli_die("engine");
        printf("weights: %.1f MiB (124.44M params); gpu ready in %.1f s\n", 124439808.0 * 4 / 1048576.0,
               cli_now() - t0);
    }
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
    float *logits = malloc(sizeof(float) * V);
    if (selftest > total) selftest = total;
    if (debug && selftest == 0) { /* stage dumps without a selftest: one per-stage GPU pass of position 0 */
        refpath *dbg = mp ? mp : rp_open(SB_MODEL_GPT2, weights, NULL, ctx);
        rp_forward(dbg, ids[0], 0, 0, NULL, 1);
        if (dbg != mp) rp_close(dbg);
    }
    if (selftest > 0) {
        printf("selftest: comparing GPU vs serial-CPU logits at position %d...\n", selftest - 1);
        /* the reference path (module M, or the built-in module) and the CPU
         * forward share one refpath: their caches are separate */
        refpath *rp = mp ? mp : rp_open(SB_MODEL_GPT2, weights, NULL, ctx);
        {
            float *tr_g = malloc(sizeof(float) * NL * C), *tr_c = malloc(sizeof(float) * NL * C);
            rp_set_trace(rp, tr_g);
            rp_forward(rp, ids[0], 0, 1, NULL, debug);
            rp_set_trace(rp, tr_c);
            rp_cpu_forward(rp, ids[0], 0, 1, logits, debug);
            rp_set_trace(rp, NULL);
            for (int l = 0; l < NL; l++) {
                float m = 0.0f, g = 0.0f;
                for (int i = 0; i < C; i++) {
                    const float d = fabsf(tr_g[(long)l * C + i] - tr_c[(long)l * C + i]);
                    if (d > m) m = d;
                    if (fabsf(tr_g[(long)l * C + i]) > g) g = fabsf(tr_g[(long)l * C + i]);
                }
                printf("  trace p0 L%02d: max|d|=%.6f (|gpu|~%.3f)\n", l, m, g);
            }
            free(tr_g);
            free(tr_c);
        }
        float *gl = malloc(sizeof(float) * V), *tmp = malloc(sizeof(float) * V);
        double ts = cli_now();
        for (int p = 0; p < selftest; p++) {
            float *out = p == selftest - 1 ? gl : NULL;
            if (mp) rp_forward(mp, ids[p], p, p == selftest - 1, out, 0);
            else if (sb_engine_forward(e, ids[p], p, p == selftest - 1, out)) cli_die("forward");
        }
        printf("  gpu forward x%d: %.1fs\n", selftest, cli_now() - ts);
        ts = cli_now();
        for (int p = 0; p < selftest; p++) rp_cpu_forward(rp, ids[p], p, p == selftest - 1, logits, 0);
        printf("  cpu reference x%d: %.1fs\n", selftest, cli_now() - ts);
        double maxerr = 0;
        for (int i = 0; i < V; i++) maxerr = fmax(maxerr, fabs((double)gl[i] - (double)logits[i]));
        int tg[5], tc[5];
        cli_top5(gl, V, tg, tmp);
        cli_top5(logits, V, tc, tmp);
        printf("  gpu top-5 ids: %d %d %d %d %d\n", tg[0], tg[1], tg[2], tg[3], tg[4]);
        printf("  cpu top-5 ids: %d %d %d %d %d\n", tc[0], tc[1], tc[2], tc[3], tc[4]);
        printf("  max |gpu-cpu| logit err: %.4f  argmax gpu=%d cpu=%d %s\n", maxerr, tg[0], tc[0],
               tg[0] == tc[0] ? "MATCH" : "MISMATCH");
        if (tg[0] != tc[0]) printf("  SELFTEST: argmax mismatch (noted — fp order sensitivity)\n");
        else printf("  SELFTEST: PASS\n");
        if (rp != mp) rp_close(rp);
        free(gl);
        free(tmp);
    }
    double ts = cli_now();
    int n = 0;
    if (mp) { /* the reference's prime-then-generate loop (gpt2_engine.c:540-560) */
        for (int p = 0; p < total; p++) rp_forward(mp, ids[p], p, p == total - 1, p == total - 1 ? logits : NULL, 0);
        n = total;
        int next = cli_argmax(logits, V);
        ids[n++] = next;
        for (int g = 0; g < n_gen && n < ctx; g++) {
            if (next == EOT) break;
            rp_forward(mp, next, n - 1, 1, logits, 0);
            next = cli_argmax(logits, V);
            ids[n++] = next;
        }
    } else if (sb_engine_generate(e, ids, total, n_gen, ids, &n, SB_GEN_STOP_EOS)) {
        cli_die("generate");
    }
    double dt = cli_now() - ts;
    printf("generated %d token(s) in %.3fs -> %.1f tok/s (fp32, 12-layer GPT-2 on B200, %s; includes priming %d "
           "prompt tokens)\n", n - total, dt, (n - total) / dt, mp ? "per-stage module kernels" : "fused engine", total);
    cli_write_ids("out.ids", ids, n);
    printf("wrote out.ids (%d ids)\n", n);
    printf("ENGINE_DONE\n");
    if (e) sb_engine_destroy(e);
    rp_close(mp);
    free(logits);
    return 0;
}
