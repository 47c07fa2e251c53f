/* ref_bench.c -- times the REFERENCE's own CPU decode (cpu_forward of
 * gpu-llm/engine/qwen_engine.c or gpt2_engine.c, compiled unmodified through
 * ref_engine_wrap.c) on the host cores, for bench.py's cpu_baseline and
 * `--impl reference` legs.  Test/measurement infrastructure only.
 *
 *   ref_<model>_bench <weights> <procs> <warmup> <steps> <tokens_per_step> <first_token>
 *                     [prompt_ids_file]
 *
 * The weight file is loaded once; then <procs> forked replicas (sharing the
 * weights copy-on-write) each run a greedy decode -- cpu_forward with logits,
 * then the reference argmax -- for (warmup + steps) x tokens_per_step
 * positions.  With a prompt file (ids, one per line) every replica first
 * primes that prompt as the reference's generation loop does
 * (qwen_engine.c:523-541: cpu_forward per prompt position, logits at the
 * last, argmax -> first generated token), untimed, and the timed decode
 * continues from position n_prompt; without one it decodes from position 0
 * starting at <first_token>.  All replicas start the timed steps together.
 * The reference engine is single-threaded, so replicas are how it uses
 * several cores.  Prints one JSON line: per-step wall time (max over
 * replicas) and aggregate decode tokens/s over the timed steps. */
#define _GNU_SOURCE
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>

#ifdef REF_QWEN
int ref_qwen_load(const char *path);
void ref_qwen_forward(int token, int pos, int want_logits, float *logits_out);
#define LOAD ref_qwen_load
#define FORWARD ref_qwen_forward
#define VOCAB 151936
#else
int ref_gpt2_load(const char *path);
void ref_gpt2_forward(int token, int pos, int want_logits, float *logits_out);
#define LOAD ref_gpt2_load
#define FORWARD ref_gpt2_forward
#define VOCAB 50257
#endif
int ref_argmax_any(const float *v, int n);

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec / 1e9;
}

int main(int argc, char **argv) {
    if (argc < 7) {
        fprintf(stderr, "usage: %s weights procs warmup steps tokens_per_step first_token [prompt_ids]\n", argv[0]);
        return 2;
    }
    const int procs = atoi(argv[2]), warmup = atoi(argv[3]), steps = atoi(argv[4]);
    const int tps = atoi(argv[5]), first = atoi(argv[6]);
    if (procs < 1 || steps < 1 || tps < 1) return 2;
    int *prompt = NULL, n_prompt = 0;
    if (argc > 7) {
        FILE *pf = fopen(argv[7], "r");
        if (!pf) return 2;
        int cap = 64, v;
        prompt = malloc(sizeof(int) * cap);
        while (fscanf(pf, "%d", &v) == 1) {
            if (v < 0 || v >= VOCAB) return 2;
            if (n_prompt == cap) prompt = realloc(prompt, sizeof(int) * (cap *= 2));
            prompt[n_prompt++] = v;
        }
        fclose(pf);
        if (n_prompt < 1) return 2;
    }
    /* the reference loader prints a banner on stdout: keep stdout for JSON */
    int saved = dup(1);
    dup2(2, 1);
    LOAD(argv[1]);
    fflush(stdout);
    dup2(saved, 1);
    close(saved);

    int go[2], res[2], ready[2], go2[2];
    if (pipe(go) || pipe(res) || pipe(ready) || pipe(go2)) return 3;
    const int nsteps = warmup + steps;
    for (int p = 0; p < procs; p++) {
        pid_t pid = fork();
        if (pid < 0) return 3;
        if (pid == 0) {
            close(go[1]);
            close(res[0]);
            char c;
            if (read(go[0], &c, 1) != 1) _exit(4);
            float *logits = malloc(sizeof(float) * VOCAB);
            int tok = (first + 7919 * p) % VOCAB, pos = 0;
            if (n_prompt > 0) {
                for (pos = 0; pos < n_prompt; pos++) FORWARD(prompt[pos], pos, pos == n_prompt - 1, logits);
                tok = ref_argmax_any(logits, VOCAB);
            }
            /* every replica starts its timed steps together, after all have primed */
            if (write(ready[1], &c, 1) != 1 || read(go2[0], &c, 1) != 1) _exit(4);
            double *dt = malloc(sizeof(double) * nsteps);
            for (int s = 0; s < nsteps; s++) {
                double t0 = now_s();
                for (int j = 0; j < tps; j++) {
                    FORWARD(tok, pos++, 1, logits);
                    tok = ref_argmax_any(logits, VOCAB);
                }
                dt[s] = now_s() - t0;
            }
            if (write(res[1], dt, sizeof(double) * nsteps) != (ssize_t)(sizeof(double) * nsteps)) _exit(5);
            _exit(0);
        }
    }
    close(go[0]);
    close(res[1]);
    close(ready[1]);
    close(go2[0]);
    char ones[4096];
    memset(ones, 1, sizeof ones);
    for (int p = 0; p < procs; p += 4096)
        if (write(go[1], ones, (size_t)(procs - p < 4096 ? procs - p : 4096)) < 0) return 3;
    for (int p = 0; p < procs; p++) {
        char c;
        if (read(ready[0], &c, 1) != 1) break; /* a replica died: its result is missing below */
    }
    for (int p = 0; p < procs; p += 4096)
        if (write(go2[1], ones, (size_t)(procs - p < 4096 ? procs - p : 4096)) < 0) return 3;
    double *mx = calloc(nsteps, sizeof(double));
    double *buf = malloc(sizeof(double) * nsteps);
    int got = 0;
    for (int p = 0; p < procs; p++) {
        size_t need = sizeof(double) * nsteps, have = 0;
        while (have < need) {
            ssize_t n = read(res[0], (char *)buf + have, need - have);
            if (n <= 0) break;
            have += (size_t)n;
        }
        if (have != need) continue;
        got++;
        for (int s = 0; s < nsteps; s++)
            if (buf[s] > mx[s]) mx[s] = buf[s];
    }
    while (wait(NULL) > 0) {
    }
    double timed = 0;
    for (int s = warmup; s < nsteps; s++) timed += mx[s];
    printf("{\"procs\":%d,\"replicas_ok\":%d,\"warmup\":%d,\"steps\":%d,\"tokens_per_step\":%d,"
           "\"n_prompt\":%d,\"first_pos\":%d,\"timed_s\":%.6f,\"tok_s\":%.6f,\"step_s\":[",
           procs, got, warmup, steps, tps, n_prompt, n_prompt, timed, got * (double)tps * steps / timed);
    for (int s = warmup; s < nsteps; s++) printf("%s%.6f", s > warmup ? "," : "", mx[s]);
    printf("]}\n");
    return got == procs ? 0 : 1;
}
