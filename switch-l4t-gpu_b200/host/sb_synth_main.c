/* sb_synth_main.c -- `sb_synth`: the seeded synthetic inputs of the
 * benchmarks as a stand-alone program, linked from sb_synth.c alone (no CUDA,
 * no libswitch_b200.so), so a process that must not map this package's GPU
 * library -- the timed reference CPU arm of bench.py -- can still write the
 * same weight file and prompt ids as the GPU arm.
 *
 *   sb_synth weights qwen|gpt2 <path> <seed>   -> weight file (reference layout)
 *   sb_synth ids <n> <vocab> <seed>            -> n ids on stdout, one per line
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/switch_b200.h"

int main(int argc, char **argv) {
    if (argc == 5 && strcmp(argv[1], "weights") == 0) {
        const int model = strcmp(argv[2], "qwen") == 0 ? SB_MODEL_QWEN : strcmp(argv[2], "gpt2") == 0 ? SB_MODEL_GPT2 : 0;
        if (!model) {
            fprintf(stderr, "sb_synth: unknown model %s\n", argv[2]);
            return 2;
        }
        const long n = sb_synth_weights(model, argv[3], strtoull(argv[4], NULL, 10));
        if (n < 0) {
            fprintf(stderr, "sb_synth: could not write %s\n", argv[3]);
            return 1;
        }
        printf("%ld\n", n);
        return 0;
    }
    if (argc == 5 && strcmp(argv[1], "ids") == 0) {
        const int n = atoi(argv[2]), vocab = atoi(argv[3]);
        if (n < 0 || vocab < 1) return 2;
        int *ids = malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
        if (!ids) return 1;
        sb_synth_ids(ids, n, vocab, strtoull(argv[4], NULL, 10));
        for (int i = 0; i < n; i++) printf("%d\n", ids[i]);
        free(ids);
        return 0;
    }
    fprintf(stderr, "usage: sb_synth weights qwen|gpt2 <path> <seed> | sb_synth ids <n> <vocab> <seed>\n");
    return 2;
}
