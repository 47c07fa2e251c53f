/* sb_cli.h -- helpers shared by the engine command-line hosts. */
#ifndef SB_CLI_H
#define SB_CLI_H
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <time.h>

#include "../../include/switch_b200.h"

static inline double cli_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec / 1e9;
}

/* ids file: u32 count, count x u32 (the reference's --ids format) */
static inline int cli_read_ids(const char *path, int *ids, int cap) {
    FILE *f = fopen(path, "rb");
    if (!f) return -1;
    uint32_t cnt = 0;
    if (fread(&cnt, 4, 1, f) != 1) { fclose(f); return -1; }
    if ((int)cnt > cap) cnt = (uint32_t)cap;
    for (uint32_t i = 0; i < cnt; i++) {
        uint32_t v;
        if (fread(&v, 4, 1, f) != 1) { fclose(f); return -1; }
        ids[i] = (int)v;
    }
    fclose(f);
    return (int)cnt;
}

static inline void cli_write_ids(const char *path, const int *ids, int n) {
    FILE *f = fopen(path, "wb");
    if (!f) return;
    uint32_t cnt = (uint32_t)n;
    fwrite(&cnt, 4, 1, f);
    fwrite(ids, 4, (size_t)n, f);
    fclose(f);
}

static inline int cli_argmax(const float *v, int n) {
    int b = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[b]) b = i;
    return b;
}

static inline void cli_die(const char *what) {
    fprintf(stderr, "%s: %s\n", what, sb_last_error());
    exit(1);
}

/* top-5 ids of v (by repeated first-index argmax) */
static inline void cli_top5(const float *v, int n, int out[5], float *tmp) {
    for (int i = 0; i < n; i++) tmp[i] = v[i];
    for (int k = 0; k < 5; k++) {
        out[k] = cli_argmax(tmp, n);
        tmp[out[k]] = -1e30f;
    }
}
#endif
