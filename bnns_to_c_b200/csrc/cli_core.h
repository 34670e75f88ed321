/* cli_core.h - what the three command-line front ends (bnn_infer,
 * bnn_infer_stem, bnn_infer_react) share: a monotonic millisecond clock,
 * repetition statistics, whole-file float32 input and output, and the
 * BNN_PROFILE switch. Header-only (static functions), C99.
 *
 * The statistics follow the reference CLIs' convention
 * (csrc/main.c:55-61, csrc/main_react.c): the reported median of n
 * timings is the element at index n/2 of the ascending order, the minimum
 * and maximum its ends.
 */
#ifndef BNN_CLI_CORE_H
#define BNN_CLI_CORE_H

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

typedef struct {
    double median, min, max;
} CliTimes;

static double cli_ms(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return 1e3 * (double)t.tv_sec + 1e-6 * (double)t.tv_nsec;
}

static int cli_order(const void *a, const void *b) {
    const double x = *(const double *)a, y = *(const double *)b;
    return x < y ? -1 : x > y;
}

/* sorts ms[0..n) in place; n >= 1 */
static CliTimes cli_times(double *ms, int n) {
    CliTimes t;
    qsort(ms, (size_t)n, sizeof *ms, cli_order);
    t.median = ms[n / 2];
    t.min = ms[0];
    t.max = ms[n - 1];
    return t;
}

/* exactly n floats from path into dst; 0 on success */
static int cli_read_f32(const char *path, float *dst, size_t n) {
    FILE *f = fopen(path, "rb");
    if (!f) return -1;
    const size_t got = fread(dst, sizeof *dst, n, f);
    fclose(f);
    return got == n ? 0 : -1;
}

/* n floats to path (created or truncated); 0 on success */
static int cli_write_f32(const char *path, const float *src, size_t n) {
    FILE *f = fopen(path, "wb");
    if (!f) return -1;
    fwrite(src, sizeof *src, n, f);
    fclose(f);
    return 0;
}

/* an environment switch: set, non-empty and not "0" */
static int cli_env_on(const char *name) {
    const char *v = getenv(name);
    return v && *v && strcmp(v, "0") != 0;
}

#endif
