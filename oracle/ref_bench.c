/* ref_bench.c - TEST/BASELINE INFRASTRUCTURE ONLY.
 *
 * Times the reference CPU engine (its unmodified bnn_load/bnn_forward,
 * compiled from the reference sources into oracle/_ref/ by oracle/Makefile)
 * on this host's cores: the same seeded synthetic patches as the GPU run
 * (include/bnn_synth.h), split into contiguous shards over `procs`
 * single-threaded worker processes (OMP_NUM_THREADS=1 each), which is the
 * fastest way to run the reference on many patches (its OpenMP only spans
 * one conv's rows).
 *
 * Built with -DREF_STEM (ref_bench_stem) it times the reference's v2
 * spectral-stem engine instead (bnn_stem_load / bnn_stem_forward), with
 * -DREF_REACT (ref_bench_react) its v3 ReAct engine (bnn_load_react /
 * bnn_forward_react).
 *
 * usage: ref_bench blob n_patches H W procs seed steps warmup [first_patch]
 * prints one line per timed step: "step <i> <seconds>", then
 * "checksum <sum of logits of patch 0>" so callers can tie it to the GPU run.
 */
#if defined(REF_REACT)
#include "bnn_model_react.h"
typedef ModelR RModel;
#define REF_LOAD bnn_load_react
#define REF_FORWARD bnn_forward_react
#define REF_FREE bnn_free_react
#elif defined(REF_STEM)
#include "bnn_model_stem.h"
typedef StemModel RModel;
#define REF_LOAD bnn_stem_load
#define REF_FORWARD bnn_stem_forward
#define REF_FREE bnn_stem_free
#else
#include "bnn_model.h"
typedef Model RModel;
#define REF_LOAD bnn_load
#define REF_FORWARD bnn_forward
#define REF_FREE bnn_free
#endif
#include "../include/bnn_synth.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

static void run_shard(const RModel *m, const float *in, float *out, int lo,
                      int hi, int H, int W) {
    size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    for (int i = lo; i < hi; ++i) REF_FORWARD(m, in + (size_t)i * ip, H, W, out + (size_t)i * op);
}

static double one_step(const RModel *m, const float *in, float *out, int n,
                       int H, int W, int procs) {
    double t0 = now_s();
    if (procs <= 1) {
        run_shard(m, in, out, 0, n, H, W);
    } else {
        pid_t *pids = calloc((size_t)procs, sizeof(pid_t));
        for (int p = 0; p < procs; ++p) {
            int lo = (int)((long)n * p / procs), hi = (int)((long)n * (p + 1) / procs);
            pid_t pid = fork();
            if (pid == 0) { run_shard(m, in, out, lo, hi, H, W); _exit(0); }
            pids[p] = pid;
        }
        for (int p = 0; p < procs; ++p) {
            int st = 0;
            waitpid(pids[p], &st, 0);
            if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) { fprintf(stderr, "worker failed\n"); exit(2); }
        }
        free(pids);
    }
    return now_s() - t0;
}

int main(int argc, char **argv) {
    if (argc < 9) {
        fprintf(stderr, "usage: %s blob n_patches H W procs seed steps warmup [first_patch]\n", argv[0]);
        return 1;
    }
    int n = atoi(argv[2]), H = atoi(argv[3]), W = atoi(argv[4]), procs = atoi(argv[5]);
    unsigned seed = (unsigned)strtoul(argv[6], NULL, 10);
    int steps = atoi(argv[7]), warm = atoi(argv[8]);
    unsigned first = argc > 9 ? (unsigned)strtoul(argv[9], NULL, 10) : 0u;
    /* one thread per worker process; libgomp read OMP_NUM_THREADS before
     * main, so set the team size directly */
#ifdef _OPENMP
    omp_set_num_threads(1);
#endif
    RModel *m = REF_LOAD(argv[1]);
    size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    float *in = malloc((size_t)n * ip * sizeof(float) + 4);
    float *out = malloc((size_t)n * op * sizeof(float) + 4);
    if (!in || !out) { fprintf(stderr, "OOM\n"); return 1; }
    for (int i = 0; i < n; ++i)
        for (size_t e = 0; e < ip; ++e)
            in[(size_t)i * ip + e] = bnn_synth_value(seed, first + (unsigned)i, (uint32_t)e);
    for (int s = 0; s < warm; ++s) one_step(m, in, out, procs > 1 ? procs : 1, H, W, procs);
    for (int s = 0; s < steps; ++s) printf("step %d %.6f\n", s, one_step(m, in, out, n, H, W, procs));
    /* patch 0's logits, computed in this process for the checksum */
    run_shard(m, in, out, 0, 1, H, W);
    double cs = 0;
    for (size_t j = 0; j < op; ++j) cs += out[j];
    printf("checksum %.9g\n", cs);
    REF_FREE(m);
    free(in); free(out);
    return 0;
}
