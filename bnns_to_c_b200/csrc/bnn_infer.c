/* bnn_infer.c - standalone CLI over the B200 engine, with the reference
 * CLI's semantics (csrc/main.c of Sboyle132/BNNs_to_C):
 *
 *   bnn_infer weights.blob input.bin|rand output.bin [H W [reps]]
 *     input.bin : n_bands*H*W float32, layout [band,row,col]; "rand" =
 *                 srand(1234), uniform[-1,1] from rand(), as the reference
 *     output.bin: n_classes*H*W float32, layout [class,row,col]
 *     reps      : run the forward N times, report median/min/max
 *
 * Coarse timing goes to stderr in the reference's format. BNN_PROFILE=1 in
 * the environment adds the per-op device-time table (the reference's
 * `make profile` build). The GPU is the calling process's current CUDA
 * device (CUDA_VISIBLE_DEVICES selects it).
 *
 * Built with -DBNN_INFER_STEM this is bnn_infer_stem, the v2 spectral-stem
 * CLI with csrc/main_stem.c's semantics (same arguments; v2 blob; the
 * report's first line is "# [stem] ... stem_channels=C").
 */
#include "bnn_b200.h"
#include "bnn_model.h"
#ifdef BNN_INFER_STEM
#include "bnn_model_stem.h"
#endif

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + (double)t.tv_nsec * 1e-9;
}

static int cmp_d(const void *a, const void *b) {
    double x = *(const double *)a, y = *(const double *)b;
    return (x > y) - (x < y);
}

int main(int argc, char **argv) {
    if (argc < 4) {
#ifdef BNN_INFER_STEM
        fprintf(stderr, "usage: %s weights_stem.blob input.bin|rand output.bin [H W [reps]]\n", argv[0]);
#else
        fprintf(stderr, "usage: %s weights.blob input.bin|rand output.bin [H W [reps]]\n", argv[0]);
#endif
        return 1;
    }
    int H = (argc > 4) ? atoi(argv[4]) : 32;
    int W = (argc > 5) ? atoi(argv[5]) : 32;
    int reps = (argc > 6) ? atoi(argv[6]) : 1;
    if (reps < 1) reps = 1;

    double t0 = now_s();
#ifdef BNN_INFER_STEM
    StemModel *sm = bnn_stem_load(argv[1]);
    Model *m = bnn_stem_as_model(sm);
#else
    Model *m = bnn_load(argv[1]);
#endif
    double t_load = now_s() - t0;
    const char *prof = getenv("BNN_PROFILE");
    if (prof && prof[0] && strcmp(prof, "0") != 0) bnn_profile_enable(m, 1);

    long n_in = (long)m->n_bands * H * W;
    float *input = malloc((size_t)n_in * sizeof(float));
    if (!input) { fprintf(stderr, "OOM input\n"); return 1; }
    if (strcmp(argv[2], "rand") == 0) {
        srand(1234);
        for (long i = 0; i < n_in; ++i) input[i] = (float)rand() / RAND_MAX * 2.0f - 1.0f;
    } else {
        FILE *fi = fopen(argv[2], "rb");
        if (!fi || fread(input, sizeof(float), (size_t)n_in, fi) != (size_t)n_in) {
            fprintf(stderr, "bad input file\n");
            return 1;
        }
        fclose(fi);
    }

    long n_out = (long)m->n_classes * H * W;
    float *logits = malloc((size_t)n_out * sizeof(float));
    double *ts = malloc((size_t)reps * sizeof(double));
    if (!logits || !ts) { fprintf(stderr, "OOM\n"); return 1; }

    for (int r = 0; r < reps; ++r) {
        double f0 = now_s();
#ifdef BNN_INFER_STEM
        bnn_stem_forward(sm, input, H, W, logits);
#else
        bnn_forward(m, input, H, W, logits);
#endif
        ts[r] = (now_s() - f0) * 1e3;
    }
    qsort(ts, (size_t)reps, sizeof(double), cmp_d);
    double med = ts[reps / 2], tmin = ts[0], tmax = ts[reps - 1];

    double w0 = now_s();
    FILE *fo = fopen(argv[3], "wb");
    if (!fo) { fprintf(stderr, "cannot open %s\n", argv[3]); return 1; }
    fwrite(logits, sizeof(float), (size_t)n_out, fo);
    fclose(fo);
    double t_write = (now_s() - w0) * 1e3;

#ifdef BNN_INFER_STEM
    fprintf(stderr, "# [stem] H=%d W=%d bands=%d classes=%d stem_channels=%d reps=%d\n", H, W, sm->n_bands,
            sm->n_classes, sm->stem_conv.Cout, reps);
#else
    fprintf(stderr, "# H=%d W=%d bands=%d classes=%d reps=%d\n", H, W, m->n_bands, m->n_classes, reps);
#endif
    fprintf(stderr, "# blob load : %9.3f ms\n", t_load * 1e3);
    fprintf(stderr, "# forward   : %9.3f ms  (median; min %.3f, max %.3f)\n", med, tmin, tmax);
    fprintf(stderr, "# out write : %9.3f ms\n", t_write);
    bnn_profile_report(m, stderr);

    free(ts); free(input); free(logits);
#ifdef BNN_INFER_STEM
    bnn_stem_free(sm);
#else
    bnn_free(m);
#endif
    return 0;
}
