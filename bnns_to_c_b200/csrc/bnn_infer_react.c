/* bnn_infer_react.c - standalone CLI over the B200 ReAct (v3) engine with
 * the reference CLI's semantics (csrc/main_react.c of Sboyle132/BNNs_to_C):
 *
 *   bnn_infer_react <blob> <input.bin|rand> <output.bin> H W [reps]
 *     input : [patch<P>:][mem:]FILE | [patch<P>:]rand
 *             FILE float32 [n_bands,H,W]; `rand` = the reference's
 *             deterministic synthetic cube; patch<P>: run independent PxP
 *             patches (P a multiple of 16) and stitch them
 *     output: float32 logits [n_classes,H,W]
 *     reps  : the same image N times; median / min / max forward time
 *
 * Report lines go to stdout in the reference's format ("# load", "# mode",
 * "# forward"); BNN_PROFILE=1 adds the per-op device-time table on stderr.
 * The reference streams a file input strip by strip to bound host memory;
 * here the cube is read once (same values). The GPU is the process's
 * current CUDA device.
 */
#include "bnn_model_react.h"

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_ms(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec * 1e3 + (double)t.tv_nsec * 1e-6;
}

static int cmp_d(const void *a, const void *b) {
    double x = *(const double *)a, y = *(const double *)b;
    return (x > y) - (x < y);
}

/* The reference's `rand` cube (csrc/main_react.c:28-40): Marsaglia
 * xorshift64 (shifts 13, 7, 17) from a fixed seed gives two uniforms in
 * (0,1) from the top 53 bits of the state, and one Box-Muller normal,
 * sqrt(-2 ln u0) cos(2 pi u1), per element. */
static void synthetic_cube(float *x, size_t n) {
    uint64_t s = 88172645463325252ULL;
    for (size_t i = 0; i < n; ++i) {
        double u[2];
        for (int k = 0; k < 2; ++k) {
            s ^= s << 13;
            s ^= s >> 7;
            s ^= s << 17;
            u[k] = ((double)(s >> 11) + 0.5) / 9007199254740992.0;
        }
        x[i] = (float)(sqrt(-2.0 * log(u[0])) * cos(6.283185307179586 * u[1]));
    }
}

static void profile_table(const ModelR *m) {
    int n = bnn_react_profile_count(m);
    double total = 0;
    for (int i = 0; i < n; ++i) {
        double ms;
        bnn_react_profile_get(m, i, NULL, NULL, NULL, &ms, NULL);
        total += ms;
    }
    fprintf(stderr, "# per-op device time (CUDA events)\n# %-28s %-10s %10s %6s\n", "op", "type", "ms", "%");
    for (int i = 0; i < n; ++i) {
        const char *label, *type;
        double ms;
        int calls;
        bnn_react_profile_get(m, i, &label, &type, NULL, &ms, &calls);
        fprintf(stderr, "  %-28s %-10s %10.3f %5.1f%%\n", label, type, ms / (calls ? calls : 1),
                total > 0 ? 100.0 * ms / total : 0.0);
    }
}

int main(int argc, char **argv) {
    if (argc < 6) {
        fprintf(stderr, "usage: %s blob input|rand output H W [reps]\n", argv[0]);
        return 2;
    }
    const char *blob = argv[1], *inp = argv[2], *outp = argv[3];
    int H = atoi(argv[4]), W = atoi(argv[5]);
    int reps = argc > 6 ? atoi(argv[6]) : 1;
    if (H <= 0 || W <= 0 || reps <= 0) {
        fprintf(stderr, "bad H/W/reps\n");
        return 2;
    }
    double t0 = now_ms();
    ModelR *m = bnn_load_react(blob);
    double t_load = now_ms() - t0;
    const char *prof = getenv("BNN_PROFILE");
    if (prof && prof[0] && strcmp(prof, "0") != 0) bnn_react_profile_enable(m, 1);

    size_t nin = (size_t)m->n_bands * H * W, nout = (size_t)m->n_classes * H * W;
    int patchP = 0;
    if (!strncmp(inp, "patch", 5)) {
        patchP = atoi(inp + 5);
        const char *q = strchr(inp, ':');
        if (patchP <= 0 || !q) {
            fprintf(stderr, "bad patch spec '%s' (use patch32:FILE)\n", inp);
            return 2;
        }
        if (patchP % 16) {
            fprintf(stderr, "patch size must be a multiple of 16\n");
            return 2;
        }
        inp = q + 1;
    }
    int is_rand = strcmp(inp, "rand") == 0;
    const char *path = strncmp(inp, "mem:", 4) == 0 ? inp + 4 : inp;
    float *in = malloc(nin * sizeof(float)), *out = malloc(nout * sizeof(float));
    double *ts = malloc((size_t)reps * sizeof(double));
    if (!in || !out || !ts) {
        fprintf(stderr, "OOM\n");
        return 1;
    }
    if (is_rand) {
        synthetic_cube(in, nin);
    } else {
        FILE *f = fopen(path, "rb");
        if (!f || fread(in, sizeof(float), nin, f) != nin) {
            fprintf(stderr, "bad input %s\n", path);
            return 1;
        }
        fclose(f);
    }
    for (int r = 0; r < reps; ++r) {
        double a = now_ms();
        if (patchP) bnn_forward_react_patched(m, in, H, W, out, patchP);
        else bnn_forward_react(m, in, H, W, out);
        ts[r] = now_ms() - a;
    }
    qsort(ts, (size_t)reps, sizeof(double), cmp_d);
    FILE *g = fopen(outp, "wb");
    if (!g) {
        fprintf(stderr, "cannot open %s\n", outp);
        return 1;
    }
    fwrite(out, sizeof(float), nout, g);
    fclose(g);
    printf("# load %.1f ms\n", t_load);
    if (patchP) printf("# mode: patch-wise P=%d\n", patchP);
    printf("# forward %dx%d reps=%d  median %.1f ms  min %.1f  max %.1f\n", H, W, reps, ts[reps / 2], ts[0],
           ts[reps - 1]);
    if (prof && prof[0] && strcmp(prof, "0") != 0) profile_table(m);
    free(ts);
    free(in);
    free(out);
    bnn_free_react(m);
    return 0;
}
