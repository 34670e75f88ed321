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
 * `rand` and mem:FILE run the in-memory forwards; a plain FILE goes to the
 * FILE forms (bnn_forward_react_file / _patched_file), as in the reference,
 * which streams it strip by strip to bound host memory and here reads the
 * cube once (same values). The messages and exit statuses are the
 * reference's, in its order (the input spec is checked after the blob has
 * loaded). The GPU is the process's current CUDA device.
 */
#include "bnn_model_react.h"
#include "cli_core.h"

#include <math.h>
#include <stdint.h>

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

typedef struct {
    const char *blob, *input, *output;
    int H, W, reps;
} Args;

/* the input spec [patch<P>:][mem:]FILE | [patch<P>:]rand, checked after
 * the blob has loaded (the reference's order of complaints) */
typedef struct {
    const char *path;  /* FILE with the prefixes removed */
    int patch;         /* 0 = whole image */
    int in_memory;     /* rand or mem:FILE; otherwise the FILE forms */
    int is_rand;
} Source;

/* returns 0, or the exit status after printing the reason */
static int parse(int argc, char **argv, Args *a) {
    if (argc < 6) {
        fprintf(stderr, "usage: %s blob input|rand output H W [reps]\n", argv[0]);
        return 2;
    }
    a->blob = argv[1];
    a->input = argv[2];
    a->output = argv[3];
    a->H = atoi(argv[4]);
    a->W = atoi(argv[5]);
    a->reps = argc > 6 ? atoi(argv[6]) : 1;
    if (a->H <= 0 || a->W <= 0 || a->reps <= 0) {
        fprintf(stderr, "bad H/W/reps\n");
        return 2;
    }
    return 0;
}

static int parse_source(const char *in, Source *s) {
    s->patch = 0;
    if (!strncmp(in, "patch", 5)) {
        const char *colon = strchr(in, ':');
        s->patch = atoi(in + 5);
        if (s->patch <= 0 || !colon) {
            fprintf(stderr, "bad patch spec '%s' (use patch32:FILE)\n", in);
            return 2;
        }
        if (s->patch % 16) {
            fprintf(stderr, "patch size must be a multiple of 16\n");
            return 2;
        }
        in = colon + 1;
    }
    s->is_rand = !strcmp(in, "rand");
    const int mem = !strncmp(in, "mem:", 4);
    s->in_memory = s->is_rand || mem;
    s->path = mem ? in + 4 : in;
    return 0;
}

/* reps forwards from an in-memory cube (rand / mem:) or from the open file */
static void forwards(const ModelR *m, const Source *s, const float *x, FILE *f, const Args *a, float *y,
                     double *ms) {
    for (int r = 0; r < a->reps; ++r) {
        const double f0 = cli_ms();
        if (x && s->patch)
            bnn_forward_react_patched(m, x, a->H, a->W, y, s->patch);
        else if (x)
            bnn_forward_react(m, x, a->H, a->W, y);
        else if (s->patch)
            bnn_forward_react_patched_file(m, f, a->H, a->W, y, s->patch);
        else
            bnn_forward_react_file(m, f, a->H, a->W, y);
        ms[r] = cli_ms() - f0;
    }
}

int main(int argc, char **argv) {
    Args a;
    int rc = parse(argc, argv, &a);
    if (rc) return rc;
    const double load0 = cli_ms();
    ModelR *m = bnn_load_react(a.blob);
    const double load_ms = cli_ms() - load0;
    const int prof = cli_env_on("BNN_PROFILE");
    if (prof) bnn_react_profile_enable(m, 1);

    const size_t n_in = (size_t)m->n_bands * a.H * a.W, n_out = (size_t)m->n_classes * a.H * a.W;
    float *y = malloc(n_out * sizeof *y);
    if (!y) {
        fprintf(stderr, "OOM out\n");
        return 1;
    }
    Source src;
    if ((rc = parse_source(a.input, &src))) return rc;
    double *ms = malloc((size_t)a.reps * sizeof *ms);
    if (!ms) {
        fprintf(stderr, "OOM\n");
        return 1;
    }
    if (src.in_memory) {
        float *x = malloc(n_in * sizeof *x);
        if (!x) {
            fprintf(stderr, "OOM in\n");
            return 1;
        }
        if (src.is_rand)
            synthetic_cube(x, n_in);
        else if (cli_read_f32(src.path, x, n_in)) {
            fprintf(stderr, "bad input %s\n", src.path);
            return 1;
        }
        forwards(m, &src, x, NULL, &a, y, ms);
        free(x);
    } else {
        FILE *f = fopen(src.path, "rb");
        if (!f) {
            fprintf(stderr, "cannot open %s\n", src.path);
            return 1;
        }
        forwards(m, &src, NULL, f, &a, y, ms);
        fclose(f);
    }
    const CliTimes t = cli_times(ms, a.reps);
    if (cli_write_f32(a.output, y, n_out)) {
        fprintf(stderr, "cannot open %s\n", a.output);
        return 1;
    }
    printf("# load %.1f ms\n", load_ms);
    if (src.patch) printf("# mode: patch-wise P=%d\n", src.patch);
    printf("# forward %dx%d reps=%d  median %.1f ms  min %.1f  max %.1f\n", a.H, a.W, a.reps, t.median, t.min,
           t.max);
    if (prof) profile_table(m);
    free(ms);
    free(y);
    bnn_free_react(m);
    return 0;
}
