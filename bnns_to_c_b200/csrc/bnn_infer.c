/* bnn_infer.c - command-line front end of the B200 engine for v1 blobs
 * (bnn_infer) and, built with -DBNN_INFER_STEM, for v2 spectral-stem blobs
 * (bnn_infer_stem).
 *
 *   bnn_infer weights.blob input.bin|rand output.bin [H W [reps]]
 *
 * Interface kept from the reference CLIs (csrc/main.c, csrc/main_stem.c):
 *   - the arguments, with H = W = 32 and reps = 1 by default, reps below 1
 *     read as 1;
 *   - input.bin: n_bands*H*W float32 [band][row][col]; "rand" is srand(1234)
 *     then rand()/RAND_MAX*2-1 per element, the reference's own input;
 *   - output.bin: n_classes*H*W float32 [class][row][col];
 *   - the messages and exit status 1 on a bad input, an allocation failure
 *     or an unwritable output; a bad blob prints the loader's message and
 *     exits 1 (inside bnn_load);
 *   - the four report lines on stderr: the shape line (v2: "# [stem] ...
 *     stem_channels=C"), blob load, forward median/min/max over reps, and
 *     output write, in milliseconds.
 * BNN_PROFILE=1 adds the per-op device-time table (the reference's
 * `make profile` build). The GPU is the process's current CUDA device.
 */
#include "bnn_b200.h"
#include "bnn_model.h"
#ifdef BNN_INFER_STEM
#include "bnn_model_stem.h"
#endif
#include "cli_core.h"

/* one engine behind the CLI: the loaded handle and the Model that carries
 * the shape and the profiler (the handle itself for v1, the body for v2) */
typedef struct {
    const char *blob_arg;  /* the blob's name in the usage line */
    void *(*load)(const char *path);
    Model *(*body)(void *h);
    void (*forward)(void *h, const float *x, int H, int W, float *logits);
    void (*shape_line)(void *h, int H, int W, int reps);
    void (*release)(void *h);
} Driver;

#ifdef BNN_INFER_STEM
static void *stem_load(const char *p) { return bnn_stem_load(p); }
static Model *stem_body(void *h) { return bnn_stem_as_model((StemModel *)h); }
static void stem_forward(void *h, const float *x, int H, int W, float *y) { bnn_stem_forward(h, x, H, W, y); }
static void stem_shape(void *h, int H, int W, int reps) {
    const StemModel *s = h;
    fprintf(stderr, "# [stem] H=%d W=%d bands=%d classes=%d stem_channels=%d reps=%d\n", H, W, s->n_bands,
            s->n_classes, s->stem_conv.Cout, reps);
}
static void stem_release(void *h) { bnn_stem_free(h); }
static const Driver DRIVER = {"weights_stem.blob", stem_load, stem_body, stem_forward, stem_shape, stem_release};
#else
static void *v1_load(const char *p) { return bnn_load(p); }
static Model *v1_body(void *h) { return h; }
static void v1_forward(void *h, const float *x, int H, int W, float *y) { bnn_forward(h, x, H, W, y); }
static void v1_shape(void *h, int H, int W, int reps) {
    const Model *m = h;
    fprintf(stderr, "# H=%d W=%d bands=%d classes=%d reps=%d\n", H, W, m->n_bands, m->n_classes, reps);
}
static void v1_release(void *h) { bnn_free(h); }
static const Driver DRIVER = {"weights.blob", v1_load, v1_body, v1_forward, v1_shape, v1_release};
#endif

typedef struct {
    const char *blob, *input, *output;
    int H, W, reps;
} Args;

static int parse(int argc, char **argv, Args *a) {
    if (argc < 4) return -1;
    a->blob = argv[1];
    a->input = argv[2];
    a->output = argv[3];
    a->H = argc > 4 ? atoi(argv[4]) : 32;
    a->W = argc > 5 ? atoi(argv[5]) : 32;
    a->reps = argc > 6 ? atoi(argv[6]) : 1;
    if (a->reps < 1) a->reps = 1;
    return 0;
}

/* the reference CLI's synthetic input */
static void fill_rand(float *x, long n) {
    srand(1234);
    for (long i = 0; i < n; ++i) x[i] = (float)rand() / RAND_MAX * 2.0f - 1.0f;
}

int main(int argc, char **argv) {
    Args a;
    if (parse(argc, argv, &a)) {
        fprintf(stderr, "usage: %s %s input.bin|rand output.bin [H W [reps]]\n", argv[0], DRIVER.blob_arg);
        return 1;
    }
    const double load0 = cli_ms();
    void *h = DRIVER.load(a.blob);
    const double load_ms = cli_ms() - load0;
    Model *m = DRIVER.body(h);
    if (cli_env_on("BNN_PROFILE")) bnn_profile_enable(m, 1);

    const long n_in = (long)m->n_bands * a.H * a.W, n_out = (long)m->n_classes * a.H * a.W;
    float *x = malloc((size_t)n_in * sizeof *x);
    if (!x) {
        fprintf(stderr, "OOM input\n");
        return 1;
    }
    if (!strcmp(a.input, "rand"))
        fill_rand(x, n_in);
    else if (cli_read_f32(a.input, x, (size_t)n_in)) {
        fprintf(stderr, "bad input file\n");
        return 1;
    }
    float *y = malloc((size_t)n_out * sizeof *y);
    double *ms = malloc((size_t)a.reps * sizeof *ms);
    if (!y || !ms) {
        fprintf(stderr, "OOM\n");
        return 1;
    }
    for (int r = 0; r < a.reps; ++r) {
        const double f0 = cli_ms();
        DRIVER.forward(h, x, a.H, a.W, y);
        ms[r] = cli_ms() - f0;
    }
    const CliTimes t = cli_times(ms, a.reps);

    const double write0 = cli_ms();
    if (cli_write_f32(a.output, y, (size_t)n_out)) {
        fprintf(stderr, "cannot open %s\n", a.output);
        return 1;
    }
    const double write_ms = cli_ms() - write0;

    DRIVER.shape_line(h, a.H, a.W, a.reps);
    fprintf(stderr, "# blob load : %9.3f ms\n", load_ms);
    fprintf(stderr, "# forward   : %9.3f ms  (median; min %.3f, max %.3f)\n", t.median, t.min, t.max);
    fprintf(stderr, "# out write : %9.3f ms\n", write_ms);
    bnn_profile_report(m, stderr);

    free(ms);
    free(y);
    free(x);
    DRIVER.release(h);
    return 0;
}
