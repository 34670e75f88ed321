/* ref_bench_bconv.c - TEST/BASELINE INFRASTRUCTURE ONLY.
 *
 * Times the reference CPU engine's isolated binary conv layer (the
 * binary-conv sweep): bconv_dispatch (csrc/bnn_conv.c:216-223) followed by
 * apply_fold_int (csrc/bnn_fold.c:37-60) and, with pool = 1, maxpool_P
 * (csrc/bnn_maxpool.c:28-48) and apply_fold_int of the pooled P - the
 * reference's encoder conv2 (csrc/bnn_model.c:170-185). All of it is the
 * reference's own code, compiled unmodified from its sources by
 * oracle/Makefile; bconv_xnor_packed spreads its output rows over the
 * OpenMP threads the environment allows (OMP_NUM_THREADS).
 *
 * usage: ref_bench_bconv C H pool budget_s [seed]
 *   Cin = Cout = C, H = W, one image per call as the reference runs them;
 *   inputs and weights uniform random +-1 bits, thresholds (rule "P >= t")
 *   uniform in [-2C, 2C]. Images are timed one after another until
 *   budget_s has passed (at least one, at most 64) after one untimed image.
 * prints "image_s <mean seconds per image>", "images <count>",
 *        "checksum <sum of P of the last image>".
 */
#include "bnn_model.h"

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <time.h>

/* csrc/bnn_conv.c: kidx-order weight packing (bench_bconv.c declares it too) */
void pack_weights(const int8_t *w, uint64_t *packed, int Cout, int Cin, int kh, int kw);

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

static uint64_t rs;
static uint32_t next32(void) {
    rs ^= rs << 13;
    rs ^= rs >> 7;
    rs ^= rs << 17;
    return (uint32_t)(rs >> 32);
}

int main(int argc, char **argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s C H pool budget_s [seed]\n", argv[0]);
        return 1;
    }
    const int C = atoi(argv[1]), H = atoi(argv[2]), pool = atoi(argv[3]);
    const double budget = atof(argv[4]);
    rs = 0x9E3779B97F4A7C15ull ^ (uint64_t)(argc > 5 ? atoll(argv[5]) : 1);
    if (C <= 0 || H < 2) return 1;
    const int W = H, nw = (9 * C + 63) / 64, Hp = H / 2, Wp = W / 2;
    const size_t hw = (size_t)H * W;
    int8_t *a = malloc((size_t)C * hw), *w = malloc((size_t)C * C * 9);
    uint64_t *pw = malloc((size_t)C * nw * 8);
    int32_t *P = malloc((size_t)C * hw * 4), *Pp = malloc((size_t)C * Hp * Wp * 4);
    int8_t *o = malloc((size_t)C * hw), *op = malloc((size_t)C * Hp * Wp);
    int32_t *ty = malloc((size_t)C * 4), *t = malloc((size_t)C * 4), *t2 = malloc((size_t)C * 4),
            *z = calloc((size_t)C, 4);
    if (!a || !w || !pw || !P || !Pp || !o || !op || !ty || !t || !t2 || !z) return 1;
    for (size_t i = 0; i < (size_t)C * hw; ++i) a[i] = (next32() & 1) ? 1 : -1;
    for (size_t i = 0; i < (size_t)C * C * 9; ++i) w[i] = (next32() & 1) ? 1 : -1;
    pack_weights(w, pw, C, C, 3, 3);
    for (int c = 0; c < C; ++c) {
        ty[c] = 1;
        t[c] = (int32_t)(next32() % (uint32_t)(4 * C + 1)) - 2 * C;
        t2[c] = (int32_t)(next32() % (uint32_t)(4 * C + 1)) - 2 * C;
    }
    int images = 0;
    double t0 = 0.0;
    for (int it = 0;; ++it) {
        if (it == 1) t0 = now_s();
        bconv_dispatch(a, pw, P, C, H, W, C, 3, 3, 1, 1);
        apply_fold_int(P, o, C, H, W, ty, t, z, z);
        if (pool) {
            maxpool_P(P, Pp, C, H, W, 2, 2);
            apply_fold_int(Pp, op, C, Hp, Wp, ty, t2, z, z);
        }
        if (it >= 1) {
            ++images;
            if (now_s() - t0 >= budget || images >= 64) break;
        }
    }
    const double per = (now_s() - t0) / images;
    long long sum = 0;
    for (size_t i = 0; i < (size_t)C * hw; ++i) sum += P[i];
    printf("image_s %.9f\nimages %d\nchecksum %lld\n", per, images, sum);
    return 0;
}
