/* ref_stages_stem.c - TEST INFRASTRUCTURE ONLY.
 *
 * The v2 (spectral-stem) twin of ref_stages.c: a driver of our own that links
 * the reference's UNMODIFIED stem loader and kernel sources (csrc/
 * bnn_model_stem.c and the shared kernel files, compiled straight from the
 * reference tree into oracle/_ref/ by oracle/Makefile) and calls the kernels
 * in exactly the order bnn_stem_forward does (csrc/bnn_model_stem.c:168-254),
 * reporting every intermediate through the oracle's stage callback. Only the
 * reference's public kernel entry points and StemModel struct
 * (csrc/bnn_model_stem.h:14-64) are used; the reference's own
 * bnn_stem_forward, linked here too, gives the logits the chain must match.
 */
#include "bnn_model_stem.h"  /* reference header, found via -I on its csrc/ */

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef void (*stage_cb)(void *ctx, const char *name, int kind, int C, int H,
                         int W, const void *data);

/* the reference's up_cat is file-static in bnn_model_stem.c; the same
 * documented behaviour (nearest 2x, pad-before = d/2, 0 where uncovered) */
static void cat_up(const int8_t *skip, int sC, int sH, int sW, const int8_t *x,
                   int xC, int hH, int hW, int8_t *out) {
    size_t plane = (size_t)sH * sW;
    memset(out, 0, (size_t)(sC + xC) * plane);
    memcpy(out, skip, (size_t)sC * plane);
    int upH = 2 * hH, upW = 2 * hW;
    int oh = sH > upH ? (sH - upH) / 2 : 0, ow = sW > upW ? (sW - upW) / 2 : 0;
    int cH = upH < sH ? upH : sH, cW = upW < sW ? upW : sW;
    for (int c = 0; c < xC; ++c)
        for (int y = 0; y < cH; ++y)
            for (int xx = 0; xx < cW; ++xx)
                out[(size_t)(sC + c) * plane + (size_t)(oh + y) * sW + ow + xx] =
                    x[((size_t)c * hH + y / 2) * hW + xx / 2];
}

static void act(const ActS *a, const int32_t *P, const float *xr, int8_t *out,
                int C, int H, int W) {
    if (a->kind == 0) apply_fold_int(P, out, C, H, W, a->type, a->t, a->lo, a->hi);
    else apply_fold_real(xr, out, C, H, W, a->A, a->B, a->slope, a->rsign);
}

static int8_t *cf(const ConvS *c, const ActS *a, const int8_t *in, int H, int W,
                  const char *blk, const char *cn, const char *an, stage_cb cb,
                  void *ctx) {
    char nm[64];
    int32_t *P = malloc((size_t)c->Cout * H * W * 4 + 4);
    bconv_dispatch(in, c->packed, P, c->Cin, H, W, c->Cout, c->kh, c->kw, c->pad, c->stride);
    snprintf(nm, sizeof nm, "%s.%s.P", blk, cn);
    cb(ctx, nm, 1, c->Cout, H, W, P);
    int8_t *o = malloc((size_t)c->Cout * H * W + 1);
    act(a, P, NULL, o, c->Cout, H, W);
    snprintf(nm, sizeof nm, "%s.%s", blk, an);
    cb(ctx, nm, 0, c->Cout, H, W, o);
    free(P);
    return o;
}

static const char *ENC[4] = {"enc1", "enc2", "enc3", "enc4"};
static const char *DEC[4] = {"dec4", "dec3", "dec2", "dec1"};

int ref_stem_stages(const StemModel *m, const float *input, int H, int W, float *logits,
                    stage_cb cb, void *ctx) {
    char nm[64];
    int8_t *skip[4];
    int sC[4], sH[4], sW[4];
    const ConvS *sc = &m->stem_conv;
    float *so = malloc((size_t)sc->Cout * H * W * 4 + 4);
    conv_realin_naive(input, sc->wsign, sc->alpha, so, sc->Cin, H, W, sc->Cout, sc->kh, sc->kw, sc->pad,
                      sc->stride);
    cb(ctx, "stem.conv.out", 2, sc->Cout, H, W, so);
    int8_t *x = malloc((size_t)sc->Cout * H * W + 1);
    act(&m->stem_act, NULL, so, x, sc->Cout, H, W);
    cb(ctx, "stem.act", 0, sc->Cout, H, W, x);
    free(so);
    int xC = sc->Cout, xH = H, xW = W;
    for (int i = 0; i < 4; ++i) {
        const ConvS *c2 = &m->enc_conv2[i];
        int8_t *h = cf(&m->enc_conv1[i], &m->enc_act1[i], x, xH, xW, ENC[i], "conv1", "act1", cb, ctx);
        free(x);
        int32_t *P2 = malloc((size_t)c2->Cout * xH * xW * 4 + 4);
        bconv_dispatch(h, c2->packed, P2, c2->Cin, xH, xW, c2->Cout, c2->kh, c2->kw, c2->pad, c2->stride);
        free(h);
        snprintf(nm, sizeof nm, "%s.conv2.P", ENC[i]);
        cb(ctx, nm, 1, c2->Cout, xH, xW, P2);
        skip[i] = malloc((size_t)c2->Cout * xH * xW + 1);
        act(&m->enc_act2_skip[i], P2, NULL, skip[i], c2->Cout, xH, xW);
        snprintf(nm, sizeof nm, "%s.act2_skip", ENC[i]);
        cb(ctx, nm, 0, c2->Cout, xH, xW, skip[i]);
        sC[i] = c2->Cout; sH[i] = xH; sW[i] = xW;
        int Hh = xH / 2, Wh = xW / 2;
        int32_t *Pd = malloc((size_t)c2->Cout * Hh * Wh * 4 + 4);
        maxpool_P(P2, Pd, c2->Cout, xH, xW, 2, 2);
        free(P2);
        snprintf(nm, sizeof nm, "%s.pool.P", ENC[i]);
        cb(ctx, nm, 1, c2->Cout, Hh, Wh, Pd);
        x = malloc((size_t)c2->Cout * Hh * Wh + 1);
        act(&m->enc_act2_down[i], Pd, NULL, x, c2->Cout, Hh, Wh);
        free(Pd);
        snprintf(nm, sizeof nm, "%s.act2_down", ENC[i]);
        cb(ctx, nm, 0, c2->Cout, Hh, Wh, x);
        xC = c2->Cout; xH = Hh; xW = Wh;
    }
    int8_t *h = cf(&m->bott_conv1, &m->bott_act1, x, xH, xW, "bottleneck", "conv1", "act1", cb, ctx);
    free(x);
    x = cf(&m->bott_conv2, &m->bott_act2, h, xH, xW, "bottleneck", "conv2", "act2", cb, ctx);
    free(h);
    xC = m->bott_conv2.Cout;
    for (int i = 0; i < 4; ++i) {
        int si = 3 - i, H2 = sH[si], W2 = sW[si], catC = sC[si] + xC;
        int8_t *cat = malloc((size_t)catC * H2 * W2 + 1);
        cat_up(skip[si], sC[si], H2, W2, x, xC, xH, xW, cat);
        snprintf(nm, sizeof nm, "%s.cat", DEC[i]);
        cb(ctx, nm, 0, catC, H2, W2, cat);
        free(x); free(skip[si]);
        h = cf(&m->dec_conv1[i], &m->dec_act1[i], cat, H2, W2, DEC[i], "conv1", "act1", cb, ctx);
        free(cat);
        x = cf(&m->dec_conv2[i], &m->dec_act2[i], h, H2, W2, DEC[i], "conv2", "act2", cb, ctx);
        free(h);
        xC = m->dec_conv2[i].Cout; xH = H2; xW = W2;
    }
    size_t n = (size_t)xC * xH * xW;
    float *xf = malloc(n * 4 + 4);
    for (size_t j = 0; j < n; ++j) xf[j] = (float)x[j];
    head_1x1(xf, m->head_W, m->head_bias, logits, m->head_Cin, xH, xW, m->head_Cout);
    cb(ctx, "logits", 2, m->head_Cout, xH, xW, logits);
    free(xf);
    free(x);
    return 0;
}
