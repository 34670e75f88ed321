/* ref_stages_react.c - TEST INFRASTRUCTURE ONLY.
 *
 * Chains the reference's own ReAct kernels (compiled unmodified from
 * csrc/ into oracle/_ref/libref_react.so) in the order of the reference
 * forward (csrc/bnn_model_react.c:160-441) on the whole image and reports
 * every intermediate under the names oracle/bnn_oracle_react.c uses, so the
 * oracle can be pinned stage by stage. Dispatch between the register-blocked
 * and the plain kernels follows the reference (proj_dispatch,
 * conv_real_dispatch, :140-159). The concat is re-done here (the
 * reference's up_cat_f is file-static; it only moves data). Also exposes the
 * reference's own bnn_forward_react so its logits can be tied to the chain.
 */
#include <stdlib.h>
#include <string.h>

#include "bnn_model_react.h"

typedef void (*stage_cb)(void *ctx, const char *name, int kind, int C, int H, int W, const void *data);

static void emit(stage_cb cb, void *ctx, const char *blk, const char *st, int kind, int C, int H, int W,
                 const void *d) {
    char nm[64];
    strcpy(nm, blk);
    strcat(nm, ".");
    strcat(nm, st);
    cb(ctx, nm, kind, C, H, W, d);
}

static void emit_p16(stage_cb cb, void *ctx, const char *blk, const char *st, int C, int H, int W,
                     const int16_t *P) {
    size_t n = (size_t)C * H * W;
    int32_t *w = malloc(n * 4 + 4);
    for (size_t i = 0; i < n; ++i) w[i] = P[i];
    emit(cb, ctx, blk, st, 1, C, H, W, w);
    free(w);
}

static void proj(const ProjR *p, const float *x, float *out, int H, int W) {
    if (p->Cout % 8 == 0) react_proj_blk(x, p->W, out, p->Cin, H, W, p->Cout);
    else react_proj_1x1(x, p->W, out, p->Cin, H, W, p->Cout);
}

static float *unit1(const BlockR *b, const float *x, int H, int W, const char *blk, stage_cb cb, void *ctx) {
    size_t HW = (size_t)H * W;
    int Ci = b->conv1.Cin, Co = b->conv1.Cout;
    float *res = malloc((size_t)Co * HW * 4 + 4);
    proj(&b->proj1, x, res, H, W);
    emit(cb, ctx, blk, "proj", 2, Co, H, W, res);
    int8_t *a = malloc((size_t)Ci * HW + 1);
    react_tap(x, a, Ci, H, W, b->tap1.rsign);
    emit(cb, ctx, blk, "tap1", 0, Ci, H, W, a);
    int16_t *P = malloc((size_t)Co * HW * 2 + 2);
    bconv_blk_b4p4_i16(a, b->conv1.packed, P, Ci, H, W, Co, 3, 3, 1, 1);
    emit_p16(cb, ctx, blk, "conv1.P", Co, H, W, P);
    free(a);
    react_epilogue_int_i16(P, res, res, Co, H, W, b->epi1.A, b->epi1.B, b->epi1.move1, b->epi1.prelu_w);
    emit(cb, ctx, blk, "h1", 2, Co, H, W, res);
    free(P);
    return res;
}

static int16_t *unit2_P(const BlockR *b, const float *h1, int H, int W, const char *blk, stage_cb cb, void *ctx) {
    size_t HW = (size_t)H * W;
    int C = b->conv2.Cin, Co = b->conv2.Cout;
    int8_t *a = malloc((size_t)C * HW + 1);
    react_tap(h1, a, C, H, W, b->tap2.rsign);
    emit(cb, ctx, blk, "tap2", 0, C, H, W, a);
    int16_t *P = malloc((size_t)Co * HW * 2 + 2);
    bconv_blk_b4p4_i16(a, b->conv2.packed, P, C, H, W, Co, 3, 3, 1, 1);
    emit_p16(cb, ctx, blk, "conv2.P", Co, H, W, P);
    free(a);
    return P;
}

static float *upcat(const float *skip, int sC, int sH, int sW, const float *x, int xC, int hH, int hW) {
    float *out = calloc((size_t)(sC + xC) * sH * sW, 4);
    memcpy(out, skip, (size_t)sC * sH * sW * 4);
    int upH = 2 * hH, upW = 2 * hW, dh = sH - upH, dw = sW - upW;
    int oh = dh > 0 ? dh / 2 : 0, ow = dw > 0 ? dw / 2 : 0;
    int cH = upH < sH ? upH : sH, cW = upW < sW ? upW : sW;
    for (int c = 0; c < xC; ++c)
        for (int y = 0; y < cH; ++y)
            for (int xx = 0; xx < cW; ++xx)
                out[((size_t)(sC + c) * sH + oh + y) * sW + ow + xx] = x[((size_t)c * hH + y / 2) * hW + xx / 2];
    return out;
}

static const char *ENC[4] = {"enc1", "enc2", "enc3", "enc4"};
static const char *DEC[4] = {"dec4", "dec3", "dec2", "dec1"};

int ref_react_stages(const char *path, const float *input, int H, int W, float *logits, stage_cb cb, void *ctx) {
    ModelR *m = bnn_load_react(path);
    float *skip[4];
    int sC[4], sH[4], sW[4];
    float *x = NULL;
    int xC = 0, xH = H, xW = W;
    for (int i = 0; i < 4; ++i) {
        const BlockR *b = &m->enc[i];
        size_t HW = (size_t)xH * xW;
        int Co = b->conv2.Cout;
        float *h1;
        if (i == 0) {
            const ConvR *c1 = &b->conv1;
            float *res = malloc((size_t)c1->Cout * HW * 4 + 4);
            proj(&b->proj1, input, res, xH, xW);
            emit(cb, ctx, "enc1", "proj", 2, c1->Cout, xH, xW, res);
            float *co1 = malloc((size_t)c1->Cout * HW * 4 + 4);
            if (c1->Cout % 8 == 0) react_conv3_blk(input, c1->wsign, c1->alpha, co1, c1->Cin, xH, xW, c1->Cout);
            else conv_realin_naive(input, c1->wsign, c1->alpha, co1, c1->Cin, xH, xW, c1->Cout, 3, 3, 1, 1);
            emit(cb, ctx, "enc1", "conv1.out", 2, c1->Cout, xH, xW, co1);
            react_epilogue_real_v2(co1, res, res, c1->Cout, xH, xW, b->epi1.A, b->epi1.B, b->epi1.move1,
                                   b->epi1.prelu_w);
            emit(cb, ctx, "enc1", "h1", 2, c1->Cout, xH, xW, res);
            free(co1);
            h1 = res;
        } else {
            h1 = unit1(b, x, xH, xW, ENC[i], cb, ctx);
            free(x);
        }
        int16_t *P2 = unit2_P(b, h1, xH, xW, ENC[i], cb, ctx);
        skip[i] = malloc((size_t)Co * HW * 4 + 4);
        react_epilogue_int_i16(P2, h1, skip[i], Co, xH, xW, b->epi_a.A, b->epi_a.B, b->epi_a.move1,
                               b->epi_a.prelu_w);
        emit(cb, ctx, ENC[i], "skip", 2, Co, xH, xW, skip[i]);
        sC[i] = Co; sH[i] = xH; sW[i] = xW;
        int Hh = xH / 2, Wh = xW / 2;
        size_t HWh = (size_t)Hh * Wh;
        int16_t *Pd = malloc((size_t)Co * HWh * 2 + 2);
        maxpool_P_i16(P2, Pd, Co, xH, xW, 2, 2);
        emit_p16(cb, ctx, ENC[i], "pool.P", Co, Hh, Wh, Pd);
        free(P2);
        float *h1d = malloc((size_t)Co * HWh * 4 + 4);
        maxpool_real_v2(h1, h1d, Co, xH, xW, 2, 2);
        emit(cb, ctx, ENC[i], "poolr", 2, Co, Hh, Wh, h1d);
        free(h1);
        react_epilogue_int_i16(Pd, h1d, h1d, Co, Hh, Wh, b->epi_b.A, b->epi_b.B, b->epi_b.move1, b->epi_b.prelu_w);
        emit(cb, ctx, ENC[i], "down", 2, Co, Hh, Wh, h1d);
        free(Pd);
        x = h1d;
        xC = Co; xH = Hh; xW = Wh;
    }
    {
        const BlockR *b = &m->bott;
        float *h1 = unit1(b, x, xH, xW, "bottleneck", cb, ctx);
        free(x);
        int16_t *P2 = unit2_P(b, h1, xH, xW, "bottleneck", cb, ctx);
        react_epilogue_int_i16(P2, h1, h1, b->conv2.Cout, xH, xW, b->epi_a.A, b->epi_a.B, b->epi_a.move1,
                               b->epi_a.prelu_w);
        emit(cb, ctx, "bottleneck", "h2", 2, b->conv2.Cout, xH, xW, h1);
        free(P2);
        x = h1;
        xC = b->conv2.Cout;
    }
    for (int i = 0; i < 4; ++i) {
        const BlockR *b = &m->dec[i];
        int si = 3 - i, H2 = sH[si], W2 = sW[si];
        float *cat = upcat(skip[si], sC[si], H2, W2, x, xC, xH, xW);
        emit(cb, ctx, DEC[i], "cat", 2, sC[si] + xC, H2, W2, cat);
        free(x);
        free(skip[si]);
        float *h1 = unit1(b, cat, H2, W2, DEC[i], cb, ctx);
        free(cat);
        int16_t *P2 = unit2_P(b, h1, H2, W2, DEC[i], cb, ctx);
        react_epilogue_int_i16(P2, h1, h1, b->conv2.Cout, H2, W2, b->epi_a.A, b->epi_a.B, b->epi_a.move1,
                               b->epi_a.prelu_w);
        emit(cb, ctx, DEC[i], "h2", 2, b->conv2.Cout, H2, W2, h1);
        free(P2);
        x = h1;
        xC = b->conv2.Cout; xH = H2; xW = W2;
    }
    head_1x1_v2(x, m->head_W, m->head_bias, logits, m->head_Cin, H, W, m->head_Cout);
    cb(ctx, "logits", 2, m->n_classes, H, W, logits);
    free(x);
    bnn_free_react(m);
    return 0;
}

/* the reference's own forward (strip-processed enc1 / dec1 + fused head) */
int ref_react_forward(const char *path, const float *input, int H, int W, float *logits) {
    ModelR *m = bnn_load_react(path);
    bnn_forward_react(m, input, H, W, logits);
    bnn_free_react(m);
    return 0;
}

/* and its patch-wise forward (csrc/bnn_model_react.c:454-476) */
int ref_react_forward_patched(const char *path, const float *input, int H, int W, float *logits, int P) {
    ModelR *m = bnn_load_react(path);
    bnn_forward_react_patched(m, input, H, W, logits, P);
    bnn_free_react(m);
    return 0;
}
