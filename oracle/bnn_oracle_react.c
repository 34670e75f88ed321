/* bnn_oracle_react.c - TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's v3 ReActNet real-highway engine
 * (Sboyle132/BNNs_to_C csrc/bnn_model_react.c and the kernels it calls),
 * the checker for the B200 ReAct path. Only tests/ (and bench.py's CPU leg)
 * load it. Pinned against the reference's own sources compiled unmodified
 * (oracle/_ref/libref_react.so, oracle/ref_stages_react.c) through golden
 * fixtures under tests/golden/.
 *
 * fp32 order: the reference is built with gcc -O3 on x86 with FMA (its
 * Makefile.react: -march=native; oracle/Makefile: -march=x86-64-v3), where
 * gcc contracts most a*b + c into one fused multiply-add. This file is
 * compiled with -ffp-contract=off and writes fmaf() exactly where that build
 * contracts (found stage by stage against the compiled reference), so its
 * roundings are the reference's step for step.
 */
#include "bnn_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- model */
typedef struct {
    int tag, Cout, Cin, kh, kw, pad, stride, nwords;
    uint64_t *packed;
    int8_t *wsign;
    float *alpha;
} RConv;
typedef struct { int kind, C; float *A, *B, *move1, *prelu_w; } REpi;
typedef struct { int C; float *rsign; } RTap;
typedef struct { int Cout, Cin; float *W; } RProj;
typedef struct {
    int is_down, input_real;
    RTap tap1, tap2;
    RConv conv1, conv2;
    RProj proj1;
    REpi epi1, epi_a, epi_b;
} RBlock;
struct ORModel {
    int version, base_channels, n_bands, n_classes, upsampler;
    RBlock enc[4], bott, dec[4];
    int head_Cout, head_Cin;
    float *head_W, *head_bias;
};
typedef struct ORModel ORModel;

typedef struct {
    const unsigned char *p;
    size_t n, off;
    int bad;
    char *err;
    int errlen;
} Rd;

static void rfail(Rd *r, const char *m) {
    if (!r->bad) { r->bad = 1; snprintf(r->err, (size_t)r->errlen, "%s", m); }
}
static void rbytes(Rd *r, void *d, size_t k) {
    if (r->bad) return;
    if (r->n - r->off < k) { rfail(r, "short read"); return; }
    memcpy(d, r->p + r->off, k);
    r->off += k;
}
static int ri(Rd *r) { int32_t v = 0; rbytes(r, &v, 4); return v; }
static void *rarr(Rd *r, size_t k) {
    if (r->bad) return NULL;
    if (r->n - r->off < k) { rfail(r, "short read"); return NULL; }
    void *q = malloc(k ? k : 1);
    rbytes(r, q, k);
    return q;
}

/* csrc/bnn_model_react.c:42-58 */
static void rd_conv(Rd *r, RConv *c) {
    memset(c, 0, sizeof *c);
    c->tag = ri(r);
    c->Cout = ri(r); c->Cin = ri(r); c->kh = ri(r); c->kw = ri(r); c->pad = ri(r); c->stride = ri(r);
    if (r->bad) return;
    if (c->tag == 1) {
        c->nwords = ri(r);
        if (!r->bad && (c->Cout < 0 || c->nwords < 0)) { rfail(r, "short read"); return; }
        c->packed = rarr(r, (size_t)c->Cout * c->nwords * 8);
    } else if (c->tag == 2) {
        if (c->Cout < 0 || c->Cin < 0 || c->kh < 0 || c->kw < 0) { rfail(r, "short read"); return; }
        c->wsign = rarr(r, (size_t)c->Cout * c->Cin * c->kh * c->kw);
        c->alpha = rarr(r, (size_t)c->Cout * 4);
    } else {
        char m[64];
        snprintf(m, sizeof m, "bad conv tag %d", c->tag);
        rfail(r, m);
    }
}
/* :60-65 */
static void rd_proj(Rd *r, RProj *p) {
    int tag = ri(r);
    if (!r->bad && tag != 5) { char m[64]; snprintf(m, sizeof m, "bad proj tag %d", tag); rfail(r, m); return; }
    p->Cout = ri(r); p->Cin = ri(r);
    if (!r->bad && (p->Cout < 0 || p->Cin < 0)) { rfail(r, "short read"); return; }
    p->W = rarr(r, (size_t)p->Cout * p->Cin * 4);
}
/* :67-73 */
static void rd_epi(Rd *r, REpi *e) {
    int tag = ri(r);
    if (!r->bad && tag != 6) { char m[64]; snprintf(m, sizeof m, "bad epi tag %d", tag); rfail(r, m); return; }
    e->kind = ri(r); e->C = ri(r);
    if (!r->bad && e->C < 0) { rfail(r, "short read"); return; }
    size_t k = (size_t)e->C * 4;
    e->A = rarr(r, k); e->B = rarr(r, k); e->move1 = rarr(r, k); e->prelu_w = rarr(r, k);
}
/* :75-79 */
static void rd_tap(Rd *r, RTap *t) {
    int tag = ri(r);
    if (!r->bad && tag != 7) { char m[64]; snprintf(m, sizeof m, "bad tap tag %d", tag); rfail(r, m); return; }
    t->C = ri(r);
    if (!r->bad && t->C < 0) { rfail(r, "short read"); return; }
    t->rsign = rarr(r, (size_t)t->C * 4);
}

/* :85-106, structural checks with the reference's messages */
static void rd_block(Rd *r, RBlock *b, int is_down, int input_real) {
    memset(b, 0, sizeof *b);
    b->is_down = is_down; b->input_real = input_real;
    if (!input_real) rd_tap(r, &b->tap1);
    rd_conv(r, &b->conv1);
    rd_proj(r, &b->proj1);
    rd_epi(r, &b->epi1);
    rd_tap(r, &b->tap2);
    rd_conv(r, &b->conv2);
    rd_epi(r, &b->epi_a);
    if (is_down) rd_epi(r, &b->epi_b);
    if (r->bad) return;
#define CHECK(ok, what) do { if (!(ok)) { rfail(r, "blob layout mismatch: " what); return; } } while (0)
    CHECK(b->conv1.tag == (input_real ? 2 : 1), "conv1 tag");
    CHECK(b->conv2.tag == 1, "conv2 tag");
    CHECK(b->proj1.Cin == b->conv1.Cin && b->proj1.Cout == b->conv1.Cout, "proj1 dims");
    CHECK(input_real || b->tap1.C == b->conv1.Cin, "tap1 channels");
    CHECK(b->tap2.C == b->conv2.Cin, "tap2 channels");
    CHECK(b->epi1.C == b->conv1.Cout && b->epi1.kind == (input_real ? 1 : 0), "epi1");
    CHECK(b->epi_a.C == b->conv2.Cout && b->epi_a.kind == 0, "epi_a");
    CHECK(!is_down || (b->epi_b.C == b->conv2.Cout && b->epi_b.kind == 0), "epi_b");
#undef CHECK
}

static void free_block(RBlock *b) {
    free(b->tap1.rsign); free(b->tap2.rsign);
    free(b->conv1.packed); free(b->conv1.wsign); free(b->conv1.alpha);
    free(b->conv2.packed); free(b->conv2.wsign); free(b->conv2.alpha);
    free(b->proj1.W);
    REpi *e[3] = {&b->epi1, &b->epi_a, &b->epi_b};
    for (int i = 0; i < 3; ++i) { free(e[i]->A); free(e[i]->B); free(e[i]->move1); free(e[i]->prelu_w); }
}

void oracle_react_free(ORModel *m) {
    if (!m) return;
    for (int i = 0; i < 4; ++i) { free_block(&m->enc[i]); free_block(&m->dec[i]); }
    free_block(&m->bott);
    free(m->head_W); free(m->head_bias);
    free(m);
}

/* csrc/bnn_model_react.c:108-134 */
ORModel *oracle_react_load_mem(const void *data, size_t n, char *err, int errlen) {
    Rd r = {(const unsigned char *)data, n, 0, 0, err, errlen};
    if (err && errlen) err[0] = 0;
    char magic[4] = {0};
    rbytes(&r, magic, 4);
    if (!r.bad && memcmp(magic, "BNNC", 4) != 0) rfail(&r, "bad magic");
    if (r.bad) return NULL;
    ORModel *m = calloc(1, sizeof *m);
    m->version = ri(&r);
    if (!r.bad && m->version != 3) {
        char msg[96];
        snprintf(msg, sizeof msg, "blob version %d, this engine reads v3 (ReActNet)", m->version);
        rfail(&r, msg);
    }
    m->base_channels = ri(&r); m->n_bands = ri(&r); m->n_classes = ri(&r); m->upsampler = ri(&r);
    if (!r.bad && m->upsampler != 0) rfail(&r, "only nearest upsampler supported");
    for (int i = 0; i < 4 && !r.bad; ++i) rd_block(&r, &m->enc[i], 1, i == 0);
    if (!r.bad) rd_block(&r, &m->bott, 0, 0);
    for (int i = 0; i < 4 && !r.bad; ++i) rd_block(&r, &m->dec[i], 0, 0);
    int tag = ri(&r);
    if (!r.bad && tag != 4) { char msg[64]; snprintf(msg, sizeof msg, "bad head tag %d", tag); rfail(&r, msg); }
    m->head_Cout = ri(&r); m->head_Cin = ri(&r);
    if (!r.bad && (m->head_Cout < 0 || m->head_Cin < 0)) rfail(&r, "short read");
    m->head_W = rarr(&r, (size_t)m->head_Cout * m->head_Cin * 4);
    m->head_bias = rarr(&r, (size_t)m->head_Cout * 4);
    if (!r.bad && r.off != r.n) rfail(&r, "trailing bytes in blob");
    if (r.bad) { oracle_react_free(m); return NULL; }
    return m;
}

int oracle_react_n_bands(const ORModel *m) { return m->n_bands; }
int oracle_react_n_classes(const ORModel *m) { return m->n_classes; }

/* ---------------------------------------------------------------- kernels */
/* real 1x1 projection, no bias (csrc/bnn_model_react.c:140-145 dispatch):
 * both kernels sum the input channels in order from 0. Cout % 8 == 0 runs
 * the register-blocked proj_blk (csrc/bnn_realin_blk.h:48-88): pixels in
 * whole blocks of 8 take one fused multiply-add per channel, the last H*W % 8
 * pixels (its scalar tail, :79-84) a separate multiply and add - that is what
 * the reference's x86 build does (gcc -O3, x86-64-v3; measured on the
 * compiled reference, oracle/_ref). Other Cout run react_proj_1x1
 * (csrc/bnn_react_ops.c:120-133): fused multiply-adds throughout. */
void oracle_react_proj(const float *x, const float *Wm, float *out, int Cin, int H, int W, int Cout) {
    size_t HW = (size_t)H * W;
    size_t nfull = Cout % 8 == 0 ? HW - HW % 8 : HW;
    for (int co = 0; co < Cout; ++co)
        for (size_t p = 0; p < HW; ++p) {
            float a = 0.0f;
            if (p < nfull)
                for (int ci = 0; ci < Cin; ++ci) a = fmaf(x[(size_t)ci * HW + p], Wm[(size_t)co * Cin + ci], a);
            else
                for (int ci = 0; ci < Cin; ++ci) a = a + Wm[(size_t)co * Cin + ci] * x[(size_t)ci * HW + p];
            out[(size_t)co * HW + p] = a;
        }
}

/* real-input 3x3 pad 1 conv with +-1 weights, register-blocked order
 * (csrc/bnn_realin_blk.h:90-150, used when Cout % 8 == 0): per output the
 * sum runs band by band, and within a band over the in-image taps row by
 * row (ky, then kx); out = acc * alpha. Every product is exact. */
void oracle_react_conv3(const float *x, const int8_t *wsign, const float *alpha, float *out, int Cin, int H,
                        int W, int Cout) {
    size_t HW = (size_t)H * W;
    for (int co = 0; co < Cout; ++co)
        for (int oy = 0; oy < H; ++oy)
            for (int ox = 0; ox < W; ++ox) {
                float a = 0.0f;
                for (int ci = 0; ci < Cin; ++ci)
                    for (int ky = 0; ky < 3; ++ky) {
                        int iy = oy + ky - 1;
                        if (iy < 0 || iy >= H) continue;
                        for (int kx = 0; kx < 3; ++kx) {
                            int ix = ox + kx - 1;
                            if (ix < 0 || ix >= W) continue;
                            a = fmaf(x[((size_t)ci * H + iy) * W + ix],
                                     (float)wsign[((size_t)co * Cin + ci) * 9 + ky * 3 + kx], a);
                        }
                    }
                out[(size_t)co * HW + (size_t)oy * W + ox] = a * alpha[co];
            }
}

/* epilogue on an integer or real accumulator (csrc/bnn_react_epi.c:34-37,
 * 56-59 scalar path, the one x86 runs): t = fma(A, v, B + move1) + res;
 * out = t >= 0 ? t : prelu_w * t */
static void epi_f(const float *v, const float *res, float *out, int C, size_t HW, const REpi *e) {
    for (int c = 0; c < C; ++c) {
        float Ac = e->A[c], Bm = e->B[c] + e->move1[c], wc = e->prelu_w[c];
        for (size_t p = 0; p < HW; ++p) {
            float t = fmaf(Ac, v[(size_t)c * HW + p], Bm) + res[(size_t)c * HW + p];
            out[(size_t)c * HW + p] = t >= 0.0f ? t : wc * t;
        }
    }
}
static void epi_i(const int32_t *P, const float *res, float *out, int C, size_t HW, const REpi *e) {
    for (int c = 0; c < C; ++c) {
        float Ac = e->A[c], Bm = e->B[c] + e->move1[c], wc = e->prelu_w[c];
        for (size_t p = 0; p < HW; ++p) {
            float t = fmaf(Ac, (float)P[(size_t)c * HW + p], Bm) + res[(size_t)c * HW + p];
            out[(size_t)c * HW + p] = t >= 0.0f ? t : wc * t;
        }
    }
}

/* binarising tap (csrc/bnn_react_ops.c:75-86): +1 iff x + rsign > 0 */
static void tap(const float *x, int8_t *out, int C, size_t HW, const float *rsign) {
    for (int c = 0; c < C; ++c)
        for (size_t p = 0; p < HW; ++p) out[(size_t)c * HW + p] = (x[(size_t)c * HW + p] + rsign[c] > 0.0f) ? 1 : -1;
}

/* 2x2 stride-2 max-pools with floor dims, compare order of
 * csrc/bnn_react_opt.c:46-85 (first element, then strictly greater) */
static void pool_f(const float *x, float *out, int C, int H, int W) {
    int Ho = H / 2, Wo = W / 2;
    for (int c = 0; c < C; ++c)
        for (int oy = 0; oy < Ho; ++oy)
            for (int ox = 0; ox < Wo; ++ox) {
                const float *r0 = x + ((size_t)c * H + 2 * oy) * W + 2 * ox, *r1 = r0 + W;
                float m = r0[0];
                if (r0[1] > m) m = r0[1];
                if (r1[0] > m) m = r1[0];
                if (r1[1] > m) m = r1[1];
                out[((size_t)c * Ho + oy) * Wo + ox] = m;
            }
}
static void pool_i(const int32_t *x, int32_t *out, int C, int H, int W) {
    int Ho = H / 2, Wo = W / 2;
    for (int c = 0; c < C; ++c)
        for (int oy = 0; oy < Ho; ++oy)
            for (int ox = 0; ox < Wo; ++ox) {
                const int32_t *r0 = x + ((size_t)c * H + 2 * oy) * W + 2 * ox, *r1 = r0 + W;
                int32_t m = r0[0];
                if (r0[1] > m) m = r0[1];
                if (r1[0] > m) m = r1[0];
                if (r1[1] > m) m = r1[1];
                out[((size_t)c * Ho + oy) * Wo + ox] = m;
            }
}

/* nearest 2x upsample of x placed at offset d/2 inside the skip's size,
 * concat [skip, up], 0 where the upsample does not reach
 * (csrc/bnn_model_react.c:263-283) */
static float *upcat_f(const float *skip, int sC, int sH, int sW, const float *x, int xC, int hH, int hW) {
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

/* fp32 1x1 head from the bias, channels in order, fused multiply-adds
 * (head_1x1_v2, csrc/bnn_react_opt.c:26-43) */
static void head(const float *a, const float *Wm, const float *bias, float *lg, int Cin, size_t HW, int Cout) {
    for (int o = 0; o < Cout; ++o)
        for (size_t p = 0; p < HW; ++p) {
            float v = bias[o];
            for (int c = 0; c < Cin; ++c) v = fmaf(Wm[(size_t)o * Cin + c], a[(size_t)c * HW + p], v);
            lg[(size_t)o * HW + p] = v;
        }
}

/* ---------------------------------------------------------------- forward */
static void emit(oracle_stage_cb cb, void *ctx, const char *blk, const char *st, int kind, int C, int H, int W,
                 const void *d) {
    if (!cb) return;
    char nm[64];
    snprintf(nm, sizeof nm, "%s.%s", blk, st);
    cb(ctx, nm, kind, C, H, W, d);
}

static int8_t *bits_of(const float *x, int C, size_t HW, const float *rsign) {
    int8_t *a = malloc((size_t)C * HW ? (size_t)C * HW : 1);
    tap(x, a, C, HW, rsign);
    return a;
}

/* unit1 of a binary-input block (csrc/bnn_model_react.c:186-199): returns h1 */
static float *unit1(const RBlock *b, const float *x, int H, int W, const char *blk, oracle_stage_cb cb, void *ctx) {
    size_t HW = (size_t)H * W;
    int Ci = b->conv1.Cin, Co = b->conv1.Cout;
    float *res = malloc((size_t)Co * HW * 4 + 4);
    oracle_react_proj(x, b->proj1.W, res, Ci, H, W, Co);
    emit(cb, ctx, blk, "proj", 2, Co, H, W, res);
    int8_t *a = bits_of(x, Ci, HW, b->tap1.rsign);
    emit(cb, ctx, blk, "tap1", 0, Ci, H, W, a);
    int32_t *P = malloc((size_t)Co * HW * 4 + 4);
    oracle_bconv_P(a, b->conv1.packed, P, Ci, H, W, Co, 3, 3, 1, 1);
    emit(cb, ctx, blk, "conv1.P", 1, Co, H, W, P);
    free(a);
    float *h1 = malloc((size_t)Co * HW * 4 + 4);
    epi_i(P, res, h1, Co, HW, &b->epi1);
    emit(cb, ctx, blk, "h1", 2, Co, H, W, h1);
    free(P);
    free(res);
    return h1;
}

/* tap2 + conv2 of every block */
static int32_t *unit2_P(const RBlock *b, const float *h1, int H, int W, const char *blk, oracle_stage_cb cb,
                        void *ctx) {
    size_t HW = (size_t)H * W;
    int C = b->conv2.Cin, Co = b->conv2.Cout;
    int8_t *a = bits_of(h1, C, HW, b->tap2.rsign);
    emit(cb, ctx, blk, "tap2", 0, C, H, W, a);
    int32_t *P = malloc((size_t)Co * HW * 4 + 4);
    oracle_bconv_P(a, b->conv2.packed, P, C, H, W, Co, 3, 3, 1, 1);
    emit(cb, ctx, blk, "conv2.P", 1, Co, H, W, P);
    free(a);
    return P;
}

static const char *ENC[4] = {"enc1", "enc2", "enc3", "enc4"};
static const char *DEC[4] = {"dec4", "dec3", "dec2", "dec1"};

/* the forward of csrc/bnn_model_react.c:395-441 on the whole image (the
 * reference's enc1 / dec1 row strips with a 2-row halo produce the same
 * values: every output row is computed from the same in-image rows) */
int oracle_react_forward(const ORModel *m, const float *input, int H, int W, float *logits, oracle_stage_cb cb,
                         void *ctx) {
    if (H < 16 || W < 16) return -1;
    float *skip[4];
    int sC[4], sH[4], sW[4];
    float *x = NULL;
    int xC = 0, xH = H, xW = W;
    for (int i = 0; i < 4; ++i) {
        const RBlock *b = &m->enc[i];
        size_t HW = (size_t)xH * xW;
        int Co = b->conv2.Cout;
        float *h1;
        if (i == 0) {
            /* enc1 unit1: raw bands, real conv + real epilogue (:222-236) */
            const RConv *c1 = &b->conv1;
            float *res = malloc((size_t)c1->Cout * HW * 4 + 4);
            oracle_react_proj(input, b->proj1.W, res, c1->Cin, xH, xW, c1->Cout);
            emit(cb, ctx, "enc1", "proj", 2, c1->Cout, xH, xW, res);
            float *co1 = malloc((size_t)c1->Cout * HW * 4 + 4);
            if (c1->Cout % 8 == 0)
                oracle_react_conv3(input, c1->wsign, c1->alpha, co1, c1->Cin, xH, xW, c1->Cout);
            else  /* conv_realin_naive (:153-159) */
                oracle_realin(input, c1->wsign, c1->alpha, co1, c1->Cin, xH, xW, c1->Cout, 3, 3, 1, 1);
            emit(cb, ctx, "enc1", "conv1.out", 2, c1->Cout, xH, xW, co1);
            h1 = malloc((size_t)c1->Cout * HW * 4 + 4);
            epi_f(co1, res, h1, c1->Cout, HW, &b->epi1);
            emit(cb, ctx, "enc1", "h1", 2, c1->Cout, xH, xW, h1);
            free(co1);
            free(res);
        } else {
            h1 = unit1(b, x, xH, xW, ENC[i], cb, ctx);
            free(x);
        }
        int32_t *P2 = unit2_P(b, h1, xH, xW, ENC[i], cb, ctx);
        skip[i] = malloc((size_t)Co * HW * 4 + 4);
        epi_i(P2, h1, skip[i], Co, HW, &b->epi_a);
        emit(cb, ctx, ENC[i], "skip", 2, Co, xH, xW, skip[i]);
        sC[i] = Co; sH[i] = xH; sW[i] = xW;
        int Hh = xH / 2, Wh = xW / 2;
        size_t HWh = (size_t)Hh * Wh;
        int32_t *Pd = malloc((size_t)Co * HWh * 4 + 4);
        pool_i(P2, Pd, Co, xH, xW);
        emit(cb, ctx, ENC[i], "pool.P", 1, Co, Hh, Wh, Pd);
        free(P2);
        float *h1d = malloc((size_t)Co * HWh * 4 + 4);
        pool_f(h1, h1d, Co, xH, xW);
        emit(cb, ctx, ENC[i], "poolr", 2, Co, Hh, Wh, h1d);
        free(h1);
        x = malloc((size_t)Co * HWh * 4 + 4);
        epi_i(Pd, h1d, x, Co, HWh, &b->epi_b);
        emit(cb, ctx, ENC[i], "down", 2, Co, Hh, Wh, x);
        free(Pd);
        free(h1d);
        xC = Co; xH = Hh; xW = Wh;
    }
    {
        const RBlock *b = &m->bott;
        size_t HW = (size_t)xH * xW;
        float *h1 = unit1(b, x, xH, xW, "bottleneck", cb, ctx);
        free(x);
        int32_t *P2 = unit2_P(b, h1, xH, xW, "bottleneck", cb, ctx);
        x = malloc((size_t)b->conv2.Cout * HW * 4 + 4);
        epi_i(P2, h1, x, b->conv2.Cout, HW, &b->epi_a);
        emit(cb, ctx, "bottleneck", "h2", 2, b->conv2.Cout, xH, xW, x);
        free(P2);
        free(h1);
        xC = b->conv2.Cout;
    }
    for (int i = 0; i < 4; ++i) {
        const RBlock *b = &m->dec[i];
        int si = 3 - i, H2 = sH[si], W2 = sW[si];
        size_t HW = (size_t)H2 * W2;
        float *cat = upcat_f(skip[si], sC[si], H2, W2, x, xC, xH, xW);
        emit(cb, ctx, DEC[i], "cat", 2, sC[si] + xC, H2, W2, cat);
        free(x);
        free(skip[si]);
        float *h1 = unit1(b, cat, H2, W2, DEC[i], cb, ctx);
        free(cat);
        int32_t *P2 = unit2_P(b, h1, H2, W2, DEC[i], cb, ctx);
        x = malloc((size_t)b->conv2.Cout * HW * 4 + 4);
        epi_i(P2, h1, x, b->conv2.Cout, HW, &b->epi_a);
        emit(cb, ctx, DEC[i], "h2", 2, b->conv2.Cout, H2, W2, x);
        free(P2);
        free(h1);
        xC = b->conv2.Cout; xH = H2; xW = W2;
    }
    head(x, m->head_W, m->head_bias, logits, m->head_Cin, (size_t)H * W, m->head_Cout);
    if (cb) cb(ctx, "logits", 2, m->n_classes, H, W, logits);
    free(x);
    return 0;
}

int oracle_react_forward_batch(const ORModel *m, const float *input, int n, int H, int W, float *logits) {
    size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    for (int i = 0; i < n; ++i) {
        int rc = oracle_react_forward(m, input + (size_t)i * ip, H, W, logits + (size_t)i * op, NULL, NULL);
        if (rc) return rc;
    }
    return 0;
}
