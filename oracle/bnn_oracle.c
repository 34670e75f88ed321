/* bnn_oracle.c - TEST INFRASTRUCTURE ONLY (see bnn_oracle.h).
 *
 * CPU restatement of the reference v1 binary-UNet forward. Written for
 * clarity over speed: +-1 integer arithmetic straight from the definitions,
 * fp32 work in exactly the reference's operation order. Each function names
 * the reference file:line whose behaviour it restates (paths relative to the
 * reference project root).
 *
 * Build with -ffp-contract=off: the only fused multiply-add is the explicit
 * fmaf() in the real fold, matching the reference as built by its Makefile
 * (-O3 -march=native on an FMA-capable x86 contracts exactly that one
 * expression; the products in the two convs and the head are exact, +-1
 * times a float, so fused or not gives the same bits there).
 */
#include "bnn_oracle.h"
#include "../include/bnn_synth.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* blob parsing: csrc/bnn_model.c:27-96, python/bnn2c/blob.py:181-199  */
/* ------------------------------------------------------------------ */
typedef struct {
    int tag, Cout, Cin, kh, kw, pad, stride, nwords;
    uint64_t *packed;
    int8_t *wsign;
    float *alpha;
} OConv;

typedef struct {
    int kind, C;
    int32_t *type, *t, *lo, *hi;
    float *A, *B, *slope, *rsign;
} OAct;

struct OModel {
    int version, base_channels, n_bands, n_classes, upsampler;
    /* v2 (spectral stem, csrc/bnn_model_stem.h:43-47): a real-input 1x1
     * binary-weight conv + real fold before enc1, whose conv1 is binary */
    int has_stem;
    OConv stem_conv;
    OAct stem_act;
    OConv enc_conv1[4], enc_conv2[4];
    OAct enc_act1[4], enc_skip[4], enc_down[4];
    OConv bott_conv1, bott_conv2;
    OAct bott_act1, bott_act2;
    OConv dec_conv1[4], dec_conv2[4];
    OAct dec_act1[4], dec_act2[4];
    int head_Cout, head_Cin;
    float *head_W, *head_bias;
};

typedef struct {
    const unsigned char *p;
    size_t n, off;
    char *err;
    int errlen;
    int bad;
} Rd;

static void rd_fail(Rd *r, const char *msg) {
    if (!r->bad) snprintf(r->err, (size_t)r->errlen, "%s", msg);
    r->bad = 1;
}

static void rd_bytes(Rd *r, void *dst, size_t n) {
    if (r->bad) return;
    if (r->n - r->off < n) { rd_fail(r, "short read"); return; }
    memcpy(dst, r->p + r->off, n);
    r->off += n;
}

static int rd_int(Rd *r) { int32_t v = 0; rd_bytes(r, &v, 4); return v; }

static void *rd_alloc(Rd *r, size_t n) {
    if (r->bad) return NULL;
    if (r->n - r->off < n) { rd_fail(r, "short read"); return NULL; }
    void *p = malloc(n ? n : 1);
    if (!p) { rd_fail(r, "OOM"); return NULL; }
    rd_bytes(r, p, n);
    return p;
}

/* load_conv: csrc/bnn_model.c:27-44 */
static void rd_conv(Rd *r, OConv *c) {
    memset(c, 0, sizeof *c);
    c->tag = rd_int(r);
    c->Cout = rd_int(r); c->Cin = rd_int(r); c->kh = rd_int(r); c->kw = rd_int(r);
    c->pad = rd_int(r); c->stride = rd_int(r);
    if (r->bad) return;
    if (c->Cout < 0 || c->Cin < 0 || c->kh < 0 || c->kw < 0) { rd_fail(r, "bad conv dims"); return; }
    if (c->tag == 1) {
        c->nwords = rd_int(r);
        if (c->nwords < 0) { rd_fail(r, "bad nwords"); return; }
        c->packed = rd_alloc(r, (size_t)c->Cout * (size_t)c->nwords * 8);
    } else if (c->tag == 2) {
        size_t nw = (size_t)c->Cout * c->Cin * c->kh * c->kw;
        c->wsign = rd_alloc(r, nw);
        c->alpha = rd_alloc(r, (size_t)c->Cout * 4);
    } else {
        char m[64]; snprintf(m, sizeof m, "bad conv tag %d", c->tag); rd_fail(r, m);
    }
}

/* load_act: csrc/bnn_model.c:46-64 */
static void rd_act(Rd *r, OAct *a) {
    memset(a, 0, sizeof *a);
    int tag = rd_int(r);
    if (r->bad) return;
    if (tag != 3) { char m[64]; snprintf(m, sizeof m, "bad act tag %d", tag); rd_fail(r, m); return; }
    a->kind = rd_int(r); a->C = rd_int(r);
    if (r->bad) return;
    if (a->C < 0) { rd_fail(r, "bad act C"); return; }
    size_t C4 = (size_t)a->C * 4;
    if (a->kind == 0) {
        a->type = rd_alloc(r, C4); a->t = rd_alloc(r, C4);
        a->lo = rd_alloc(r, C4);   a->hi = rd_alloc(r, C4);
    } else {
        a->A = rd_alloc(r, C4);     a->B = rd_alloc(r, C4);
        a->slope = rd_alloc(r, C4); a->rsign = rd_alloc(r, C4);
    }
}

static void free_conv(OConv *c) { free(c->packed); free(c->wsign); free(c->alpha); }
static void free_act(OAct *a) {
    free(a->type); free(a->t); free(a->lo); free(a->hi);
    free(a->A); free(a->B); free(a->slope); free(a->rsign);
}

void oracle_free(OModel *m) {
    if (m && m->has_stem) { free_conv(&m->stem_conv); free_act(&m->stem_act); }
    if (!m) return;
    for (int i = 0; i < 4; ++i) {
        free_conv(&m->enc_conv1[i]); free_conv(&m->enc_conv2[i]);
        free_act(&m->enc_act1[i]); free_act(&m->enc_skip[i]); free_act(&m->enc_down[i]);
        free_conv(&m->dec_conv1[i]); free_conv(&m->dec_conv2[i]);
        free_act(&m->dec_act1[i]); free_act(&m->dec_act2[i]);
    }
    free_conv(&m->bott_conv1); free_conv(&m->bott_conv2);
    free_act(&m->bott_act1); free_act(&m->bott_act2);
    free(m->head_W); free(m->head_bias);
    free(m);
}

/* bnn_load: csrc/bnn_model.c:66-96 (magic, 5-int header, 18 conv + 22 act
 * records in fixed order, head, no trailing bytes). */
OModel *oracle_load(const char *path, char *err, int errlen) {
    FILE *f = fopen(path, "rb");
    if (!f) { snprintf(err, (size_t)errlen, "cannot open %s", path); return NULL; }
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    unsigned char *buf = malloc(sz > 0 ? (size_t)sz : 1);
    if (!buf || fread(buf, 1, (size_t)sz, f) != (size_t)sz) {
        fclose(f); free(buf); snprintf(err, (size_t)errlen, "read error"); return NULL;
    }
    fclose(f);
    Rd r = {buf, (size_t)sz, 0, err, errlen, 0};
    char magic[4] = {0};
    rd_bytes(&r, magic, 4);
    if (!r.bad && memcmp(magic, "BNNC", 4) != 0) rd_fail(&r, "bad magic");
    OModel *m = calloc(1, sizeof *m);
    if (!m) { free(buf); snprintf(err, (size_t)errlen, "OOM"); return NULL; }
    m->version = rd_int(&r); m->base_channels = rd_int(&r);
    m->n_bands = rd_int(&r); m->n_classes = rd_int(&r); m->upsampler = rd_int(&r);
    if (!r.bad && m->version == 2) {
        /* csrc/bnn_model_stem.c:82-95: has_stem, n_stem_layers (both 1), stem records */
        m->has_stem = rd_int(&r);
        int nsl = rd_int(&r);
        if (!r.bad && (m->has_stem != 1 || nsl != 1))
            rd_fail(&r, "bnn_stem: only has_stem=1, n_stem_layers=1 supported");
        rd_conv(&r, &m->stem_conv);
        rd_act(&r, &m->stem_act);
    }
    for (int i = 0; i < 4; ++i) {
        rd_conv(&r, &m->enc_conv1[i]); rd_act(&r, &m->enc_act1[i]);
        rd_conv(&r, &m->enc_conv2[i]); rd_act(&r, &m->enc_skip[i]);
        rd_act(&r, &m->enc_down[i]);
    }
    rd_conv(&r, &m->bott_conv1); rd_act(&r, &m->bott_act1);
    rd_conv(&r, &m->bott_conv2); rd_act(&r, &m->bott_act2);
    for (int i = 0; i < 4; ++i) {
        rd_conv(&r, &m->dec_conv1[i]); rd_act(&r, &m->dec_act1[i]);
        rd_conv(&r, &m->dec_conv2[i]); rd_act(&r, &m->dec_act2[i]);
    }
    int tag = rd_int(&r);
    if (!r.bad && tag != 4) { char msg[64]; snprintf(msg, sizeof msg, "bad head tag %d", tag); rd_fail(&r, msg); }
    m->head_Cout = rd_int(&r); m->head_Cin = rd_int(&r);
    if (!r.bad && (m->head_Cout < 0 || m->head_Cin < 0)) rd_fail(&r, "bad head dims");
    m->head_W = rd_alloc(&r, (size_t)m->head_Cout * m->head_Cin * 4);
    m->head_bias = rd_alloc(&r, (size_t)m->head_Cout * 4);
    if (!r.bad && r.off != r.n) rd_fail(&r, "trailing bytes in blob");
    free(buf);
    if (r.bad) { oracle_free(m); return NULL; }
    return m;
}

int oracle_n_bands(const OModel *m) { return m->n_bands; }
int oracle_n_classes(const OModel *m) { return m->n_classes; }
int oracle_base_channels(const OModel *m) { return m->base_channels; }

/* ------------------------------------------------------------------ */
/* kernels                                                              */
/* ------------------------------------------------------------------ */
static int odim(int in, int k, int pad, int stride) { return (in + 2 * pad - k) / stride + 1; }

/* pack_weights: csrc/bnn_conv.c:80-95 / blob.py:47-58.
 * kidx = (ci*kh + ky)*kw + kx; bit kidx&63 of word kidx>>6 set iff w > 0. */
void oracle_pack_weights(const int8_t *wsign, uint64_t *packed, int Cout,
                         int Cin, int kh, int kw) {
    int K = Cin * kh * kw, nw = (K + 63) / 64;
    memset(packed, 0, (size_t)Cout * nw * 8);
    for (int co = 0; co < Cout; ++co)
        for (int k = 0; k < K; ++k)
            if (wsign[(size_t)co * K + k] > 0)
                packed[(size_t)co * nw + (k >> 6)] |= (uint64_t)1 << (k & 63);
}

/* Binary conv accumulator as bconv_dispatch produces it
 * (csrc/bnn_conv.c:100-223): P = sum over in-bounds taps and all Cin of
 * w*a with w = bit(kidx) ? +1 : -1 and a = (a_int8 > 0) ? +1 : -1. Padded
 * (out-of-image) taps contribute nothing. Note a = 0 counts as -1 here,
 * which is what both packed kernels do (bnn_conv.c:123,162); the decoder's
 * zero-filled up_cat border relies on it. */
void oracle_bconv_P(const int8_t *a, const uint64_t *pw, int32_t *P, int Cin,
                    int H, int W, int Cout, int kh, int kw, int pad,
                    int stride) {
    int Ho = odim(H, kh, pad, stride), Wo = odim(W, kw, pad, stride);
    int K = Cin * kh * kw, nw = (K + 63) / 64;
    for (int co = 0; co < Cout; ++co) {
        const uint64_t *w = pw + (size_t)co * nw;
        for (int oy = 0; oy < Ho; ++oy)
            for (int ox = 0; ox < Wo; ++ox) {
                int32_t acc = 0;
                for (int ci = 0; ci < Cin; ++ci)
                    for (int ky = 0; ky < kh; ++ky) {
                        int iy = oy * stride + ky - pad;
                        if (iy < 0 || iy >= H) continue;
                        for (int kx = 0; kx < kw; ++kx) {
                            int ix = ox * stride + kx - pad;
                            if (ix < 0 || ix >= W) continue;
                            int k = (ci * kh + ky) * kw + kx;
                            int wv = ((w[k >> 6] >> (k & 63)) & 1) ? 1 : -1;
                            int av = a[((size_t)ci * H + iy) * W + ix] > 0 ? 1 : -1;
                            acc += wv * av;
                        }
                    }
                P[((size_t)co * Ho + oy) * Wo + ox] = acc;
            }
    }
}

/* bconv_xnor_packed: csrc/bnn_conv.c:145-213, on an input that is already
 * channel-packed per pixel (the reference packs a[Cin][H][W] into
 * apack[H*W][Wc] first, :156-164; here the words are 32 channels wide,
 * bits [H][W][ceil(Cin/32)], channel c -> bit c&31 of word c>>5). The
 * weights are repacked from kidx order to [Cout][9][cw] (:166-180); per
 * output, over the in-bounds taps only, P = 2 * (equal bits) - valid, the
 * last word masked to the Cin tail (:183-208). 3x3, pad 1, stride 1.
 * Same integers as oracle_bconv_P, fast enough for the 512-channel,
 * 128x128 sweep shapes. */
__attribute__((target("popcnt")))
void oracle_bconv_P_bits(const uint32_t *bits, const uint64_t *pw, int32_t *P,
                         int Cin, int H, int W, int Cout) {
    int cw = (Cin + 31) / 32, nwords = (9 * Cin + 63) / 64;
    uint32_t tail = (Cin & 31) ? ((1u << (Cin & 31)) - 1u) : 0xFFFFFFFFu;
    uint32_t *wp = calloc((size_t)Cout * 9 * cw, sizeof(uint32_t));
    if (!wp) return;
    for (int co = 0; co < Cout; ++co)
        for (int ci = 0; ci < Cin; ++ci)
            for (int t = 0; t < 9; ++t) {
                int k = ci * 9 + t;
                if ((pw[(size_t)co * nwords + (k >> 6)] >> (k & 63)) & 1)
                    wp[((size_t)co * 9 + t) * cw + (ci >> 5)] |= 1u << (ci & 31);
            }
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            int ky0 = y == 0 ? 1 : 0, ky1 = y == H - 1 ? 2 : 3;
            int kx0 = x == 0 ? 1 : 0, kx1 = x == W - 1 ? 2 : 3;
            int valid = (ky1 - ky0) * (kx1 - kx0) * Cin;
            for (int co = 0; co < Cout; ++co) {
                int eq = 0;
                for (int ky = ky0; ky < ky1; ++ky)
                    for (int kx = kx0; kx < kx1; ++kx) {
                        const uint32_t *a = bits + ((size_t)(y + ky - 1) * W + (x + kx - 1)) * cw;
                        const uint32_t *w = wp + ((size_t)co * 9 + ky * 3 + kx) * cw;
                        for (int j = 0; j < cw; ++j) {
                            uint32_t m = j == cw - 1 ? tail : 0xFFFFFFFFu;
                            eq += __builtin_popcount(~(a[j] ^ w[j]) & m);
                        }
                    }
                P[((size_t)co * H + y) * W + x] = 2 * eq - valid;
            }
        }
    free(wp);
}

/* conv_realin_general: csrc/bnn_conv_realin.c:66-116. Per output: for each
 * in-bounds tap in row-major (ky,kx) order, s = sequential fp32 sum over ci
 * of x*w (w = +-1, product exact), acc += s; out = alpha*acc. */
void oracle_realin(const float *x, const int8_t *wsign, const float *alpha,
                   float *out, int Cin, int H, int W, int Cout, int kh, int kw,
                   int pad, int stride) {
    int Ho = odim(H, kh, pad, stride), Wo = odim(W, kw, pad, stride);
    for (int co = 0; co < Cout; ++co)
        for (int oy = 0; oy < Ho; ++oy)
            for (int ox = 0; ox < Wo; ++ox) {
                float acc = 0.0f;
                for (int ky = 0; ky < kh; ++ky) {
                    int iy = oy * stride - pad + ky;
                    if (iy < 0 || iy >= H) continue;
                    for (int kx = 0; kx < kw; ++kx) {
                        int ix = ox * stride - pad + kx;
                        if (ix < 0 || ix >= W) continue;
                        float s = 0.0f;
                        for (int ci = 0; ci < Cin; ++ci) {
                            float xv = x[((size_t)ci * H + iy) * W + ix];
                            float wv = (float)wsign[(((size_t)co * Cin + ci) * kh + ky) * kw + kx];
                            s = s + xv * wv;
                        }
                        acc = acc + s;
                    }
                }
                out[((size_t)co * Ho + oy) * Wo + ox] = alpha[co] * acc;
            }
}

/* apply_fold_int: csrc/bnn_fold.c:37-60. Rule per channel: 0 const (t>0),
 * 1 P>=t, 2 P<t, 3 lo<=P<hi, 4 P<lo||P>=hi, anything else -> -1. */
void oracle_fold_int(const int32_t *P, int8_t *out, int C, int H, int W,
                     const int32_t *type, const int32_t *t, const int32_t *lo,
                     const int32_t *hi) {
    size_t HW = (size_t)H * W;
    for (int c = 0; c < C; ++c)
        for (size_t p = 0; p < HW; ++p) {
            int32_t v = P[c * HW + p];
            int b;
            switch (type[c]) {
                case 0: b = t[c] > 0; break;
                case 1: b = v >= t[c]; break;
                case 2: b = v < t[c]; break;
                case 3: b = v >= lo[c] && v < hi[c]; break;
                case 4: b = v < lo[c] || v >= hi[c]; break;
                default: b = 0; break;
            }
            out[c * HW + p] = b ? 1 : -1;
        }
}

/* apply_fold_real: csrc/bnn_fold.c:62-77, as the reference Makefile builds
 * it on x86 with FMA: z = fma(A, x, B); z < 0 -> z = slope*z (rounded);
 * r = z + rsign (rounded); +1 iff r > 0. */
void oracle_fold_real(const float *x, int8_t *out, int C, int H, int W,
                      const float *A, const float *B, const float *slope,
                      const float *rsign) {
    size_t HW = (size_t)H * W;
    for (int c = 0; c < C; ++c)
        for (size_t p = 0; p < HW; ++p) {
            float z = fmaf(A[c], x[c * HW + p], B[c]);
            if (z < 0.0f) z = slope[c] * z;
            float r = z + rsign[c];
            out[c * HW + p] = r > 0.0f ? 1 : -1;
        }
}

/* maxpool_P: csrc/bnn_maxpool.c:28-48 (k x k / stride, floor). */
void oracle_maxpool(const int32_t *P, int32_t *Pout, int C, int H, int W,
                    int k, int stride) {
    int Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
    if (Ho < 0) Ho = 0;
    if (Wo < 0) Wo = 0;
    for (int c = 0; c < C; ++c)
        for (int oy = 0; oy < Ho; ++oy)
            for (int ox = 0; ox < Wo; ++ox) {
                int32_t mx = INT32_MIN;
                for (int dy = 0; dy < k; ++dy)
                    for (int dx = 0; dx < k; ++dx) {
                        int32_t v = P[((size_t)c * H + oy * stride + dy) * W + ox * stride + dx];
                        if (v > mx) mx = v;
                    }
                Pout[((size_t)c * Ho + oy) * Wo + ox] = mx;
            }
}

/* up_cat: csrc/bnn_model.c:130-148. out[0:sC] = skip; out[sC:] = nearest 2x
 * of x placed at offset (d/2) when the skip is larger; everything the
 * upsample does not cover stays 0. */
void oracle_up_cat(const int8_t *skip, int sC, int sH, int sW, const int8_t *x,
                   int xC, int hH, int hW, int8_t *out) {
    size_t plane = (size_t)sH * sW;
    memset(out, 0, (size_t)(sC + xC) * plane);
    memcpy(out, skip, (size_t)sC * plane);
    int upH = 2 * hH, upW = 2 * hW;
    int dh = sH - upH, dw = sW - upW;
    int oh = dh > 0 ? dh / 2 : 0, ow = dw > 0 ? dw / 2 : 0;
    int cH = upH < sH ? upH : sH, cW = upW < sW ? upW : sW;
    for (int c = 0; c < xC; ++c)
        for (int y = 0; y < cH; ++y)
            for (int xx = 0; xx < cW; ++xx)
                out[(size_t)(sC + c) * plane + (size_t)(oh + y) * sW + (ow + xx)] =
                    x[((size_t)c * hH + y / 2) * hW + xx / 2];
}

/* head_1x1: csrc/bnn_head.c:21-34; acc starts at bias, sequential over c. */
void oracle_head(const float *a, const float *Wt, const float *bias,
                 float *logits, int Cin, int H, int W, int Cout) {
    size_t HW = (size_t)H * W;
    for (int o = 0; o < Cout; ++o)
        for (size_t p = 0; p < HW; ++p) {
            float acc = bias[o];
            for (int c = 0; c < Cin; ++c) acc = acc + Wt[(size_t)o * Cin + c] * a[c * HW + p];
            logits[o * HW + p] = acc;
        }
}

void oracle_synth(uint32_t seed, uint32_t patch0, int n, int bands, int H,
                  int W, float *out) {
    size_t per = (size_t)bands * H * W;
    for (int i = 0; i < n; ++i)
        for (size_t e = 0; e < per; ++e)
            out[(size_t)i * per + e] = bnn_synth_value(seed, patch0 + (uint32_t)i, (uint32_t)e);
}

/* ------------------------------------------------------------------ */
/* forward: csrc/bnn_model.c:150-253                                   */
/* ------------------------------------------------------------------ */
static void *xm(size_t n) { return malloc(n ? n : 1); }

static void emit(oracle_stage_cb cb, void *ctx, const char *name, int kind,
                 int C, int H, int W, const void *d) {
    if (cb) cb(ctx, name, kind, C, H, W, d);
}

static void fold(const OAct *a, const int32_t *P, const float *xr, int8_t *out,
                 int C, int H, int W) {
    if (a->kind == 0) oracle_fold_int(P, out, C, H, W, a->type, a->t, a->lo, a->hi);
    else oracle_fold_real(xr, out, C, H, W, a->A, a->B, a->slope, a->rsign);
}

/* conv (+-1 in) -> P -> int fold; csrc/bnn_model.c:109-123 */
static int8_t *conv_fold(const OConv *c, const OAct *a, const int8_t *in, int H,
                         int W, const char *blk, const char *cname,
                         const char *aname, oracle_stage_cb cb, void *ctx) {
    char nm[64];
    int32_t *P = xm((size_t)c->Cout * H * W * 4);
    oracle_bconv_P(in, c->packed, P, c->Cin, H, W, c->Cout, c->kh, c->kw, c->pad, c->stride);
    snprintf(nm, sizeof nm, "%s.%s.P", blk, cname);
    emit(cb, ctx, nm, 1, c->Cout, H, W, P);
    int8_t *o = xm((size_t)c->Cout * H * W);
    fold(a, P, NULL, o, c->Cout, H, W);
    snprintf(nm, sizeof nm, "%s.%s", blk, aname);
    emit(cb, ctx, nm, 0, c->Cout, H, W, o);
    free(P);
    return o;
}

static const char *ENC[4] = {"enc1", "enc2", "enc3", "enc4"};
static const char *DEC[4] = {"dec4", "dec3", "dec2", "dec1"};

int oracle_forward(const OModel *m, const float *input, int H, int W,
                   float *logits, oracle_stage_cb cb, void *ctx) {
    char nm[64];
    /* Below 16 some encoder level is one pixel wide and the reference's
     * maxpool_P (bnn_maxpool.c:29-30, truncating division) writes a row
     * past the H/2 = 0 buffer bnn_forward allocated: undefined there, so
     * refused here. */
    if (H < 16 || W < 16) return -1;
    int8_t *skip[4];
    int sC[4], sH[4], sW[4];
    int8_t *x = NULL;
    int xC = 0, xH = H, xW = W;
    for (int i = 0; i < 4; ++i) {
        const OConv *c1 = &m->enc_conv1[i], *c2 = &m->enc_conv2[i];
        int8_t *h;
        if (i == 0 && m->has_stem) {
            /* v2: 1x1 real-input stem + real fold (csrc/bnn_model_stem.c:172-187),
             * then enc1.conv1 binary like the other levels (:189-193) */
            const OConv *sc = &m->stem_conv;
            float *so = xm((size_t)sc->Cout * H * W * 4);
            oracle_realin(input, sc->wsign, sc->alpha, so, sc->Cin, H, W, sc->Cout, sc->kh, sc->kw, sc->pad,
                          sc->stride);
            emit(cb, ctx, "stem.conv.out", 2, sc->Cout, H, W, so);
            int8_t *st = xm((size_t)sc->Cout * H * W);
            fold(&m->stem_act, NULL, so, st, sc->Cout, H, W);
            emit(cb, ctx, "stem.act", 0, sc->Cout, H, W, st);
            free(so);
            h = conv_fold(c1, &m->enc_act1[0], st, xH, xW, ENC[0], "conv1", "act1", cb, ctx);
            free(st);
        } else if (i == 0) {
            /* enc1: real-input conv + real fold (bnn_model.c:156-167) */
            float *co1 = xm((size_t)c1->Cout * H * W * 4);
            oracle_realin(input, c1->wsign, c1->alpha, co1, c1->Cin, H, W, c1->Cout,
                          c1->kh, c1->kw, c1->pad, c1->stride);
            emit(cb, ctx, "enc1.conv1.out", 2, c1->Cout, H, W, co1);
            h = xm((size_t)c1->Cout * H * W);
            fold(&m->enc_act1[0], NULL, co1, h, c1->Cout, H, W);
            emit(cb, ctx, "enc1.act1", 0, c1->Cout, H, W, h);
            free(co1);
        } else {
            h = conv_fold(c1, &m->enc_act1[i], x, xH, xW, ENC[i], "conv1", "act1", cb, ctx);
            free(x);
        }
        /* conv2 shared by skip and down (bnn_model.c:168-185, 193-215) */
        int32_t *P2 = xm((size_t)c2->Cout * xH * xW * 4);
        oracle_bconv_P(h, c2->packed, P2, c2->Cin, xH, xW, c2->Cout, c2->kh, c2->kw, c2->pad, c2->stride);
        free(h);
        snprintf(nm, sizeof nm, "%s.conv2.P", ENC[i]);
        emit(cb, ctx, nm, 1, c2->Cout, xH, xW, P2);
        skip[i] = xm((size_t)c2->Cout * xH * xW);
        fold(&m->enc_skip[i], P2, NULL, skip[i], c2->Cout, xH, xW);
        snprintf(nm, sizeof nm, "%s.act2_skip", ENC[i]);
        emit(cb, ctx, nm, 0, c2->Cout, xH, xW, skip[i]);
        sC[i] = c2->Cout; sH[i] = xH; sW[i] = xW;
        int Hh = xH / 2, Wh = xW / 2;
        int32_t *Pd = xm((size_t)c2->Cout * Hh * Wh * 4);
        oracle_maxpool(P2, Pd, c2->Cout, xH, xW, 2, 2);
        free(P2);
        snprintf(nm, sizeof nm, "%s.pool.P", ENC[i]);
        emit(cb, ctx, nm, 1, c2->Cout, Hh, Wh, Pd);
        x = xm((size_t)c2->Cout * Hh * Wh);
        fold(&m->enc_down[i], Pd, NULL, x, c2->Cout, Hh, Wh);
        free(Pd);
        snprintf(nm, sizeof nm, "%s.act2_down", ENC[i]);
        emit(cb, ctx, nm, 0, c2->Cout, Hh, Wh, x);
        xC = c2->Cout; xH = Hh; xW = Wh;
    }
    /* bottleneck (bnn_model.c:219-223) */
    {
        int8_t *h = conv_fold(&m->bott_conv1, &m->bott_act1, x, xH, xW, "bottleneck", "conv1", "act1", cb, ctx);
        free(x);
        x = conv_fold(&m->bott_conv2, &m->bott_act2, h, xH, xW, "bottleneck", "conv2", "act2", cb, ctx);
        free(h);
        xC = m->bott_conv2.Cout;
    }
    /* decoder dec4..dec1 (bnn_model.c:225-239) */
    for (int i = 0; i < 4; ++i) {
        int si = 3 - i;
        int H2 = sH[si], W2 = sW[si];
        int catC = sC[si] + xC;
        int8_t *cat = xm((size_t)catC * H2 * W2);
        oracle_up_cat(skip[si], sC[si], H2, W2, x, xC, xH, xW, cat);
        snprintf(nm, sizeof nm, "%s.cat", DEC[i]);
        emit(cb, ctx, nm, 0, catC, H2, W2, cat);
        free(x); free(skip[si]);
        int8_t *h = conv_fold(&m->dec_conv1[i], &m->dec_act1[i], cat, H2, W2, DEC[i], "conv1", "act1", cb, ctx);
        free(cat);
        x = conv_fold(&m->dec_conv2[i], &m->dec_act2[i], h, H2, W2, DEC[i], "conv2", "act2", cb, ctx);
        free(h);
        xC = m->dec_conv2[i].Cout; xH = H2; xW = W2;
    }
    /* head (bnn_model.c:241-251) */
    {
        size_t n = (size_t)xC * xH * xW;
        float *xf = xm(n * 4);
        for (size_t j = 0; j < n; ++j) xf[j] = (float)x[j];
        oracle_head(xf, m->head_W, m->head_bias, logits, m->head_Cin, xH, xW, m->head_Cout);
        emit(cb, ctx, "logits", 2, m->head_Cout, xH, xW, logits);
        free(xf);
    }
    free(x);
    return 0;
}

/* Patch-wise forward of a whole scene (csrc/bnn_model_react.c:454-476, the
 * reference's tiler, applied to the v1 forward): non-overlapping PxP tiles,
 * each cut from the [n_bands][H][W] cube and zero-padded at the right and
 * bottom edges, run through the full network as a standalone PxP image; the
 * in-scene part of each tile's logits is written to [n_classes][H][W]. */
int oracle_forward_patched(const OModel *m, const float *input, int H, int W,
                           float *logits, int P) {
    const int nb = m->n_bands, ncl = m->n_classes;
    if (P <= 0 || H <= 0 || W <= 0) return 1;
    float *pin = (float *)malloc((size_t)nb * P * P * sizeof(float));
    float *pout = (float *)malloc((size_t)ncl * P * P * sizeof(float));
    if (!pin || !pout) { free(pin); free(pout); return 1; }
    int rc = 0;
    for (int py = 0; py < H && !rc; py += P) {
        const int ph = py + P < H ? P : H - py;
        for (int px = 0; px < W && !rc; px += P) {
            const int pw = px + P < W ? P : W - px;
            memset(pin, 0, (size_t)nb * P * P * sizeof(float));
            for (int b = 0; b < nb; ++b)
                for (int y = 0; y < ph; ++y)
                    memcpy(pin + ((size_t)b * P + y) * P, input + ((size_t)b * H + py + y) * W + px,
                           (size_t)pw * sizeof(float));
            rc = oracle_forward(m, pin, P, P, pout, NULL, NULL);
            for (int c = 0; c < ncl && !rc; ++c)
                for (int y = 0; y < ph; ++y)
                    memcpy(logits + ((size_t)c * H + py + y) * W + px, pout + ((size_t)c * P + y) * P,
                           (size_t)pw * sizeof(float));
        }
    }
    free(pin);
    free(pout);
    return rc;
}

int oracle_forward_batch(const OModel *m, const float *input, int n, int H,
                         int W, float *logits) {
    size_t in_per = (size_t)m->n_bands * H * W, out_per = (size_t)m->n_classes * H * W;
    for (int i = 0; i < n; ++i) {
        int rc = oracle_forward(m, input + i * in_per, H, W, logits + i * out_per, NULL, NULL);
        if (rc) return rc;
    }
    return 0;
}
