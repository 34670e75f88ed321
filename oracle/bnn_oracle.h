/* bnn_oracle.h - TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, CPU-only restatement of the reference engine's v1 forward path
 * (Sboyle132/BNNs_to_C csrc/bnn_model.c and the kernels it calls), of its
 * v2 spectral-stem variant (csrc/bnn_model_stem.c) and of the v3 ReActNet
 * engine (csrc/bnn_model_react.c, in bnn_oracle_react.c), written
 * from the reference's documented semantics, used as the checker for the
 * B200 engine. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it; the product library never links it.
 *
 * Parity pin: every function here is checked against the reference's own
 * sources compiled unmodified into oracle/_ref/ (recipe: oracle/Makefile),
 * through golden fixtures committed under tests/golden/.
 */
#ifndef BNN_ORACLE_H
#define BNN_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Stage callback: kind 0 = int8 (+-1 activation or concat), 1 = int32 P,
 * 2 = float32 (real conv output, logits). Layout [C][H][W]. */
typedef void (*oracle_stage_cb)(void *ctx, const char *name, int kind,
                                int C, int H, int W, const void *data);

typedef struct OModel OModel;

OModel *oracle_load(const char *path, char *err, int errlen);
void oracle_free(OModel *m);
int oracle_n_bands(const OModel *m);
int oracle_n_classes(const OModel *m);
int oracle_base_channels(const OModel *m);
/* returns 0 on success */
int oracle_forward(const OModel *m, const float *input, int H, int W,
                   float *logits, oracle_stage_cb cb, void *ctx);
/* n patches of [bands][H][W], contiguous */
int oracle_forward_patched(const OModel *m, const float *input, int H, int W,
                           float *logits, int P);
int oracle_forward_batch(const OModel *m, const float *input, int n, int H,
                         int W, float *logits);

/* kernels */
void oracle_pack_weights(const int8_t *wsign, uint64_t *packed, int Cout,
                         int Cin, int kh, int kw);
void oracle_bconv_P(const int8_t *a, const uint64_t *packed_w, int32_t *P,
                    int Cin, int H, int W, int Cout, int kh, int kw, int pad,
                    int stride);
void oracle_realin(const float *x, const int8_t *wsign, const float *alpha,
                   float *out, int Cin, int H, int W, int Cout, int kh,
                   int kw, int pad, int stride);
/* bconv_xnor_packed (csrc/bnn_conv.c:145-213) on channel-packed bits
 * [H][W][ceil(Cin/32)] (32 channels per word): P [Cout][H][W], 3x3 pad 1. */
void oracle_bconv_P_bits(const uint32_t *bits, const uint64_t *packed_w,
                         int32_t *P, int Cin, int H, int W, int Cout);
void oracle_fold_int(const int32_t *P, int8_t *out, int C, int H, int W,
                     const int32_t *type, const int32_t *t, const int32_t *lo,
                     const int32_t *hi);
void oracle_fold_real(const float *x, int8_t *out, int C, int H, int W,
                      const float *A, const float *B, const float *slope,
                      const float *rsign);
void oracle_maxpool(const int32_t *P, int32_t *Pout, int C, int H, int W,
                    int k, int stride);
void oracle_up_cat(const int8_t *skip, int sC, int sH, int sW,
                   const int8_t *x, int xC, int hH, int hW, int8_t *out);
void oracle_head(const float *a, const float *Wt, const float *bias,
                 float *logits, int Cin, int H, int W, int Cout);
void oracle_synth(uint32_t seed, uint32_t patch0, int n, int bands, int H,
                  int W, float *out);

/* v3 ReActNet real-highway engine (csrc/bnn_model_react.c), bnn_oracle_react.c.
 * Stages: "<block>.proj", ".tap1", ".conv1.P" (enc1: ".conv1.out"), ".h1",
 * ".tap2", ".conv2.P", then ".skip", ".pool.P", ".poolr", ".down" (encoder)
 * or ".h2"; decoder blocks start with ".cat"; "logits" last. */
typedef struct ORModel ORModel;
ORModel *oracle_react_load_mem(const void *data, size_t n, char *err, int errlen);
void oracle_react_free(ORModel *m);
int oracle_react_n_bands(const ORModel *m);
int oracle_react_n_classes(const ORModel *m);
int oracle_react_forward(const ORModel *m, const float *input, int H, int W,
                         float *logits, oracle_stage_cb cb, void *ctx);
int oracle_react_forward_batch(const ORModel *m, const float *input, int n,
                               int H, int W, float *logits);
void oracle_react_proj(const float *x, const float *Wm, float *out, int Cin,
                       int H, int W, int Cout);
void oracle_react_conv3(const float *x, const int8_t *wsign, const float *alpha,
                        float *out, int Cin, int H, int W, int Cout);

#ifdef __cplusplus
}
#endif
#endif
