/* bnn_model_stem.h - drop-in public header of the B200 engine for the v2
 * (spectral-stem) binary UNet.
 *
 * Replaces the reference's csrc/bnn_model_stem.h (Sboyle132/BNNs_to_C):
 * same ConvS / ActS / StemModel records with the same public fields in the
 * same order, same three entry points with the same signatures, argument
 * meaning, ownership and error behaviour (csrc/bnn_model_stem.c). A caller
 * of the reference's stem engine (csrc/main_stem.c) recompiles against this
 * header and links libbnn_b200.so.
 *
 * The reference header also declares its shared CPU kernels
 * (csrc/bnn_model_stem.h:14-24); they are not re-declared here: on this
 * engine they run on the GPU inside bnn_stem_forward. Their GPU-backed
 * host-pointer equivalents are in bnn_b200.h.
 *
 * The v2 network: a real-input 1x1 conv with +-1 weights (the stem) and a
 * real fold binarise the bands, then enc1..enc4 are all binary (enc1.conv1
 * included), the rest as in v1. This engine runs stems that are 1x1, pad 0,
 * stride 1 (what the reference's blob writer emits); others are refused at
 * load.
 */
#ifndef BNN_MODEL_STEM_H
#define BNN_MODEL_STEM_H
#include <stddef.h>
#include <stdint.h>

#include "bnn_model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Conv / activation records (reference csrc/bnn_model_stem.h:27-41),
 * field for field the same as bnn_model.h's Conv / Act. */
typedef struct {
    int tag;                 /* 1 = binary (packed), 2 = real (wsign+alpha) */
    int Cout, Cin, kh, kw, pad, stride, nwords;
    uint64_t *packed;
    int8_t *wsign;
    float *alpha;
} ConvS;

typedef struct {
    int kind;                /* 0 = integer-P fold, 1 = real fold */
    int C;
    int32_t *type, *t, *lo, *hi;
    float *A, *B, *slope, *rsign;
} ActS;

/* Parsed v2 blob (reference csrc/bnn_model_stem.h:43-61). `engine` is this
 * library's addition (the device state, released by bnn_stem_free); callers
 * never touch it. */
typedef struct StemModel {
    int version, base_channels, n_bands, n_classes, upsampler;
    int has_stem, n_stem_layers;   /* v2: has_stem==1, n_stem_layers==1 */
    ConvS stem_conv;
    ActS  stem_act;
    ConvS enc_conv1[4], enc_conv2[4];
    ActS  enc_act1[4], enc_act2_skip[4], enc_act2_down[4];
    ConvS bott_conv1, bott_conv2;
    ActS  bott_act1, bott_act2;
    ConvS dec_conv1[4], dec_conv2[4];
    ActS  dec_act1[4], dec_act2[4];
    int head_Cout, head_Cin;
    float *head_W, *head_bias;
    void *engine;
} StemModel;

/* Parse a v2 blob (reference csrc/bnn_model_stem.c:77-115: version must be
 * 2, has_stem == n_stem_layers == 1). On any error prints the reason to
 * stderr and exits with status 1, as the reference does. No GPU work. */
StemModel *bnn_stem_load(const char *path);

/* Release the model and its device state (reference
 * csrc/bnn_model_stem.c:260-271). NULL is a no-op. */
void bnn_stem_free(StemModel *m);

/* One patch: input [n_bands][H][W] float32 -> logits [n_classes][H][W]
 * float32, host memory the caller owns (reference
 * csrc/bnn_model_stem.c:168-255), on the calling thread's current CUDA
 * device; bit-identical to the reference. Errors print and exit(1). */
void bnn_stem_forward(const StemModel *m, const float *input, int H, int W, float *logits);

/* ---- extensions (no counterpart in the reference) ---- */

/* Status-returning forms of bnn_stem_load (codes of bnn_b200.h, message in
 * bnn_last_error()); the in-memory form parses `n` bytes at `data`. */
int bnn_stem_load_ex(const char *path, StemModel **out);
int bnn_stem_load_mem(const void *data, size_t n, StemModel **out);

/* The engine handle of a v2 model, accepted by every Model entry point of
 * bnn_model.h and bnn_b200.h (batched, device-pointer, patched-scene, stage
 * dump, devices, chunk, profiler), which then run the v2 forward. Its
 * fields describe the v2 body (enc_conv1[0] binary); it belongs to the
 * StemModel, stays valid until bnn_stem_free, and bnn_free on it is a
 * no-op. The stage dump reports "stem.conv.out" (float32) and "stem.act"
 * before "enc1.conv1.P". */
Model *bnn_stem_as_model(StemModel *m);

#ifdef __cplusplus
}
#endif
#endif
