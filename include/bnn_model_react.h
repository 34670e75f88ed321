/* bnn_model_react.h - drop-in public header of the B200 engine for the v3
 * ReActNet real-highway binary UNet.
 *
 * Replaces the reference's csrc/bnn_model_react.h (Sboyle132/BNNs_to_C):
 * same ConvR / EpiR / TapR / ProjR / BlockR / ModelR records with the same
 * public fields in the same order, same entry points with the same
 * signatures, argument meaning, ownership and error behaviour
 * (csrc/bnn_model_react.c). A caller of the reference's ReAct engine
 * (csrc/main_react.c) recompiles against this header and links
 * libbnn_b200.so. The reference header's CPU kernel prototypes
 * (csrc/bnn_model_react.h:9-50) are not re-declared: on this engine that work
 * runs on the GPU inside the forwards.
 *
 * Results equal the reference engine built with gcc -O3 on x86 with FMA, bit
 * for bit (every highway value, tap, accumulator and logit); the fp32
 * roundings follow that build (fused multiply-adds where it contracts).
 */
#ifndef BNN_MODEL_REACT_H
#define BNN_MODEL_REACT_H
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#include "bnn_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Records (reference csrc/bnn_model_react.h:54-80). */
typedef struct {
    int tag;                 /* 1 = binary (packed), 2 = real (wsign+alpha) */
    int Cout, Cin, kh, kw, pad, stride, nwords;
    uint64_t *packed;
    int8_t *wsign;
    float *alpha;
} ConvR;

typedef struct { int kind, C; float *A, *B, *move1, *prelu_w; } EpiR;  /* kind 0=int 1=real */
typedef struct { int C; float *rsign; } TapR;                          /* C==0: absent (enc1) */
typedef struct { int Cout, Cin; float *W; } ProjR;                     /* real 1x1, no bias */

typedef struct {
    int is_down;             /* 1: DownBlock (fork), 0: PlainBlock */
    int input_real;          /* enc1 only: conv1 consumes raw spectra, no tap1 */
    TapR  tap1, tap2;
    ConvR conv1, conv2;
    ProjR proj1;
    EpiR  epi1;
    EpiR  epi_a;             /* down: skip epilogue ; plain: epi2 */
    EpiR  epi_b;             /* down: pooled-down epilogue ; plain: unused */
} BlockR;

/* Parsed v3 blob (reference csrc/bnn_model_react.h:82-88). `engine` is this
 * library's addition (device state, released by bnn_free_react). */
typedef struct {
    int version, base_channels, n_bands, n_classes, upsampler;
    BlockR enc[4], bott, dec[4];     /* dec[0..3] == dec4..dec1 */
    int head_Cout, head_Cin;
    float *head_W, *head_bias;
    void *engine;
} ModelR;

/* Parse a v3 blob (reference csrc/bnn_model_react.c:108-135, the same
 * structural checks and messages); errors print and exit(1). No GPU work. */
ModelR *bnn_load_react(const char *path);
void bnn_free_react(ModelR *m);

/* input: [n_bands,H,W] float; logits: [n_classes,H,W] float (caller allocs);
 * the current CUDA device; errors print and exit(1) (reference :443-446). */
void bnn_forward_react(const ModelR *m, const float *input, int H, int W, float *logits);
/* the cube read from a [n_bands,H,W] float32 file (reference :528-531) */
void bnn_forward_react_file(const ModelR *m, FILE *in_f, int H, int W, float *logits);
/* independent zero-padded PxP patches stitched (reference :454-476); P a
 * multiple of 16 */
void bnn_forward_react_patched(const ModelR *m, const float *input, int H, int W, float *logits, int P);
void bnn_forward_react_patched_file(const ModelR *m, FILE *f, int H, int W, float *logits, int P);

/* ---- extensions (no counterpart in the reference) ---- */

/* Status-returning loaders (codes of bnn_b200.h, message in bnn_last_error). */
int bnn_react_load_ex(const char *path, ModelR **out);
int bnn_react_load_mem(const void *data, size_t n, ModelR **out);

/* N patches [N][n_bands][H][W] -> logits [N][n_classes][H][W], host memory,
 * on the calling thread's current device; each patch equals
 * bnn_forward_react on it. Blocks until the logits are in host memory. */
int bnn_forward_react_batch(const ModelR *m, const float *input, int N, int H, int W, float *logits);
/* The same on device memory of `device`, enqueued on `stream` (NULL = legacy
 * default stream); repeated shapes replay one captured CUDA graph. */
int bnn_forward_react_device(const ModelR *m, int device, const float *d_input, int N, int H, int W,
                             float *d_logits, void *stream);
/* Status-returning form of bnn_forward_react_patched (same result; all the
 * tiles run as one batch on the current device). */
int bnn_forward_react_patched_ex(const ModelR *m, const float *input, int H, int W, float *logits, int P);
/* Debug / parity: one patch on the current device, every intermediate the
 * engine holds reported in forward order under the oracle's names
 * ("<block>.proj", ".tap1" / ".tap2" (int8 +-1), ".conv1.P" / ".conv2.P"
 * (int32), "enc1.conv1.out", ".h1", ".skip", ".down", ".h2" (float32),
 * "logits"); kinds as bnn_forward_stages. */
int bnn_forward_react_stages(const ModelR *m, const float *input, int H, int W, float *logits, bnn_stage_cb cb,
                             void *ctx);
/* Per-op profiler (CUDA events around each launch, eager launches while on),
 * the same record interface as bnn_profile_* for the v1 engine. */
int bnn_react_profile_enable(ModelR *m, int on);
void bnn_react_profile_reset(ModelR *m);
int bnn_react_profile_count(const ModelR *m);
int bnn_react_profile_get(const ModelR *m, int i, const char **label, const char **optype, double *work, double *ms,
                          int *calls);
/* A/B choice of the enc1 real-conv kernel: 0 = input staged by TMA through
 * a shared-memory ring (default where W % 4 == 0), 1 = thread-staged. Both
 * keep the reference's order, so both give its bits. */
int bnn_react_set_conv_kernel(int kind);
/* Bounded device waits of the ReAct kernels that gave up on `device` since
 * the library was loaded (expected to stay 0). */
int bnn_react_device_error(int device, unsigned int *wait_timeouts);
/* Kernel launches of one device forward of N patches of H x W. */
int bnn_react_forward_launches(const ModelR *m, int N, int H, int W);

#ifdef __cplusplus
}
#endif
#endif
