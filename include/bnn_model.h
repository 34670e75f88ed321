/* bnn_model.h - drop-in public header of the B200 binary-UNet engine.
 *
 * Replaces the reference's csrc/bnn_model.h (Sboyle132/BNNs_to_C): same
 * structs with the same public fields in the same order, same three entry
 * points with the same signatures, argument meaning, ownership and error
 * behaviour. A caller of the reference engine (csrc/main.c, ctypes users)
 * recompiles against this header and links libbnn_b200.so instead of the
 * reference's bnn_model.c + kernel objects.
 *
 * The reference's CPU kernel prototypes (csrc/bnn_model.h:7-23) are not
 * re-declared: on this engine they run on the GPU inside bnn_forward. Their
 * GPU-backed host-pointer equivalents, plus the batched, device-pointer and
 * multi-GPU extensions, are in bnn_b200.h.
 */
#ifndef BNN_MODEL_H
#define BNN_MODEL_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One conv record of the blob (reference csrc/bnn_model.h:26-32). */
typedef struct {
    int tag;                 /* 1 = binary (packed), 2 = real (wsign+alpha) */
    int Cout, Cin, kh, kw, pad, stride, nwords;
    uint64_t *packed;        /* binary conv: [Cout][nwords], kidx bit order */
    int8_t *wsign;           /* real conv: [Cout][Cin][kh][kw] in {-1,+1} */
    float *alpha;            /* real conv: [Cout] */
} Conv;

/* One activation-fold record (reference csrc/bnn_model.h:34-39). */
typedef struct {
    int kind;                /* 0 = integer-P fold, 1 = real fold */
    int C;
    int32_t *type, *t, *lo, *hi;     /* int fold */
    float *A, *B, *slope, *rsign;    /* real fold */
} Act;

/* Parsed blob (reference csrc/bnn_model.h:41-55). `engine` is this
 * library's addition: per-device weight arenas, activation arenas and CUDA
 * graphs, owned by the Model and released by bnn_free. Callers never touch
 * it. */
typedef struct {
    int version, base_channels, n_bands, n_classes, upsampler;
    Conv enc_conv1[4], enc_conv2[4];
    Act  enc_act1[4], enc_act2_skip[4], enc_act2_down[4];
    Conv bott_conv1, bott_conv2;
    Act  bott_act1, bott_act2;
    Conv dec_conv1[4], dec_conv2[4];
    Act  dec_act1[4], dec_act2[4];
    int head_Cout, head_Cin;
    float *head_W, *head_bias;
    void *engine;
} Model;

/* Parse a v1 blob (reference csrc/bnn_model.c:66-96). On any error prints
 * the reason to stderr and exits with status 1, as the reference does. Pure
 * host work: no GPU is touched until the first forward. */
Model *bnn_load(const char *path);

/* Release the Model and everything it owns on every device it used
 * (reference csrc/bnn_model.c:258-268). NULL is a no-op. */
void bnn_free(Model *m);

/* One patch: input [n_bands][H][W] float32, logits [n_classes][H][W]
 * float32, both host memory the caller owns (reference
 * csrc/bnn_model.h:59-60, csrc/bnn_model.c:150-253). Runs on the calling
 * thread's current CUDA device. Results are bit-identical to the reference
 * engine's. Errors print and exit(1), matching the reference's behaviour. */
void bnn_forward(const Model *m, const float *input, int H, int W, float *logits);

#ifdef __cplusplus
}
#endif
#endif
