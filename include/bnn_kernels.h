/* bnn_kernels.h - the reference's kernel-level C ABI (csrc/bnn_model.h:7-23
 * and csrc/bnn_conv.c of Sboyle132/BNNs_to_C) on the GPU, exported under the
 * reference's own names from lib/libbnn_kernels.so (a library apart from
 * libbnn_b200.so, so that a program can link both this and the
 * reference's .c files without a clash).
 *
 * A harness that binds the reference's kernels with ctypes or links them
 * (python/verify/bconv_harness.py binds bconv_naive_int / pack_weights /
 * bconv_xnor from csrc/libbnnconv.so) runs unchanged against this library
 * with only the library path changed. Every function keeps the
 * reference's signature, host-pointer arguments, [C][H][W] row-major
 * layouts, batch size 1, output size (in + 2*pad - k) / stride + 1, and
 * result:
 *   - integer work (binary convs, max-pool, integer fold) bit-exact;
 *   - float work bit-exact in the reference's source operation order
 *     (conv_realin_naive, apply_fold_real, and head_1x1 on +-1 input),
 *     see head_1x1 for arbitrary float input.
 * Each call copies its inputs to the current CUDA device, runs there
 * (the 3x3 stride-1 binary convs and the 3x3 pad-1 stride-1 real-input
 * conv on the tcgen05 kernels of the forward, other shapes on direct
 * kernels) and returns when the output is back in host memory. Like the
 * reference, these functions return nothing: a failure (no device, out of
 * memory, an argument the reference cannot take either) prints a message
 * to stderr and exits with status 1. Nothing runs on the host CPU except
 * pack_weights, which is a host-side weight format conversion in the
 * reference too.
 */
#ifndef BNN_KERNELS_H
#define BNN_KERNELS_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* csrc/bnn_conv.c:50-76: P[co][oy][ox] = sum over in-image taps of
 * wsign * a (int8 products, padded taps contribute 0). */
void bconv_naive_int(const int8_t *a, const int8_t *wsign, int32_t *P, int Cin, int H, int W, int Cout,
                     int kh, int kw, int pad, int stride);

/* csrc/bnn_conv.c:80-95: sign bits (w > 0 -> 1) per output channel in kidx
 * order, kidx = (ci*kh + ky)*kw + kx, into ceil(Cin*kh*kw/64) words. */
void pack_weights(const int8_t *wsign, uint64_t *packed, int Cout, int Cin, int kh, int kw);

/* csrc/bnn_conv.c:100-142 (kidx-packed XNOR), 145-213 (channel-packed) and
 * 216-223 (the dispatcher): P = 2 * (equal bits among the in-image taps) -
 * (in-image taps * Cin); activations a > 0 read as +1, the rest as -1.
 * The three give the same P, as in the reference. */
void bconv_xnor(const int8_t *a, const uint64_t *packed_w, int32_t *P, int Cin, int H, int W, int Cout,
                int kh, int kw, int pad, int stride);
void bconv_xnor_packed(const int8_t *a, const uint64_t *packed_w, int32_t *P, int Cin, int H, int W,
                       int Cout, int kh, int kw, int pad, int stride);
void bconv_dispatch(const int8_t *a, const uint64_t *packed_w, int32_t *P, int Cin, int H, int W, int Cout,
                    int kh, int kw, int pad, int stride);

/* csrc/bnn_conv_realin.c:165-172 and the two bodies it picks:
 * out[co] = alpha[co] * sum over in-image taps (ky, kx) of the band sum
 * s = sum_ci wsign * x, each s in band order, the taps in (ky, kx) order
 * (conv_realin_general, :66-116); for kh = kw = 1, pad 0, stride 1 the
 * per-pixel band sum times alpha (conv_realin_1x1, :140-155). */
void conv_realin_naive(const float *x, const int8_t *wsign, const float *alpha, float *out, int Cin, int H,
                       int W, int Cout, int kh, int kw, int pad, int stride);

/* csrc/bnn_maxpool.c:28-48: k x k max over P, floor output size. */
void maxpool_P(const int32_t *P, int32_t *Pout, int C, int H, int W, int k, int stride);

/* csrc/bnn_fold.c:37-60: per-channel rule 0 const (t > 0), 1 P >= t,
 * 2 P < t, 3 lo <= P < hi, 4 P < lo || P >= hi, other codes -1; out +-1. */
void apply_fold_int(const int32_t *P, int8_t *out, int C, int H, int W, const int32_t *type,
                    const int32_t *t, const int32_t *lo, const int32_t *hi);

/* csrc/bnn_fold.c:62-77: z = A*x + B (one fused multiply-add, as the
 * reference's Makefile build contracts it), z < 0 -> slope*z, r = z + rsign,
 * out = r > 0 ? +1 : -1. */
void apply_fold_real(const float *x, int8_t *out, int C, int H, int W, const float *A, const float *B,
                     const float *slope, const float *rsign);

/* csrc/bnn_head.c:21-34: logits[o] = bias[o] + W[o][0]*a[0] + ... in
 * channel order, each product rounded, then added. On the network's +-1
 * input every product is exact and this is the reference's result bit for
 * bit. For arbitrary float input the reference's own builds already differ
 * in the last bits: with -O3 on an FMA machine gcc groups the products by
 * four and fuses the multiply-adds of the Cin % 4 tail. This function keeps
 * the source order without fusing. */
void head_1x1(const float *a, const float *W, const float *bias, float *logits, int Cin, int H, int W_,
              int Cout);

#ifdef __cplusplus
}
#endif
#endif
