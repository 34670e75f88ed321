/* bnn_synth.h - seeded, counter-based synthetic inputs for the binary UNet.
 *
 * Every value is a pure function of (seed, patch index, element index), so a
 * shard of a batch is bit-identical whichever GPU (or CPU) produces it and
 * however the batch is split. Integer-only hashing plus one exact int->float
 * conversion and one correctly rounded float multiply: host C (any compiler,
 * any -march) and CUDA device code produce the same bytes.
 *
 * Distribution: Irwin-Hall sum of four 16-bit uniforms, centred and scaled to
 * unit variance. That is a smooth, bounded (|v| <= 3.46) stand-in for the
 * N(0,1) patches the benchmark configs name; every value carries a full
 * 24-bit mantissa after the scale, so the first conv's fp32 rounding behaves
 * as it would on real spectra.
 *
 * Element index of patch element (band, row, col) in the reference input
 * layout [band][row][col] (csrc/main.c:2-4 of the reference) is
 *     elem = (band * H + row) * W + col.
 */
#ifndef BNN_SYNTH_H
#define BNN_SYNTH_H
#include <stdint.h>

#if defined(__CUDACC__)
#define BNN_SYNTH_FN static __host__ __device__ __forceinline__
#else
#define BNN_SYNTH_FN static inline
#endif

/* 32-bit avalanche mix (xor-shift-multiply finaliser). */
BNN_SYNTH_FN uint32_t bnn_synth_mix32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du;
    x ^= x >> 15; x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

/* 1 / (2 * sqrt((65536^2 - 1) / 3)) rounded to float: maps the centred
 * integer sum (step 2) to unit variance. */
#define BNN_SYNTH_SCALE 0x1.bb67aep-17f

BNN_SYNTH_FN float bnn_synth_value(uint32_t seed, uint32_t patch, uint32_t elem) {
    uint32_t k  = bnn_synth_mix32(bnn_synth_mix32(seed ^ 0x5bd1e995u) ^ patch);
    uint32_t h1 = bnn_synth_mix32(k ^ (elem * 2u + 0x68e31da4u));
    uint32_t h2 = bnn_synth_mix32(k ^ (elem * 2u + 0x1b56c4e9u));
    int32_t s = (int32_t)(h1 & 0xffffu) + (int32_t)(h1 >> 16) +
                (int32_t)(h2 & 0xffffu) + (int32_t)(h2 >> 16);
    int32_t c = 2 * s - 4 * 65535;          /* exact, |c| <= 262140 < 2^24 */
    return (float)c * BNN_SYNTH_SCALE;      /* one RN multiply */
}

#endif
