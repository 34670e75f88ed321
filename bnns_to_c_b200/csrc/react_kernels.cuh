// react_kernels.cuh - device kernels of the v3 ReActNet real-highway engine
// (csrc/bnn_model_react.c and the kernels it calls). The binary convs run on
// the v1 engine's kernels (bnn_bconv_layer_*, P output); these are the float
// parts around them. Every fp32 result is the reference's bit for bit: the
// roundings are those of the reference built with gcc -O3 on x86 with FMA
// (fused multiply-adds exactly where that build contracts), pinned stage by
// stage against it.
//
// Layouts: float maps (the real highway) [N][C][H][W]; tap bits
// [N][H][W][ceil(C/32)] (bit c&31 of word c>>5, 1 = +1), the binary convs'
// input; P int32 [N][C][H][W].
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace bnn {
namespace react {

// ---------------------------------------------------------------------
// 1x1 projection (+ the tap of its input). out[co] = sum over ci in order
// from 0 of x[ci]*W[co][ci]: one fused multiply-add per channel for pixels
// q < nfull of each image, a rounded product then an add past it (the
// register-blocked kernel's scalar pixel tail, csrc/bnn_realin_blk.h:48-88;
// react_proj_1x1, csrc/bnn_react_ops.c:120-133, uses nfull = H*W). The
// input is the plain map x0, or for a decoder the reference's up_cat_f
// (csrc/bnn_model_react.c:263-283) read in place: channels [0, c0) from the
// skip map x0, the rest from the half-resolution x1 at (y-oh)/2, (x-ow)/2
// inside the covered rectangle, 0 outside. With rsign set, slice 0 also
// writes the input's tap bits: x + rsign > 0 (csrc/bnn_react_ops.c:75-86).
// Thread = one pixel x CB output channels (blockIdx.y = channel slice).
// ---------------------------------------------------------------------
struct ProjParams {
    const float* x0;
    const float* x1;
    int c0, c1, h1, w1, oh, ow, cH, cW;
    int N, H, W, Cin, Cout;
    const float* w;      // [slices][Cin][CB], zero past Cout
    int nfull;
    float* out;          // [N][Cout][H][W]
    const float* rsign;  // [Cin] or nullptr
    uint32_t* bits;      // [N][H][W][ceil(Cin/32)]
};

constexpr int PROJ_CB = 16;
constexpr int PROJ_MAX_CIN = 3072;  // weights of one slice in shared memory: Cin x 64 bytes

__device__ __forceinline__ float cat_value(const ProjParams& p, int n, int ci, int y, int x) {
    if (ci < p.c0) return __ldg(p.x0 + (((size_t)n * p.c0 + ci) * p.H + y) * p.W + x);
    const int yy = y - p.oh, xx = x - p.ow;
    if ((unsigned)yy >= (unsigned)p.cH || (unsigned)xx >= (unsigned)p.cW) return 0.0f;
    return __ldg(p.x1 + (((size_t)n * p.c1 + (ci - p.c0)) * p.h1 + (yy >> 1)) * p.w1 + (xx >> 1));
}

__global__ void __launch_bounds__(256) proj_tap_kernel(const ProjParams p) {
    constexpr int CB = PROJ_CB;
    extern __shared__ __align__(16) float sw[];  // [Cin][CB]
    {
        const float4* src = reinterpret_cast<const float4*>(p.w + (size_t)blockIdx.y * p.Cin * CB);
        float4* dst = reinterpret_cast<float4*>(sw);
        for (int i = threadIdx.x; i < p.Cin * CB / 4; i += blockDim.x) dst[i] = __ldg(src + i);
    }
    __syncthreads();
    const int HW = p.H * p.W;
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= (long long)p.N * HW) return;
    const int n = (int)(g / HW), q = (int)(g - (long long)n * HW);
    const int y = q / p.W, x = q - y * p.W;
    float acc[CB];
#pragma unroll
    for (int c = 0; c < CB; ++c) acc[c] = 0.0f;
    const bool tap = p.rsign != nullptr && blockIdx.y == 0;
    const int cw = (p.Cin + 31) >> 5;
    uint32_t word = 0u;
    const bool fused = q < p.nfull;
    for (int ci = 0; ci < p.Cin; ++ci) {
        const float xv = cat_value(p, n, ci, y, x);
        if (tap) {
            word |= (__fadd_rn(xv, __ldg(p.rsign + ci)) > 0.0f ? 1u : 0u) << (ci & 31);
            if ((ci & 31) == 31 || ci == p.Cin - 1) {
                p.bits[(size_t)g * cw + (ci >> 5)] = word;
                word = 0u;
            }
        }
        const float4* wr = reinterpret_cast<const float4*>(sw + ci * CB);
        if (fused) {
#pragma unroll
            for (int c4 = 0; c4 < CB / 4; ++c4) {
                const float4 w4 = wr[c4];
                acc[4 * c4 + 0] = __fmaf_rn(xv, w4.x, acc[4 * c4 + 0]);
                acc[4 * c4 + 1] = __fmaf_rn(xv, w4.y, acc[4 * c4 + 1]);
                acc[4 * c4 + 2] = __fmaf_rn(xv, w4.z, acc[4 * c4 + 2]);
                acc[4 * c4 + 3] = __fmaf_rn(xv, w4.w, acc[4 * c4 + 3]);
            }
        } else {
#pragma unroll
            for (int c4 = 0; c4 < CB / 4; ++c4) {
                const float4 w4 = wr[c4];
                acc[4 * c4 + 0] = __fadd_rn(acc[4 * c4 + 0], __fmul_rn(w4.x, xv));
                acc[4 * c4 + 1] = __fadd_rn(acc[4 * c4 + 1], __fmul_rn(w4.y, xv));
                acc[4 * c4 + 2] = __fadd_rn(acc[4 * c4 + 2], __fmul_rn(w4.z, xv));
                acc[4 * c4 + 3] = __fadd_rn(acc[4 * c4 + 3], __fmul_rn(w4.w, xv));
            }
        }
    }
#pragma unroll
    for (int c = 0; c < CB; ++c) {
        const int co = blockIdx.y * CB + c;
        if (co < p.Cout) p.out[((size_t)n * p.Cout + co) * HW + q] = acc[c];
    }
}

// ---------------------------------------------------------------------
// enc1.conv1: real input, +-1 weights, 3x3 pad 1, register-blocked order
// (csrc/bnn_realin_blk.h:90-150, Cout % 8 == 0): each output's sum runs band
// by band and, inside a band, over the taps row by row (ky, then kx), one
// fused multiply-add per tap (exact products; out-of-image taps read staged
// zeros, and adding a zero product leaves a sum that is never -0 unchanged,
// as skipping the tap does); out = sum * alpha. CTA tile: 16 rows x 32
// columns of one patch x 16 channels; thread: 4 consecutive pixels x 8
// channels; bands staged 8 at a time with their weights in shared memory.
// ---------------------------------------------------------------------
struct Conv3Params {
    const float* x;      // [N][Cin][H][W]
    const float* w;      // [Cout/16][Cin][9][16] (+1 / 0 / -1, zero past Cout)
    const float* alpha;  // [Cout]
    float* out;          // [N][Cout][H][W]
    int N, Cin, H, W, Cout, tiles_x, tiles_y;
};

// row stride 35 (odd): the 4 rows x 8 column groups a warp reads hit 32 banks
constexpr int C3_TR = 16, C3_TC = 32, C3_CK = 8, C3_SR = C3_TR + 2, C3_SC = C3_TC + 2, C3_SCP = 35;

__global__ void __launch_bounds__(256) conv3_blk_kernel(const Conv3Params p) {
    __shared__ __align__(16) float sx[C3_CK][C3_SR][C3_SCP];
    __shared__ __align__(16) float sw[C3_CK][9][16];
    const int tid = threadIdx.x;
    const int per = p.tiles_x * p.tiles_y;
    const int n = blockIdx.x / per, r = blockIdx.x - n * per;
    const int y0 = (r / p.tiles_x) * C3_TR, x0 = (r % p.tiles_x) * C3_TC;
    const int cb = blockIdx.y;
    const int g = tid >> 7, rest = tid & 127;     // channel group (8 channels), row, column group
    const int row = rest >> 3, cg = rest & 7;
    float acc[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[j][c] = 0.0f;
    const size_t plane = (size_t)p.H * p.W;
    const float* xn = p.x + (size_t)n * p.Cin * plane;
    for (int c0 = 0; c0 < p.Cin; c0 += C3_CK) {
        const int nc = min(C3_CK, p.Cin - c0);
        __syncthreads();
        for (int e = tid; e < C3_CK * C3_SR * C3_SC; e += 256) {
            const int ci = e / (C3_SR * C3_SC), rr = e - ci * (C3_SR * C3_SC);
            const int sy = rr / C3_SC, sxx = rr - sy * C3_SC;
            const int yy = y0 + sy - 1, xx = x0 + sxx - 1;
            float v = 0.0f;
            if (ci < nc && (unsigned)yy < (unsigned)p.H && (unsigned)xx < (unsigned)p.W)
                v = __ldg(xn + (size_t)(c0 + ci) * plane + (size_t)yy * p.W + xx);
            sx[ci][sy][sxx] = v;
        }
        for (int e = tid; e < C3_CK * 9 * 16; e += 256) {
            const int ci = e / 144, rr = e - ci * 144;
            sw[ci][rr / 16][rr % 16] =
                ci < nc ? __ldg(p.w + (((size_t)cb * p.Cin + c0 + ci) * 9) * 16 + rr) : 0.0f;
        }
        __syncthreads();
        for (int ci = 0; ci < nc; ++ci)
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
                float xr[6];
#pragma unroll
                for (int k = 0; k < 6; ++k) xr[k] = sx[ci][row + ky][4 * cg + k];
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const float4 wa = *reinterpret_cast<const float4*>(&sw[ci][ky * 3 + kx][8 * g]);
                    const float4 wb = *reinterpret_cast<const float4*>(&sw[ci][ky * 3 + kx][8 * g + 4]);
                    const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
#pragma unroll
                        for (int c = 0; c < 8; ++c) acc[j][c] = __fmaf_rn(xr[j + kx], w8[c], acc[j][c]);
                }
            }
    }
    const int y = y0 + row;
    if (y >= p.H) return;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const int co = cb * 16 + 8 * g + c;
        if (co >= p.Cout) break;
        const float a = __ldg(p.alpha + co);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int x = x0 + 4 * cg + j;
            if (x < p.W) p.out[((size_t)n * p.Cout + co) * plane + (size_t)y * p.W + x] = __fmul_rn(acc[j][c], a);
        }
    }
}

// The same conv in the order of conv_realin_naive (csrc/bnn_conv_realin.c:
// 66-116, used when Cout % 8 != 0): per tap (ky, kx) the bands are summed in
// order from 0, then the taps' sums are added in tap order; out = alpha*sum.
// Thread = one pixel x 4 channels, nine tap sums in registers.
__global__ void __launch_bounds__(128) conv3_naive_kernel(const Conv3Params p) {
    const size_t plane = (size_t)p.H * p.W;
    const int ng = (p.Cout + 3) / 4;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)p.N * plane * ng) return;
    const int grp = (int)(t % ng);
    const long long pix = t / ng;
    const int n = (int)(pix / plane), q = (int)(pix - (long long)n * plane);
    const int y = q / p.W, x = q - y * p.W;
    float s[9][4];
#pragma unroll
    for (int k = 0; k < 9; ++k)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[k][c] = 0.0f;
    const float* xn = p.x + (size_t)n * p.Cin * plane;
    const int cbk = (grp * 4) / 16, off = (grp * 4) % 16;
    for (int ci = 0; ci < p.Cin; ++ci) {
#pragma unroll
        for (int k = 0; k < 9; ++k) {
            const int yy = y + k / 3 - 1, xx = x + k % 3 - 1;
            const float v =
                ((unsigned)yy < (unsigned)p.H && (unsigned)xx < (unsigned)p.W) ? __ldg(xn + ci * plane + yy * p.W + xx) : 0.0f;
            const float* wr = p.w + (((size_t)cbk * p.Cin + ci) * 9 + k) * 16 + off;
#pragma unroll
            for (int c = 0; c < 4; ++c) s[k][c] = __fmaf_rn(v, __ldg(wr + c), s[k][c]);
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int co = grp * 4 + c;
        if (co >= p.Cout) break;
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 9; ++k) acc = __fadd_rn(acc, s[k][c]);
        p.out[((size_t)n * p.Cout + co) * plane + q] = __fmul_rn(__ldg(p.alpha + co), acc);
    }
}

// ---------------------------------------------------------------------
// Epilogue (csrc/bnn_react_epi.c:34-37 and 56-59, the scalar path x86
// runs): t = fma(A, v, B + move1) + res, out = t >= 0 ? t : prelu_w * t,
// with v = (float)P (binary conv) or the real conv output; B + move1 is
// added once per channel on the host, in fp32, as the reference does.
// With rsign set the output's tap bits are written too (the next conv's
// input). Thread = one pixel, all channels.
// ---------------------------------------------------------------------
struct EpiParams {
    const int32_t* P;    // [N][C][HW] or nullptr
    const float* v;      // [N][C][HW] when P is nullptr
    const float* res;    // [N][C][HW]
    float* out;          // [N][C][HW]
    const float* A;
    const float* Bm;
    const float* pw;
    const float* rsign;  // [C] or nullptr
    uint32_t* bits;      // [N][HW][ceil(C/32)]
    int N, C, HW;
};

__device__ __forceinline__ float rprelu(float A, float v, float Bm, float r, float pw) {
    const float t = __fadd_rn(__fmaf_rn(A, v, Bm), r);
    return t >= 0.0f ? t : __fmul_rn(pw, t);
}

__global__ void __launch_bounds__(256) epi_kernel(const EpiParams p) {
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= (long long)p.N * p.HW) return;
    const int n = (int)(g / p.HW), q = (int)(g - (long long)n * p.HW);
    const int cw = (p.C + 31) >> 5;
    uint32_t word = 0u;
    for (int c = 0; c < p.C; ++c) {
        const size_t i = ((size_t)n * p.C + c) * p.HW + q;
        const float v = p.P ? (float)__ldg(p.P + i) : __ldg(p.v + i);
        const float o = rprelu(__ldg(p.A + c), v, __ldg(p.Bm + c), __ldg(p.res + i), __ldg(p.pw + c));
        p.out[i] = o;
        if (p.rsign) {
            word |= (__fadd_rn(o, __ldg(p.rsign + c)) > 0.0f ? 1u : 0u) << (c & 31);
            if ((c & 31) == 31 || c == p.C - 1) {
                p.bits[(size_t)g * cw + (c >> 5)] = word;
                word = 0u;
            }
        }
    }
}

// Pooled branch of a DownBlock (csrc/bnn_model_react.c:245-258): Pd = 2x2
// max of P, hd = 2x2 max of h1 (compare chains of csrc/bnn_react_opt.c:
// 46-85: first element, then each strictly greater one), down = epilogue(Pd,
// hd). Floor dims. Thread = one half-resolution pixel, all channels.
struct PoolEpiParams {
    const int32_t* P;    // [N][C][H][W]
    const float* h1;     // [N][C][H][W]
    float* out;          // [N][C][H/2][W/2]
    const float* A;
    const float* Bm;
    const float* pw;
    int N, C, H, W;
};

__global__ void __launch_bounds__(256) pool_epi_kernel(const PoolEpiParams p) {
    const int Ho = p.H / 2, Wo = p.W / 2;
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= (long long)p.N * Ho * Wo) return;
    const int HWo = Ho * Wo;
    const int n = (int)(g / HWo), q = (int)(g - (long long)n * HWo);
    const int oy = q / Wo, ox = q - oy * Wo;
    for (int c = 0; c < p.C; ++c) {
        const size_t b = (((size_t)n * p.C + c) * p.H + 2 * oy) * p.W + 2 * ox;
        int32_t m = __ldg(p.P + b), v1 = __ldg(p.P + b + 1), v2 = __ldg(p.P + b + p.W), v3 = __ldg(p.P + b + p.W + 1);
        if (v1 > m) m = v1;
        if (v2 > m) m = v2;
        if (v3 > m) m = v3;
        float f = __ldg(p.h1 + b), f1 = __ldg(p.h1 + b + 1), f2 = __ldg(p.h1 + b + p.W), f3 = __ldg(p.h1 + b + p.W + 1);
        if (f1 > f) f = f1;
        if (f2 > f) f = f2;
        if (f3 > f) f = f3;
        p.out[((size_t)n * p.C + c) * HWo + q] =
            rprelu(__ldg(p.A + c), (float)m, __ldg(p.Bm + c), f, __ldg(p.pw + c));
    }
}

// fp32 1x1 head (head_1x1_v2, csrc/bnn_react_opt.c:26-43): each logit starts
// at the bias and takes one fused multiply-add per input channel, in order.
constexpr int HEADR_MAXC = 16;
struct HeadParams {
    const float* a;      // [N][Cin][HW]
    const float* W;      // [Cout][Cin]
    const float* bias;
    float* out;          // [N][Cout][HW]
    int N, Cin, Cout, HW;
};

__global__ void __launch_bounds__(256) head_kernel(const HeadParams p) {
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= (long long)p.N * p.HW) return;
    const int n = (int)(g / p.HW), q = (int)(g - (long long)n * p.HW);
    float v[HEADR_MAXC];
#pragma unroll
    for (int o = 0; o < HEADR_MAXC; ++o) v[o] = o < p.Cout ? __ldg(p.bias + o) : 0.0f;
    for (int c = 0; c < p.Cin; ++c) {
        const float a = __ldg(p.a + ((size_t)n * p.Cin + c) * p.HW + q);
#pragma unroll
        for (int o = 0; o < HEADR_MAXC; ++o)
            if (o < p.Cout) v[o] = __fmaf_rn(__ldg(p.W + o * p.Cin + c), a, v[o]);
    }
#pragma unroll
    for (int o = 0; o < HEADR_MAXC; ++o)
        if (o < p.Cout) p.out[((size_t)n * p.Cout + o) * p.HW + q] = v[o];
}

// bit plane [N][HW][cw] -> int8 +-1 [N][C][HW] (stage dumps)
__global__ void unpack_bits_kernel(const uint32_t* bits, int N, int C, int HW, int8_t* out) {
    const int cw = (C + 31) >> 5;
    const long long total = (long long)N * C * HW;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int q = (int)(i % HW);
        const long long nc = i / HW;
        const int c = (int)(nc % C);
        const long long n = nc / C;
        out[i] = ((bits[((size_t)n * HW + q) * cw + (c >> 5)] >> (c & 31)) & 1u) ? 1 : -1;
    }
}

}  // namespace react
}  // namespace bnn
