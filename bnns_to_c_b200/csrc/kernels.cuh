// kernels.cuh - sm_100a CUDA kernels of the binary-UNet forward.
//
// Data layout in HBM (all activations after the first conv are bit planes):
//   act  uint32 [N][H][W][cw], cw = ceil(C/32); channel c -> bit c&31 of word
//        c>>5; 1 = +1, 0 = -1; unused high bits 0.
//   input float32 [N][bands][H][W] (the reference's [band][row][col] per patch)
//   logits float32 [N][classes][H][W]
//   binary weights uint32 [CoutP][9 taps][Kw], tap t = ky*3+kx, same bit
//        convention, Kw = words per tap (for a decoder concat: the skip's
//        words, then the upsampled tensor's words, each segment word-aligned)
//
// Binary conv accumulator (reference csrc/bnn_conv.c:23-28,183-211):
//   P = (#in-bounds taps)*Cin - 2 * (#mismatching bits over in-bounds taps).
// The kernel zero-fills out-of-image halo words and counts mismatches over
// all 9 taps branch-free; an out-of-image tap then contributes exactly
// popc(weight bits of that tap), which the epilogue subtracts again.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/bnn_synth.h"

namespace bnn {

// Per-channel fold in interval form. Every reference rule
// (csrc/bnn_fold.c:37-60) is bit = (lo <= P < hi) XOR inv:
//   const: [-2^30, 2^30) with inv = !(t > 0); ge: [t, 2^30); lt: [-2^30, t);
//   band_in: [lo, hi); band_out: [lo, hi) with inv = 1; unknown: empty.
// |P| <= 9*Cin < 2^30, so the open ends never bind.
struct __align__(16) FoldIv {
    int lo, hi, inv, pad;
};

struct BconvParams {
    const uint32_t* in0;  // [N][H][W][cw0] (the plain input, or the skip)
    const uint32_t* in1;  // concat only: half-res tensor [N][h1][w1][cw1]
    int cw0, cw1, Kw;     // words per pixel of in0, in1; Kw = cw0 + cw1
    int N, H, W;
    int h1, w1, oh, ow, cH, cW;  // upsample placement (reference up_cat)
    int Cin, Cout, cwo;
    const uint32_t* wt;   // [CoutP][9][Kw]
    const int* wpop;      // [CoutP][9]
    const FoldIv* fold;   // [CoutP]
    const FoldIv* fold2;  // pooled-branch fold, or nullptr
    uint32_t* out;        // [N][H][W][cwo]
    uint32_t* out2;       // [N][H/2][W/2][cwo] or nullptr
    int32_t* P;           // debug: [N][Cout][H][W] or nullptr
    int32_t* P2;          // debug: [N][Cout][H/2][W/2] or nullptr
    int TR, TC, TNI;      // tile: rows, cols, whole images per tile
    int tiles_x, tiles_y; // tiles per image (TNI == 1)
    int HP;               // halo pixels = TNI*(TR+2)*(TC+2)
};

template <int KC>
struct KcTraits {
    static constexpr int VW = KC >= 4 ? 4 : KC;                 // words per smem load
    static constexpr int KCP = (KC >= 8 && ((KC / 4) % 2 == 0)) ? KC + 4 : KC;  // pitch
};

template <int BN, int TM, int TN, int KC>
struct BconvCfg {
    static constexpr int NT = 256;
    static constexpr int NG = BN / TN;   // cout groups
    static constexpr int MG = NT / NG;   // slot groups
    static constexpr int BM = MG * TM;   // output pixel slots per tile
    static constexpr int BNP = BN;       // B row pitch
    static constexpr int PSP = BN + 1;   // P tile pitch (ints)
    // words of the A (halo) region, padded so the B region is 16-byte aligned
    __host__ __device__ static size_t a_words(int HP) { return ((size_t)HP * KcTraits<KC>::KCP + 3) & ~(size_t)3; }
    __host__ __device__ static size_t main_words(int HP) {
        size_t a = a_words(HP) + (size_t)9 * KC * BNP;
        size_t ps = ((size_t)BM * PSP + 3) & ~(size_t)3;
        return a > ps ? a : ps;
    }
    static size_t smem_bytes(int HP) {
        return main_words(HP) * 4 + (size_t)BN * 2 * sizeof(FoldIv) + (size_t)BN * 9 * 4;
    }
};

__device__ __forceinline__ int fold_bit(int P, FoldIv f) {
    return ((P >= f.lo) & (P < f.hi)) ^ f.inv;
}

template <int VW>
struct VecW;
template <>
struct VecW<1> {
    __device__ __forceinline__ static void ld(const uint32_t* p, uint32_t* v) { v[0] = p[0]; }
};
template <>
struct VecW<2> {
    __device__ __forceinline__ static void ld(const uint32_t* p, uint32_t* v) {
        uint2 t = *reinterpret_cast<const uint2*>(p);
        v[0] = t.x; v[1] = t.y;
    }
};
template <>
struct VecW<4> {
    __device__ __forceinline__ static void ld(const uint32_t* p, uint32_t* v) {
        uint4 t = *reinterpret_cast<const uint4*>(p);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    }
};

template <int TN>
__device__ __forceinline__ void ld_b(const uint32_t* p, uint32_t* v) {
#pragma unroll
    for (int q = 0; q < TN / 4; ++q) {
        uint4 t = *reinterpret_cast<const uint4*>(p + 4 * q);
        v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
}

// Fused binary 3x3 conv (stride 1, zero pad 1) -> integer fold -> bit pack,
// optionally + 2x2 max-pool of P -> second fold -> bit pack.
// Implicit GEMM: M = output pixels (a tile of BM slots: whole small images,
// or row bands of one image), N = Cout (BN per CTA), K = 9 taps x Kw words.
// The input halo of the tile is staged in shared memory per K chunk, so each
// activation word is read from L2/HBM once per CTA, not once per tap.
template <int BN, int TM, int TN, int KC>
__global__ void __launch_bounds__(256, 2) bconv3x3_kernel(const BconvParams p) {
    using C = BconvCfg<BN, TM, TN, KC>;
    constexpr int NT = C::NT, MG = C::MG, BM = C::BM, BNP = C::BNP, PSP = C::PSP;
    constexpr int VW = KcTraits<KC>::VW, KCP = KcTraits<KC>::KCP;
    extern __shared__ __align__(16) uint32_t smem[];
    const int HP = p.HP;
    uint32_t* As = smem;                                  // [HP][KCP]
    uint32_t* Bs = smem + C::a_words(HP);                 // [9][KC][BNP]
    FoldIv* fs = reinterpret_cast<FoldIv*>(smem + C::main_words(HP));  // [BN]
    FoldIv* fs2 = fs + BN;                                      // [BN]
    int* wps = reinterpret_cast<int*>(fs2 + BN);                // [BN][9]
    int32_t* Ps = reinterpret_cast<int32_t*>(smem);             // [BM][PSP] (after main loop)

    const int tid = threadIdx.x;
    const int mg = tid % MG, ng = tid / MG;
    const int cout0 = blockIdx.y * BN;

    int n0, y0, x0;
    if (p.TNI > 1) {
        n0 = blockIdx.x * p.TNI; y0 = 0; x0 = 0;
    } else {
        const int per = p.tiles_x * p.tiles_y;
        n0 = blockIdx.x / per;
        const int r = blockIdx.x - n0 * per;
        y0 = (r / p.tiles_x) * p.TR;
        x0 = (r % p.tiles_x) * p.TC;
    }
    const int HC = p.TC + 2, HRC = (p.TR + 2) * HC, TRC = p.TR * p.TC;

    for (int c = tid; c < BN; c += NT) {
        fs[c] = p.fold[cout0 + c];
        fs2[c] = p.fold2 ? p.fold2[cout0 + c] : FoldIv{0, 0, 0, 0};
    }
    for (int e = tid; e < BN * 9; e += NT) wps[e] = p.wpop[(size_t)cout0 * 9 + e];

    int hc[TM];
#pragma unroll
    for (int j = 0; j < TM; ++j) {
        const int m = mg + MG * j;
        const int i = m / TRC, rem = m - i * TRC, yy = rem / p.TC, xx = rem - yy * p.TC;
        hc[j] = (i < p.TNI) ? (i * HRC + (yy + 1) * HC + xx + 1) : (HC + 1);
    }

    uint32_t acc[TM][TN];
#pragma unroll
    for (int j = 0; j < TM; ++j)
#pragma unroll
        for (int c = 0; c < TN; ++c) acc[j][c] = 0u;

    for (int kc0 = 0; kc0 < p.Kw; kc0 += KC) {
        __syncthreads();
        // ---- stage the halo chunk: As[hp][k] = word kc0+k of halo pixel hp
        for (int e = tid; e < HP * KC; e += NT) {
            const int hp = e / KC, k = e - hp * KC;
            const int i = hp / HRC, rem = hp - i * HRC, r = rem / HC, cc = rem - r * HC;
            const int n = n0 + i, y = y0 + r - 1, x = x0 + cc - 1, kk = kc0 + k;
            uint32_t v = 0u;
            if (n < p.N && (unsigned)y < (unsigned)p.H && (unsigned)x < (unsigned)p.W && kk < p.Kw) {
                if (kk < p.cw0) {
                    v = __ldg(p.in0 + (((size_t)n * p.H + y) * p.W + x) * p.cw0 + kk);
                } else {
                    const int uy = y - p.oh, ux = x - p.ow;
                    if ((unsigned)uy < (unsigned)p.cH && (unsigned)ux < (unsigned)p.cW)
                        v = __ldg(p.in1 + (((size_t)n * p.h1 + (uy >> 1)) * p.w1 + (ux >> 1)) * p.cw1 +
                                  (kk - p.cw0));
                }
            }
            As[hp * KCP + k] = v;
        }
        // ---- stage the weight chunk: Bs[t][k][c]
        for (int e = tid; e < 9 * KC * BN; e += NT) {
            const int c = e % BN, k = (e / BN) % KC, t = e / (BN * KC);
            const int kk = kc0 + k;
            Bs[(t * KC + k) * BNP + c] =
                kk < p.Kw ? __ldg(p.wt + ((size_t)(cout0 + c) * 9 + t) * p.Kw + kk) : 0u;
        }
        __syncthreads();
        // ---- XOR + POPC over 9 taps x KC words
#pragma unroll 1
        for (int t = 0; t < 9; ++t) {
            const int off = (t / 3 - 1) * HC + (t % 3 - 1);
#pragma unroll
            for (int k4 = 0; k4 < KC / VW; ++k4) {
                uint32_t a[TM][VW];
#pragma unroll
                for (int j = 0; j < TM; ++j) VecW<VW>::ld(As + (hc[j] + off) * KCP + k4 * VW, a[j]);
#pragma unroll
                for (int kk = 0; kk < VW; ++kk) {
                    uint32_t b[TN];
                    ld_b<TN>(Bs + (t * KC + k4 * VW + kk) * BNP + ng * TN, b);
#pragma unroll
                    for (int j = 0; j < TM; ++j)
#pragma unroll
                        for (int c = 0; c < TN; ++c) acc[j][c] += __popc(a[j][kk] ^ b[c]);
                }
            }
        }
    }
    __syncthreads();  // main-loop smem is reused as the P tile

    // ---- P = nv*Cin - 2*(mismatches - out-of-image tap weight bits)
#pragma unroll
    for (int j = 0; j < TM; ++j) {
        const int m = mg + MG * j;
        const int i = m / TRC, rem = m - i * TRC, yy = rem / p.TC, xx = rem - yy * p.TC;
        const int y = y0 + yy, x = x0 + xx;
        const bool ylo = (y == 0), yhi = (y == p.H - 1), xlo = (x == 0), xhi = (x == p.W - 1);
        const int nv = (3 - ylo - yhi) * (3 - xlo - xhi);
        const bool border = ylo | yhi | xlo | xhi;
#pragma unroll
        for (int c = 0; c < TN; ++c) {
            const int cl = ng * TN + c;
            int corr = 0;
            if (border) {
#pragma unroll
                for (int t = 0; t < 9; ++t) {
                    const int dy = t / 3, dx = t % 3;
                    const bool oob = (dy == 0 && ylo) || (dy == 2 && yhi) || (dx == 0 && xlo) || (dx == 2 && xhi);
                    if (oob) corr += wps[cl * 9 + t];
                }
            }
            Ps[m * PSP + cl] = nv * p.Cin - 2 * ((int)acc[j][c] - corr);
        }
    }
    __syncthreads();

    // ---- fold + pack, one output word (32 channels) per item
    constexpr int WPT = BN / 32;
    const int word0 = cout0 >> 5;
    for (int e = tid; e < BM * WPT; e += NT) {
        const int m = e / WPT, w = e - m * WPT;
        const int i = m / TRC, rem = m - i * TRC, yy = rem / p.TC, xx = rem - yy * p.TC;
        const int n = n0 + i, y = y0 + yy, x = x0 + xx;
        // words wholly past Cout (Cout not a multiple of BN) do not exist
        if (i >= p.TNI || n >= p.N || y >= p.H || x >= p.W || cout0 + w * 32 >= p.Cout) continue;
        const int32_t* Pm = Ps + m * PSP + w * 32;
        uint32_t bits = 0u;
#pragma unroll 8
        for (int b = 0; b < 32; ++b) {
            const int c = w * 32 + b;
            if (cout0 + c < p.Cout) bits |= (uint32_t)fold_bit(Pm[b], fs[c]) << b;
        }
        p.out[(((size_t)n * p.H + y) * p.W + x) * p.cwo + word0 + w] = bits;
        if (p.P) {
            for (int b = 0; b < 32 && cout0 + w * 32 + b < p.Cout; ++b)
                p.P[(((size_t)n * p.Cout + cout0 + w * 32 + b) * p.H + y) * p.W + x] = Pm[b];
        }
        if (p.out2 && !(yy & 1) && !(xx & 1) && y + 1 < p.H && x + 1 < p.W) {
            const int Hh = p.H >> 1, Wh = p.W >> 1;
            const int32_t* P01 = Pm + PSP;
            const int32_t* P10 = Pm + p.TC * PSP;
            const int32_t* P11 = P10 + PSP;
            uint32_t bits2 = 0u;
            for (int b = 0; b < 32; ++b) {
                const int c = w * 32 + b;
                if (cout0 + c >= p.Cout) break;
                const int mx = max(max(Pm[b], P01[b]), max(P10[b], P11[b]));
                bits2 |= (uint32_t)fold_bit(mx, fs2[c]) << b;
                if (p.P2)
                    p.P2[(((size_t)n * p.Cout + cout0 + c) * Hh + (y >> 1)) * Wh + (x >> 1)] = mx;
            }
            p.out2[(((size_t)n * Hh + (y >> 1)) * Wh + (x >> 1)) * p.cwo + word0 + w] = bits2;
        }
    }
}

// ---------------------------------------------------------------------
// First conv: real input, +-1 weights, 3x3 pad 1, in the reference's exact
// fp32 operation order (csrc/bnn_conv_realin.c:90-112), fused with the real
// fold (csrc/bnn_fold.c:62-77) and the bit pack.
// Tile: 4 rows x 32 columns of one patch, 4 warps; warp w owns output
// channels 8w..8w+7 of this CTA's 32-channel group, lane l owns the 4
// pixels (row j, column l). The tile's input halo (6 x 34 pixels, all bands)
// sits in shared memory as [pixel][band] so a lane fetches 4 bands with one
// 16-byte load.
// ---------------------------------------------------------------------
struct RealinParams {
    const float* x;      // [N][Cin][H][W]
    const float* wf;     // [CoutP][9][CinP] (+1.0f / -1.0f, zero padded)
    const float* fold;   // [CoutP][5]: alpha, A, B, slope, rsign
    uint32_t* out;       // [N][H][W][cwo]
    float* dbg;          // optional [N][Cout][H][W] conv output (alpha*acc)
    int N, Cin, CinP, CIP, H, W, Cout, cwo;
    int tiles_x, tiles_y;
};

constexpr int RI_TR = 4, RI_TC = 32, RI_HR = RI_TR + 2, RI_HC = RI_TC + 2, RI_HP = RI_HR * RI_HC;

__global__ void __launch_bounds__(128) realin3x3_fold_kernel(const RealinParams p) {
    extern __shared__ __align__(16) float xs[];        // [RI_HP][CIP]
    __shared__ uint32_t words[RI_TR * RI_TC];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = p.tiles_x * p.tiles_y;
    const int n = blockIdx.x / per, r = blockIdx.x - n * per;
    const int y0 = (r / p.tiles_x) * RI_TR, x0 = (r % p.tiles_x) * RI_TC;
    const int co0 = blockIdx.y * 32 + warp * 8;

    words[tid] = 0u;
    // stage the halo, zero outside the image
    const size_t plane = (size_t)p.H * p.W;
    const float* xn = p.x + (size_t)n * p.Cin * plane;
    for (int e = tid; e < RI_HP * p.Cin; e += 128) {
        const int ci = e / RI_HP, hp = e - ci * RI_HP;
        const int hr = hp / RI_HC, hcn = hp - hr * RI_HC;
        const int y = y0 + hr - 1, x = x0 + hcn - 1;
        float v = 0.0f;
        if ((unsigned)y < (unsigned)p.H && (unsigned)x < (unsigned)p.W) v = __ldg(xn + ci * plane + (size_t)y * p.W + x);
        xs[hp * p.CIP + ci] = v;
    }
    __syncthreads();

    float acc[RI_TR][8];
#pragma unroll
    for (int j = 0; j < RI_TR; ++j)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[j][c] = 0.0f;

    if (co0 < p.Cout) {
        const int Cin4 = p.Cin & ~3;
#pragma unroll 1
        for (int t = 0; t < 9; ++t) {
            const int dy = t / 3, dx = t % 3;
            const float* xb = xs + ((dy) * RI_HC + lane + dx) * p.CIP;   // row j adds j*RI_HC*CIP
            const float* wb = p.wf + ((size_t)co0 * 9 + t) * p.CinP;
            float s[RI_TR][8];
#pragma unroll
            for (int j = 0; j < RI_TR; ++j)
#pragma unroll
                for (int c = 0; c < 8; ++c) s[j][c] = 0.0f;
#pragma unroll 2
            for (int ci = 0; ci < Cin4; ci += 4) {
                float4 xv[RI_TR], wv[8];
#pragma unroll
                for (int j = 0; j < RI_TR; ++j)
                    xv[j] = *reinterpret_cast<const float4*>(xb + j * RI_HC * p.CIP + ci);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    wv[c] = __ldg(reinterpret_cast<const float4*>(wb + (size_t)c * 9 * p.CinP + ci));
#pragma unroll
                for (int j = 0; j < RI_TR; ++j)
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        s[j][c] = __fmaf_rn(xv[j].x, wv[c].x, s[j][c]);
                        s[j][c] = __fmaf_rn(xv[j].y, wv[c].y, s[j][c]);
                        s[j][c] = __fmaf_rn(xv[j].z, wv[c].z, s[j][c]);
                        s[j][c] = __fmaf_rn(xv[j].w, wv[c].w, s[j][c]);
                    }
            }
            for (int ci = Cin4; ci < p.Cin; ++ci) {
#pragma unroll
                for (int j = 0; j < RI_TR; ++j) {
                    const float xv = xb[j * RI_HC * p.CIP + ci];
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        s[j][c] = __fmaf_rn(xv, __ldg(wb + (size_t)c * 9 * p.CinP + ci), s[j][c]);
                }
            }
            // out-of-image taps stage zeros: s is exactly +0 there and
            // acc + (+0) == acc, which is the reference skipping the tap.
#pragma unroll
            for (int j = 0; j < RI_TR; ++j)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[j][c] = __fadd_rn(acc[j][c], s[j][c]);
        }
        // fold: z = fma(A, alpha*acc, B); z<0 -> slope*z; r = z + rsign; bit = r > 0
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int co = co0 + c;
            if (co >= p.Cout) break;
            const float* f = p.fold + (size_t)co * 5;
            const float alpha = __ldg(f), A = __ldg(f + 1), B = __ldg(f + 2), sl = __ldg(f + 3), rs = __ldg(f + 4);
#pragma unroll
            for (int j = 0; j < RI_TR; ++j) {
                const float o = __fmul_rn(alpha, acc[j][c]);
                float z = __fmaf_rn(A, o, B);
                if (z < 0.0f) z = __fmul_rn(sl, z);
                const float rr = __fadd_rn(z, rs);
                const int y = y0 + j, x = x0 + lane;
                if (rr > 0.0f) atomicOr(&words[j * RI_TC + lane], 1u << ((warp * 8 + c) & 31));
                if (p.dbg && y < p.H && x < p.W)
                    p.dbg[(((size_t)n * p.Cout + co) * p.H + y) * p.W + x] = o;
            }
        }
    }
    __syncthreads();
    {
        const int j = tid >> 5, y = y0 + j, x = x0 + lane;
        if (y < p.H && x < p.W) p.out[(((size_t)n * p.H + y) * p.W + x) * p.cwo + blockIdx.y] = words[tid];
    }
}

// ---------------------------------------------------------------------
// FP32 1x1 head on the last bit plane: logits = bias + sum_c W*a, sequential
// over c from the bias (csrc/bnn_head.c:21-34, after the int8 -> float widen
// of csrc/bnn_model.c:241-251). a = +-1 makes every product exact.
// ---------------------------------------------------------------------
struct HeadParams {
    const uint32_t* in;  // [N][H][W][cwi]
    const float* Wt;     // [ncls][Cin]
    const float* bias;   // [ncls]
    float* out;          // [N][ncls][H][W]
    int N, H, W, Cin, cwi, ncls;
};

__global__ void head1x1_kernel(const HeadParams p) {
    const size_t HW = (size_t)p.H * p.W;
    const size_t total = (size_t)p.N * HW;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const size_t n = g / HW, px = g - n * HW;
        const uint32_t* a = p.in + g * p.cwi;
        for (int o = 0; o < p.ncls; ++o) {
            float acc = __ldg(p.bias + o);
            const float* w = p.Wt + (size_t)o * p.Cin;
            uint32_t word = 0u;
            for (int c = 0; c < p.Cin; ++c) {
                if ((c & 31) == 0) word = __ldg(a + (c >> 5));
                const float wv = __ldg(w + c);
                acc = __fadd_rn(acc, ((word >> (c & 31)) & 1u) ? wv : -wv);
            }
            p.out[(n * p.ncls + o) * HW + px] = acc;
        }
    }
}

// ---------------------------------------------------------------------
// helpers: synthetic inputs, int8 <-> bit-plane conversion
// ---------------------------------------------------------------------
__global__ void synth_kernel(uint32_t seed, uint32_t first, size_t per, size_t total, float* out) {
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const size_t i = g / per;
        out[g] = bnn_synth_value(seed, first + (uint32_t)i, (uint32_t)(g - i * per));
    }
}

// one thread per output word
__global__ void pack_act_kernel(const int8_t* a, int N, int C, int H, int W, uint32_t* bits) {
    const int cw = (C + 31) >> 5;
    const size_t HW = (size_t)H * W, total = (size_t)N * HW * cw;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const size_t pix = g / cw;
        const int w = (int)(g - pix * cw);
        const size_t n = pix / HW, px = pix - n * HW;
        uint32_t v = 0u;
        for (int b = 0; b < 32; ++b) {
            const int c = w * 32 + b;
            if (c >= C) break;
            if (a[(n * C + c) * HW + px] > 0) v |= 1u << b;
        }
        bits[g] = v;
    }
}

__global__ void unpack_act_kernel(const uint32_t* bits, int N, int C, int H, int W, int8_t* a) {
    const int cw = (C + 31) >> 5;
    const size_t HW = (size_t)H * W, total = (size_t)N * C * HW;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const size_t px = g % HW, nc = g / HW;
        const int c = (int)(nc % C);
        const size_t n = nc / C;
        const uint32_t v = bits[(n * HW + px) * cw + (c >> 5)];
        a[g] = ((v >> (c & 31)) & 1u) ? 1 : -1;
    }
}

}  // namespace bnn
