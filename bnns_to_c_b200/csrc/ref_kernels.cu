// ref_kernels.cu - lib/libbnn_kernels.so: the reference's kernel-level C ABI
// (include/bnn_kernels.h; csrc/bnn_model.h:7-23 and csrc/bnn_conv.c of the
// reference) on the current CUDA device, under the reference's own names.
//
// Shapes the forward uses go to its tcgen05 kernels through the
// libbnn_b200.so twins (bnn_gpu_bconv_dispatch for 3x3 stride-1 pad-0/1
// binary convs, bnn_gpu_conv_realin for the 3x3 pad-1 stride-1 real-input
// conv). Every other shape runs on the direct kernels below: one thread per
// output element, the reference's loop order inside it, so the integer
// results are the reference's and the float ones round as its source
// orders them. These calls are synchronous and host-pointer like the
// reference's. A failure prints "<function>: <reason>" and exits 1, as the
// reference does on its own failures.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../include/bnn_b200.h"
#include "../../include/bnn_kernels.h"

#define KAPI extern "C" __attribute__((visibility("default")))

namespace {

constexpr int kThreads = 256;

// the in-image tap range [k0, k1) of output coordinate o along one axis and
// its first input coordinate b (csrc/bnn_conv.c:187-191)
struct TapRange {
    int b, k0, k1;
};
__host__ __device__ inline TapRange tap_range(int o, int stride, int pad, int k, int n) {
    TapRange t;
    t.b = o * stride - pad;
    t.k0 = t.b < 0 ? -t.b : 0;
    t.k1 = t.b + k > n ? n - t.b : k;
    return t;
}

// a [Cin][H][W] int8 -> ap [H*W][Wc] words, bit ci%64 of word ci/64 = a > 0;
// thread i = (wc, pixel), pixel fastest (coalesced reads of a)
__global__ void pack_act_kernel(const int8_t* __restrict__ a, uint64_t* __restrict__ ap, int Cin, long HW, int Wc) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= HW * Wc) return;
    const int wc = (int)(i / HW);
    const long px = i - (long)wc * HW;
    const int c0 = wc * 64, n = min(64, Cin - c0);
    uint64_t v = 0;
    for (int b = 0; b < n; ++b) v |= (uint64_t)(a[(long)(c0 + b) * HW + px] > 0) << b;
    ap[px * Wc + wc] = v;
}

// kidx-packed weights [Cout][nwords] (kidx = (ci*kh + ky)*kw + kx) ->
// per-tap channel words wp [Cout][kh*kw][Wc]
__global__ void repack_w_kernel(const uint64_t* __restrict__ pw, uint64_t* __restrict__ wp, int Cout, int Cin,
                                int kh, int kw, int nwords, int Wc) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int taps = kh * kw;
    if (i >= (long)Cout * taps * Wc) return;
    const int wc = (int)(i % Wc), tap = (int)((i / Wc) % taps), co = (int)(i / ((long)Wc * taps));
    const int ky = tap / kw, kx = tap - ky * kw;
    const uint64_t* src = pw + (long)co * nwords;
    const int c0 = wc * 64, n = min(64, Cin - c0);
    uint64_t v = 0;
    for (int b = 0; b < n; ++b) {
        const long kidx = ((long)(c0 + b) * kh + ky) * kw + kx;
        v |= ((src[kidx >> 6] >> (kidx & 63)) & 1ull) << b;
    }
    wp[i] = v;
}

// XNOR-popcount conv on channel words, one thread per output (co, oy, ox).
// P = 2*equal - valid. raw_valid: valid = (ky1-ky0)*(kx1-kx0)*Cin as
// bconv_xnor_packed counts it (csrc/bnn_conv.c:192); otherwise the taps
// actually visited, as bconv_xnor's mask counts them (csrc/bnn_conv.c:127-129).
// The two differ only where pad > k leaves an output with no tap at all.
__global__ void bconv_popc_kernel(const uint64_t* __restrict__ ap, const uint64_t* __restrict__ wp,
                                  int32_t* __restrict__ P, int Cin, int H, int W, int Cout, int kh, int kw,
                                  int pad, int stride, int Ho, int Wo, int Wc, uint64_t tail, int raw_valid) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)Cout * Ho * Wo) return;
    const int ox = (int)(i % Wo), oy = (int)((i / Wo) % Ho), co = (int)(i / ((long)Wo * Ho));
    const TapRange ty = tap_range(oy, stride, pad, kh, H), tx = tap_range(ox, stride, pad, kw, W);
    int equal = 0, visited = 0;
    for (int ky = ty.k0; ky < ty.k1; ++ky) {
        for (int kx = tx.k0; kx < tx.k1; ++kx) {
            const uint64_t* av = ap + ((long)(ty.b + ky) * W + (tx.b + kx)) * Wc;
            const uint64_t* wv = wp + (((long)co * kh + ky) * kw + kx) * Wc;
            for (int wc = 0; wc < Wc; ++wc)
                equal += __popcll(~(av[wc] ^ wv[wc]) & (wc == Wc - 1 ? tail : ~0ull));
            visited += Cin;
        }
    }
    const int valid = raw_valid ? (ty.k1 - ty.k0) * (tx.k1 - tx.k0) * Cin : visited;
    P[i] = 2 * equal - valid;
}

// bconv_naive_int (csrc/bnn_conv.c:50-76): int8 products over in-image taps,
// in (ci, ky, kx) order
__global__ void bconv_naive_kernel(const int8_t* __restrict__ a, const int8_t* __restrict__ ws,
                                   int32_t* __restrict__ P, int Cin, int H, int W, int Cout, int kh, int kw,
                                   int pad, int stride, int Ho, int Wo) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)Cout * Ho * Wo) return;
    const int ox = (int)(i % Wo), oy = (int)((i / Wo) % Ho), co = (int)(i / ((long)Wo * Ho));
    const TapRange ty = tap_range(oy, stride, pad, kh, H), tx = tap_range(ox, stride, pad, kw, W);
    int acc = 0;
    for (int ci = 0; ci < Cin; ++ci)
        for (int ky = ty.k0; ky < ty.k1; ++ky)
            for (int kx = tx.k0; kx < tx.k1; ++kx)
                acc += (int)ws[(((long)co * Cin + ci) * kh + ky) * kw + kx] *
                       (int)a[((long)ci * H + ty.b + ky) * W + tx.b + kx];
    P[i] = acc;
}

// conv_realin_general (csrc/bnn_conv_realin.c:66-116): per output, over the
// in-image taps in (ky, kx) order, s = the band sum of wsign*x (each product
// rounded, then added), acc += s, out = alpha*acc. The intrinsics keep the
// compiler from fusing any multiply into an add.
__global__ void realin_general_kernel(const float* __restrict__ x, const int8_t* __restrict__ ws,
                                      const float* __restrict__ alpha, float* __restrict__ out, int Cin, int H,
                                      int W, int Cout, int kh, int kw, int pad, int stride, int Ho, int Wo) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)Cout * Ho * Wo) return;
    const int ox = (int)(i % Wo), oy = (int)((i / Wo) % Ho), co = (int)(i / ((long)Wo * Ho));
    const TapRange ty = tap_range(oy, stride, pad, kh, H), tx = tap_range(ox, stride, pad, kw, W);
    const long HW = (long)H * W;
    float acc = 0.0f;
    for (int ky = ty.k0; ky < ty.k1; ++ky) {
        for (int kx = tx.k0; kx < tx.k1; ++kx) {
            const float* xv = x + (long)(ty.b + ky) * W + (tx.b + kx);
            const int8_t* wv = ws + ((long)co * Cin * kh + ky) * kw + kx;
            float s = 0.0f;
            for (int ci = 0; ci < Cin; ++ci)
                s = __fadd_rn(s, __fmul_rn(xv[ci * HW], (float)wv[(long)ci * kh * kw]));
            acc = __fadd_rn(acc, s);
        }
    }
    out[i] = __fmul_rn(alpha[co], acc);
}

// conv_realin_1x1 (csrc/bnn_conv_realin.c:140-155): out = (band sum of
// wsign*x from 0.0f) * alpha, one thread per (co, pixel)
__global__ void realin_1x1_kernel(const float* __restrict__ x, const int8_t* __restrict__ ws,
                                  const float* __restrict__ alpha, float* __restrict__ out, int Cin, long HW,
                                  int Cout) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)Cout * HW) return;
    const int co = (int)(i / HW);
    const long px = i - (long)co * HW;
    const int8_t* wr = ws + (long)co * Cin;
    float o = 0.0f;
    for (int ci = 0; ci < Cin; ++ci) o = __fadd_rn(o, __fmul_rn((float)wr[ci], x[(long)ci * HW + px]));
    out[i] = __fmul_rn(o, alpha[co]);
}

// maxpool_P (csrc/bnn_maxpool.c:28-48)
__global__ void maxpool_kernel(const int32_t* __restrict__ P, int32_t* __restrict__ Po, int C, int H, int W, int k,
                               int stride, int Ho, int Wo) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)C * Ho * Wo) return;
    const int ox = (int)(i % Wo), oy = (int)((i / Wo) % Ho), c = (int)(i / ((long)Wo * Ho));
    int32_t m = INT32_MIN;
    for (int dy = 0; dy < k; ++dy)
        for (int dx = 0; dx < k; ++dx) m = max(m, P[((long)c * H + oy * stride + dy) * W + ox * stride + dx]);
    Po[i] = m;
}

// apply_fold_int (csrc/bnn_fold.c:37-60)
__global__ void fold_int_kernel(const int32_t* __restrict__ P, int8_t* __restrict__ out, int C, long HW,
                                const int32_t* __restrict__ type, const int32_t* __restrict__ t,
                                const int32_t* __restrict__ lo, const int32_t* __restrict__ hi) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)C * HW) return;
    const int c = (int)(i / HW), v = P[i];
    bool b;
    switch (type[c]) {
        case 0: b = t[c] > 0; break;
        case 1: b = v >= t[c]; break;
        case 2: b = v < t[c]; break;
        case 3: b = v >= lo[c] && v < hi[c]; break;
        case 4: b = v < lo[c] || v >= hi[c]; break;
        default: b = false; break;
    }
    out[i] = b ? 1 : -1;
}

// apply_fold_real (csrc/bnn_fold.c:62-77), A*x + B fused as the reference's
// Makefile build fuses it
__global__ void fold_real_kernel(const float* __restrict__ x, int8_t* __restrict__ out, int C, long HW,
                                 const float* __restrict__ A, const float* __restrict__ B,
                                 const float* __restrict__ slope, const float* __restrict__ rsign) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)C * HW) return;
    const int c = (int)(i / HW);
    float z = __fmaf_rn(A[c], x[i], B[c]);
    if (z < 0.0f) z = __fmul_rn(slope[c], z);
    out[i] = __fadd_rn(z, rsign[c]) > 0.0f ? 1 : -1;
}

// head_1x1 (csrc/bnn_head.c:21-34): bias, then each channel's rounded
// product added in channel order
__global__ void head_kernel(const float* __restrict__ a, const float* __restrict__ Wt, const float* __restrict__ bias,
                            float* __restrict__ logits, int Cin, long HW, int Cout) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)Cout * HW) return;
    const int o = (int)(i / HW);
    const long px = i - (long)o * HW;
    const float* wr = Wt + (long)o * Cin;
    float acc = bias[o];
    for (int c = 0; c < Cin; ++c) acc = __fadd_rn(acc, __fmul_rn(wr[c], a[(long)c * HW + px]));
    logits[i] = acc;
}

[[noreturn]] void die(const char* fn, const char* what) {
    fprintf(stderr, "%s: %s\n", fn, what);
    exit(1);
}

int out_dim(int in, int k, int pad, int stride) { return (in + 2 * pad - k) / stride + 1; }

// shape checks every function shares: the reference takes any shape whose
// loops are defined; these are the ones whose loops are not
void check_conv(const char* fn, int Cin, int H, int W, int Cout, int kh, int kw, int pad, int stride) {
    if (Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0 || kh <= 0 || kw <= 0 || pad < 0 || stride <= 0)
        die(fn, "bad shape (Cin, H, W, Cout, kh, kw, stride must be > 0, pad >= 0)");
}

unsigned grid_for(long n) { return (unsigned)((n + kThreads - 1) / kThreads); }

// device buffers of one call, released on return
struct Scratch {
    const char* fn;
    void* p[8] = {};
    int n = 0;
    explicit Scratch(const char* f) : fn(f) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            die(fn, "no CUDA device available");
        }
    }
    ~Scratch() {
        for (int i = 0; i < n; ++i) cudaFree(p[i]);
    }
    template <class T>
    T* alloc(size_t count) {
        if (n == (int)(sizeof p / sizeof p[0])) die(fn, "internal: more device buffers than one call holds");
        void* q = nullptr;
        if (cudaMalloc(&q, count ? count * sizeof(T) : 1) != cudaSuccess) {
            cudaGetLastError();
            die(fn, "out of device memory");
        }
        p[n++] = q;
        return static_cast<T*>(q);
    }
    template <class T>
    T* upload(const T* host, size_t count) {
        T* d = alloc<T>(count);
        if (count && cudaMemcpy(d, host, count * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess) die(fn, "H2D copy");
        return d;
    }
    template <class T>
    void download(T* host, const T* d, size_t count) {
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) die(fn, cudaGetErrorString(e));
        if (count && cudaMemcpy(host, d, count * sizeof(T), cudaMemcpyDeviceToHost) != cudaSuccess) die(fn, "D2H copy");
    }
};

// the three XNOR kernels: the forward's tcgen05 path where its shape fits,
// the channel-word kernel otherwise. raw_valid as in bconv_popc_kernel.
void bconv_packed_run(const char* fn, const int8_t* a, const uint64_t* packed_w, int32_t* P, int Cin, int H, int W,
                      int Cout, int kh, int kw, int pad, int stride, int raw_valid) {
    check_conv(fn, Cin, H, W, Cout, kh, kw, pad, stride);
    if (!a || !packed_w || !P) die(fn, "NULL argument");
    const int Ho = out_dim(H, kh, pad, stride), Wo = out_dim(W, kw, pad, stride);
    if (Ho <= 0 || Wo <= 0) return;
    if (kh == 3 && kw == 3 && stride == 1 && (pad == 0 || pad == 1)) {
        if (bnn_gpu_bconv_dispatch(a, packed_w, P, Cin, H, W, Cout, kh, kw, pad, stride) != BNN_OK)
            die(fn, bnn_last_error());
        return;
    }
    Scratch s(fn);
    const long HW = (long)H * W;
    const int Wc = (Cin + 63) / 64, taps = kh * kw;
    const long K = (long)Cin * taps;
    const int nwords = (int)((K + 63) / 64);
    const uint64_t tail = (Cin & 63) ? ((1ull << (Cin & 63)) - 1) : ~0ull;
    const int8_t* da = s.upload(a, (size_t)Cin * HW);
    const uint64_t* dpw = s.upload(packed_w, (size_t)Cout * nwords);
    uint64_t* dap = s.alloc<uint64_t>((size_t)HW * Wc);
    uint64_t* dwp = s.alloc<uint64_t>((size_t)Cout * taps * Wc);
    int32_t* dP = s.alloc<int32_t>((size_t)Cout * Ho * Wo);
    pack_act_kernel<<<grid_for(HW * Wc), kThreads>>>(da, dap, Cin, HW, Wc);
    repack_w_kernel<<<grid_for((long)Cout * taps * Wc), kThreads>>>(dpw, dwp, Cout, Cin, kh, kw, nwords, Wc);
    bconv_popc_kernel<<<grid_for((long)Cout * Ho * Wo), kThreads>>>(dap, dwp, dP, Cin, H, W, Cout, kh, kw, pad,
                                                                    stride, Ho, Wo, Wc, tail, raw_valid);
    s.download(P, dP, (size_t)Cout * Ho * Wo);
}

}  // namespace

KAPI void bconv_naive_int(const int8_t* a, const int8_t* wsign, int32_t* P, int Cin, int H, int W, int Cout, int kh,
                          int kw, int pad, int stride) {
    const char* fn = "bconv_naive_int";
    check_conv(fn, Cin, H, W, Cout, kh, kw, pad, stride);
    if (!a || !wsign || !P) die(fn, "NULL argument");
    const int Ho = out_dim(H, kh, pad, stride), Wo = out_dim(W, kw, pad, stride);
    if (Ho <= 0 || Wo <= 0) return;
    Scratch s(fn);
    const int8_t* da = s.upload(a, (size_t)Cin * H * W);
    const int8_t* dw = s.upload(wsign, (size_t)Cout * Cin * kh * kw);
    int32_t* dP = s.alloc<int32_t>((size_t)Cout * Ho * Wo);
    bconv_naive_kernel<<<grid_for((long)Cout * Ho * Wo), kThreads>>>(da, dw, dP, Cin, H, W, Cout, kh, kw, pad, stride,
                                                                     Ho, Wo);
    s.download(P, dP, (size_t)Cout * Ho * Wo);
}

// a host-side weight format conversion in the reference as well
// (csrc/bnn_conv.c:80-95): sign bits in kidx order
KAPI void pack_weights(const int8_t* wsign, uint64_t* packed, int Cout, int Cin, int kh, int kw) {
    const long K = (long)Cin * kh * kw, nwords = (K + 63) / 64;
    memset(packed, 0, (size_t)Cout * nwords * sizeof(uint64_t));
    for (long co = 0; co < Cout; ++co)
        for (long k = 0; k < K; ++k)  // wsign's [ci][ky][kx] order is the kidx order
            if (wsign[co * K + k] > 0) packed[co * nwords + (k >> 6)] |= 1ull << (k & 63);
}

// bconv_xnor counts the taps it visits (its bit mask); bconv_xnor_packed the
// clipped range product; bconv_dispatch picks between them on Cin >= 36
// (csrc/bnn_conv.c:48,216-223)
KAPI void bconv_xnor(const int8_t* a, const uint64_t* packed_w, int32_t* P, int Cin, int H, int W, int Cout, int kh,
                     int kw, int pad, int stride) {
    bconv_packed_run("bconv_xnor", a, packed_w, P, Cin, H, W, Cout, kh, kw, pad, stride, 0);
}

KAPI void bconv_xnor_packed(const int8_t* a, const uint64_t* packed_w, int32_t* P, int Cin, int H, int W, int Cout,
                            int kh, int kw, int pad, int stride) {
    bconv_packed_run("bconv_xnor_packed", a, packed_w, P, Cin, H, W, Cout, kh, kw, pad, stride, 1);
}

KAPI void bconv_dispatch(const int8_t* a, const uint64_t* packed_w, int32_t* P, int Cin, int H, int W, int Cout,
                         int kh, int kw, int pad, int stride) {
    bconv_packed_run("bconv_dispatch", a, packed_w, P, Cin, H, W, Cout, kh, kw, pad, stride, Cin >= 36 ? 1 : 0);
}

// conv_realin_naive's dispatch (csrc/bnn_conv_realin.c:165-172): 1x1 pad 0
// stride 1 -> conv_realin_1x1's order, everything else -> conv_realin_general's;
// the 3x3 pad-1 stride-1 shape of the forward (Cin <= 256) runs on its
// tcgen05 kernel, which keeps conv_realin_general's order
KAPI void conv_realin_naive(const float* x, const int8_t* wsign, const float* alpha, float* out, int Cin, int H, int W,
                            int Cout, int kh, int kw, int pad, int stride) {
    const char* fn = "conv_realin_naive";
    check_conv(fn, Cin, H, W, Cout, kh, kw, pad, stride);
    if (!x || !wsign || !alpha || !out) die(fn, "NULL argument");
    const int Ho = out_dim(H, kh, pad, stride), Wo = out_dim(W, kw, pad, stride);
    if (Ho <= 0 || Wo <= 0) return;
    if (kh == 3 && kw == 3 && pad == 1 && stride == 1 && Cin <= 256) {
        if (bnn_gpu_conv_realin(x, wsign, alpha, out, Cin, H, W, Cout, kh, kw, pad, stride) != BNN_OK)
            die(fn, bnn_last_error());
        return;
    }
    Scratch s(fn);
    const long HW = (long)H * W;
    const float* dx = s.upload(x, (size_t)Cin * HW);
    const int8_t* dw = s.upload(wsign, (size_t)Cout * Cin * kh * kw);
    const float* da = s.upload(alpha, (size_t)Cout);
    const long n = (long)Cout * Ho * Wo;
    float* dout = s.alloc<float>((size_t)n);
    if (kh == 1 && kw == 1 && pad == 0 && stride == 1)
        realin_1x1_kernel<<<grid_for(n), kThreads>>>(dx, dw, da, dout, Cin, HW, Cout);
    else
        realin_general_kernel<<<grid_for(n), kThreads>>>(dx, dw, da, dout, Cin, H, W, Cout, kh, kw, pad, stride, Ho,
                                                         Wo);
    s.download(out, dout, (size_t)n);
}

KAPI void maxpool_P(const int32_t* P, int32_t* Pout, int C, int H, int W, int k, int stride) {
    const char* fn = "maxpool_P";
    if (C <= 0 || H <= 0 || W <= 0 || k <= 0 || stride <= 0) die(fn, "bad shape");
    // below k the reference's window reads past P (bnn_maxpool.c:29-30 floors
    // toward zero, so H - k < 0 still gives one output row)
    if (H < k || W < k) die(fn, "H or W below the window: the reference reads past P there");
    if (!P || !Pout) die(fn, "NULL argument");
    const int Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
    Scratch s(fn);
    const int32_t* dP = s.upload(P, (size_t)C * H * W);
    const long n = (long)C * Ho * Wo;
    int32_t* dO = s.alloc<int32_t>((size_t)n);
    maxpool_kernel<<<grid_for(n), kThreads>>>(dP, dO, C, H, W, k, stride, Ho, Wo);
    s.download(Pout, dO, (size_t)n);
}

KAPI void apply_fold_int(const int32_t* P, int8_t* out, int C, int H, int W, const int32_t* type, const int32_t* t,
                         const int32_t* lo, const int32_t* hi) {
    const char* fn = "apply_fold_int";
    if (C <= 0 || H <= 0 || W <= 0) die(fn, "bad shape");
    if (!P || !out || !type || !t || !lo || !hi) die(fn, "NULL argument");
    Scratch s(fn);
    const long HW = (long)H * W, n = (long)C * HW;
    const int32_t* dP = s.upload(P, (size_t)n);
    const int32_t* dty = s.upload(type, (size_t)C);
    const int32_t* dt = s.upload(t, (size_t)C);
    const int32_t* dlo = s.upload(lo, (size_t)C);
    const int32_t* dhi = s.upload(hi, (size_t)C);
    int8_t* dO = s.alloc<int8_t>((size_t)n);
    fold_int_kernel<<<grid_for(n), kThreads>>>(dP, dO, C, HW, dty, dt, dlo, dhi);
    s.download(out, dO, (size_t)n);
}

KAPI void apply_fold_real(const float* x, int8_t* out, int C, int H, int W, const float* A, const float* B,
                          const float* slope, const float* rsign) {
    const char* fn = "apply_fold_real";
    if (C <= 0 || H <= 0 || W <= 0) die(fn, "bad shape");
    if (!x || !out || !A || !B || !slope || !rsign) die(fn, "NULL argument");
    Scratch s(fn);
    const long HW = (long)H * W, n = (long)C * HW;
    const float* dx = s.upload(x, (size_t)n);
    const float* dA = s.upload(A, (size_t)C);
    const float* dB = s.upload(B, (size_t)C);
    const float* ds = s.upload(slope, (size_t)C);
    const float* dr = s.upload(rsign, (size_t)C);
    int8_t* dO = s.alloc<int8_t>((size_t)n);
    fold_real_kernel<<<grid_for(n), kThreads>>>(dx, dO, C, HW, dA, dB, ds, dr);
    s.download(out, dO, (size_t)n);
}

KAPI void head_1x1(const float* a, const float* Wt, const float* bias, float* logits, int Cin, int H, int W_,
                   int Cout) {
    const char* fn = "head_1x1";
    if (Cin < 0 || H <= 0 || W_ <= 0 || Cout <= 0) die(fn, "bad shape");
    if ((Cin && !a) || (Cin && !Wt) || !bias || !logits) die(fn, "NULL argument");
    Scratch s(fn);
    const long HW = (long)H * W_, n = (long)Cout * HW;
    const float* da = s.upload(a, (size_t)Cin * HW);
    const float* dW = s.upload(Wt, (size_t)Cout * Cin);
    const float* db = s.upload(bias, (size_t)Cout);
    float* dO = s.alloc<float>((size_t)n);
    head_kernel<<<grid_for(n), kThreads>>>(da, dW, db, dO, Cin, HW, Cout);
    s.download(logits, dO, (size_t)n);
}
