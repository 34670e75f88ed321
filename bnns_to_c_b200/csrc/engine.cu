// engine.cu - the B200 forward engine behind bnn_forward and its extensions.
//
// Per device, a Model owns (created on first use on that device):
//   * a weight arena: the blob's weights re-laid out once for the kernels
//     (first conv as +-1.0f [Cout][tap][band]; binary convs as tap-major
//     channel-packed uint32 [CoutP][9][Kw] with per-tap popcounts; folds in
//     interval form),
//   * an activation arena: every intermediate bit plane of one (N, H, W),
//   * captured CUDA graphs of the whole forward, keyed by (N, H, W, in, out),
//   * a compute stream and two copy streams for pipelined host batches.
// The forward order is the reference's (csrc/bnn_model.c:150-253): 19
// kernel launches (first conv, 17 fused binary convs, head).
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "common.h"
#include "kernels.cuh"
#include "realin_tx.cuh"

namespace bnn {

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) return set_error(BNN_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

static inline int cdiv(long a, long b) { return (int)((a + b - 1) / b); }
static inline int cw_of(int c) { return (c + 31) >> 5; }

// -------------------------------------------------------------------
// host-side fault injection (bnn_debug_inject_fault; tests of the failure
// paths, no GPU fault involved)
// -------------------------------------------------------------------
static std::atomic<int> g_fail_alloc{0};   // the k-th next device allocation fails
static std::atomic<int> g_fail_wait{0};    // the next synchronous call meets a wait that gives up
static std::atomic<int> g_fail_shard{-1};  // this shard of the next multi-device batch fails

// arena poison byte: -2 = not yet read from the environment, -1 = off
static std::atomic<int> g_poison{-2};

int arena_poison_byte() {
    int v = g_poison.load();
    if (v == -2) {
        const char* e = getenv("BNN_ARENA_POISON");
        const int want = e ? (atoi(e) & 255) : -1;
        g_poison.compare_exchange_strong(v, want);
        v = g_poison.load();
    }
    return v;
}

// fill a whole activation arena with the poison byte on stream s (no-op when off)
static int poison_arena(void* base, size_t bytes, cudaStream_t s) {
    const int b = arena_poison_byte();
    if (b < 0 || !base) return BNN_OK;
    if (cudaMemsetAsync(base, b, bytes, s) != cudaSuccess)
        return set_error(BNN_ERR_CUDA, "arena poison: %s", cudaGetErrorString(cudaGetLastError()));
    return BNN_OK;
}

// Programmatic dependent launch for the forward's kernels when the batch is
// small (most SMs idle, so the next kernel's prologue - TMEM, barriers,
// weights - overlaps this one's tail): set per forward by forward_launches,
// read by the launch sites below. BNN_PDL=0 in the environment turns it off.
static thread_local bool t_pdl = false;
static bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("BNN_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}
constexpr double kPdlPixels = 16.0 * 1024;  // batches of at most 16 32x32 patches

// launch kern<<<grid, block, smem, st>>>(args...), with the programmatic
// stream serialisation attribute when t_pdl is set
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                            Args&&... args) {
    if (!t_pdl) {
        kern<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// every device allocation of the engine goes through here
template <class T>
static cudaError_t dev_malloc(T** p, size_t bytes) {
    int k = g_fail_alloc.load();
    while (k > 0 && !g_fail_alloc.compare_exchange_weak(k, k - 1)) {
    }
    if (k == 1) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMalloc((void**)p, bytes);
}

// name of the last binary-conv kernel this thread launched (with its
// template parameters), for benchmarks and tests that must know which
// implementation ran
static thread_local char g_last_kernel[96];
static void note_kernel(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
static void note_kernel(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_kernel, sizeof g_last_kernel, fmt, ap);
    va_end(ap);
}

// -------------------------------------------------------------------
// device-side layer descriptions
// -------------------------------------------------------------------
struct BinLayer {
    int Cin, Cout, CoutP, cw0, cw1, Kw, sC;  // sC: channels from the first source
    uint32_t* wt = nullptr;
    int* wpop = nullptr;
    int8_t* w8 = nullptr;     // mma.sync kernel weights [Kw][9][CoutP][32]
    int8_t* wu = nullptr;     // tcgen05 kernel weights [Cout/ubn][Kw][9][2][ubn][16]
    int ubn = 0;              // tcgen05 channel block (N of one MMA)
    int8_t* wx = nullptr;     // ubn == 32: the same weights for bconv_wsx_kernel [Kw][3 dy][2][3 dx][32][16]
    int8_t* w4 = nullptr;     // the same weights as e2m1 nibbles for the kind::mxf4 kernel (layout of wu, two words a step)
    int8_t* wus = nullptr;    // the layout of wu in 32-channel blocks (small batches: more CTAs per layer)
    FoldIv* fold = nullptr;
    FoldIv* fold2 = nullptr;  // pooled branch (encoder conv2) or nullptr
};

struct Profiler {
    struct Rec {
        std::string label, optype;
        double work = 0, ms = 0;
        int calls = 0;
    };
    bool on = false;
    std::vector<Rec> recs;
    std::mutex mu;
    void add(const std::string& label, const char* optype, double work, double ms) {
        std::lock_guard<std::mutex> g(mu);
        for (auto& r : recs)
            if (r.label == label) { r.work += work; r.ms += ms; r.calls++; return; }
        recs.push_back(Rec{label, optype, work, ms, 1});
    }
};

struct Arena {
    int N = 0, H = 0, W = 0;
    void* base = nullptr;
    size_t bytes = 0;
    uint32_t *enc_h[4], *skip[4], *down[4], *bott_h, *bott_x, *dec_h[4], *dec_x[4];
    uint32_t* stem = nullptr; // v2: the stem's bit plane (enc1.conv1's input)
    uint32_t* rm_list;        // first conv: undecided (pixel, channel group, mask) entries
    unsigned int* rm_ctl;     // [entries, overflow, outputs]
    int rm_cap;
};

struct GraphKey {
    int N, H, W;
    const void* in;
    const void* out;
    bool operator<(const GraphKey& o) const {
        return std::tie(N, H, W, in, out) < std::tie(o.N, o.H, o.W, o.in, o.out);
    }
};

struct DevState {
    int device = -1;
    std::mutex mu;
    void* wbase = nullptr;
    float* ri_wf = nullptr;
    float* ri_fold = nullptr;
    int ri_CinP = 0, ri_CIP = 0;
    uint4* rm_wfrag = nullptr;  // first conv +-1 int8 weights in mma B-fragment order
    int* rm_exact = nullptr;    // per channel: fold not monotone -> exact path
    int8_t* rw_wu = nullptr;    // first conv +-1 int8 weights for realin_ws_kernel (Cin <= 128, Cout <= 32)
    int8_t* rx_wu = nullptr;    // the same for realin_dxn_kernel (column taps stacked in N)
    std::vector<RwThr> rw_thr;  // first conv fold thresholds for realin_ws_kernel (host copy, 32 entries)
    long long rw_wsum[32] = {};  // per channel: the sum of its first-conv weights over taps and bands
    float* st_w = nullptr;      // v2 stem weights [slice][band][st_CB] (+-1, 0)
    float* st_fold = nullptr;   // v2 stem [channel][5]: alpha, A, B, slope, rsign
    int st_CB = 0, st_slices = 0;
    BinLayer enc1[4], enc2[4], bott1, bott2, dec1[4], dec2[4];
    float *head_W = nullptr, *head_b = nullptr;
    Arena ar;
    cudaStream_t cs = nullptr, h2d = nullptr, d2h = nullptr;
    std::map<GraphKey, cudaGraphExec_t> graphs;
    // pipelined host batches: two device staging slots
    float* pin[2] = {nullptr, nullptr};
    float* pout[2] = {nullptr, nullptr};
    size_t pcap = 0;  // patches per slot
    int pbands = 0, pclasses = 0, pH = 0, pW = 0;
    cudaEvent_t ev_in[2], ev_comp[2], ev_out[2];
    cudaEvent_t ev_last;  // completion of the last forward enqueued on this device
    bool events = false;
    unsigned int* wt_host = nullptr;  // pinned: the device wait give-up counter at a call's start and end
    // patched (scene) forward: a chunk of tiles in and out, and a scene slab
    float *tin = nullptr, *tout = nullptr;
    size_t tcap = 0;  // floats of tin / tout
    size_t tcap_out = 0;
    float *scube = nullptr, *slog = nullptr;
    size_t scube_cap = 0, slog_cap = 0;  // floats
};

struct Engine {
    std::mutex mu;
    std::map<int, std::unique_ptr<DevState>> devs;
    std::vector<int> devices;  // empty: current device
    int chunk = 256;
    Profiler prof;
    // v2 model: the stem run before the body (arrays borrowed from the
    // StemModel that owns this engine); stem_c = 0 for a v1 model
    int stem_c = 0;
    Conv stem_conv{};
    Act stem_act{};
};

void* engine_create() { return new (std::nothrow) Engine(); }

void* engine_create_stem(const Conv* stem_conv, const Act* stem_act) {
    Engine* E = new (std::nothrow) Engine();
    if (!E) return nullptr;
    E->stem_c = stem_conv->Cout;
    E->stem_conv = *stem_conv;
    E->stem_act = *stem_act;
    return E;
}

int engine_stem_c(const void* e) { return e ? ((const Engine*)e)->stem_c : 0; }

static const Engine* eng(const Model* m) { return (const Engine*)m->engine; }

// topology of the model behind an engine (v1, or the body of a v2 model)
static int topo(const Model* m, Topology* t) { return validate_topology(m, t, eng(m)->stem_c); }

static void dev_release(DevState* d) {
    if (!d || d->device < 0) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(d->device);
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
    if (d->cs) cudaStreamSynchronize(d->cs);
    if (d->h2d) cudaStreamSynchronize(d->h2d);
    if (d->d2h) cudaStreamSynchronize(d->d2h);
    cudaFree(d->wbase);
    cudaFree(d->ar.base);
    for (int s = 0; s < 2; ++s) { cudaFree(d->pin[s]); cudaFree(d->pout[s]); }
    cudaFree(d->tin); cudaFree(d->tout); cudaFree(d->scube); cudaFree(d->slog);
    if (d->events)
    {
        for (int s = 0; s < 2; ++s) {
            cudaEventDestroy(d->ev_in[s]); cudaEventDestroy(d->ev_comp[s]); cudaEventDestroy(d->ev_out[s]);
        }
        cudaEventDestroy(d->ev_last);
    }
    if (d->cs) cudaStreamDestroy(d->cs);
    if (d->h2d) cudaStreamDestroy(d->h2d);
    if (d->d2h) cudaStreamDestroy(d->d2h);
    if (d->wt_host) cudaFreeHost(d->wt_host);
    d->wt_host = nullptr;
    cudaSetDevice(prev);
}

void engine_destroy(void* e) {
    Engine* E = (Engine*)e;
    if (!E) return;
    for (auto& kv : E->devs) dev_release(kv.second.get());
    delete E;
}

// -------------------------------------------------------------------
// host-side relayout of the blob into the device formats
// -------------------------------------------------------------------
static FoldIv to_iv(int type, int t, int lo, int hi) {
    const int MN = INT32_MIN, MX = INT32_MAX;
    switch (type) {
        case 0: return FoldIv{MN, MX, t > 0 ? 0 : 1, 0};
        case 1: return FoldIv{t, MX, 0, 0};
        case 2: return FoldIv{MN, t, 0, 0};
        case 3: return FoldIv{lo, hi, 0, 0};
        case 4: return FoldIv{lo, hi, 1, 0};
        default: return FoldIv{MX, MN, 0, 0};  // empty: always -1
    }
}

struct HostBin {
    std::vector<uint32_t> wt;
    std::vector<int8_t> w8, wu, wx, w4, wus;
    std::vector<int> wpop;
    std::vector<FoldIv> fold, fold2;
};

// tiles per work item of the tcgen05 binary conv at 128 / 256 channels
// (TMEM: two accumulator sets when BN * MT <= 256, one otherwise). Measured:
// 512 positions x 128 channels and 256 x 256 (one set each, weights re-read
// half as often) beat 256 x 128 and 128 x 256 (two sets) by 10-25% on the
// 128- and 256-channel layers.
#ifndef BNN_WS128_MT
#define BNN_WS128_MT 4
#endif
#ifndef BNN_WS256_MT
#define BNN_WS256_MT 2
#endif
// epilogue warps of the pooled tcgen05 kernel (4 or 8; the producers take the other 14 - EW)
#ifndef BNN_POOL_EPI_WARPS
#define BNN_POOL_EPI_WARPS 8
#endif
// tiles per work item of the kind::mxf4 (e2m1) kernel: 32 TMEM columns hold
// the block scales, so the item shapes that filled all 512 columns shrink
#ifndef BNN_F4_MT32
#define BNN_F4_MT32 7
#endif
#ifndef BNN_F4_MT64
#define BNN_F4_MT64 3
#endif
#ifndef BNN_F4_MT128
#define BNN_F4_MT128 3
#endif

// tcgen05 channel block for a layer of Cout channels: the whole layer up to
// 256 channels (N of one MMA), 256-channel blocks beyond
static int ws_bn(int Cout) { return Cout <= 32 ? 32 : Cout <= 64 ? 64 : Cout <= 128 ? 128 : 256; }

// kidx-ordered uint64 rows (bit (ci*9+t)) -> [CoutP][9][Kw] with the first
// sC channels in words [0, cw0) and the rest in words [cw0, cw0+cw1).
static void relayout_bin(const uint64_t* packed, int nwords, int Cin, int Cout, int sC, BinLayer& L,
                         HostBin& h, bool pooled) {
    L.Cin = Cin; L.Cout = Cout; L.sC = sC;
    L.cw0 = cw_of(sC);
    L.cw1 = Cin > sC ? cw_of(Cin - sC) : 0;
    L.Kw = L.cw0 + L.cw1;
    L.CoutP = cdiv(Cout, 128) * 128;
    h.wt.assign((size_t)L.CoutP * 9 * L.Kw, 0u);
    h.w8.assign((size_t)L.Kw * 9 * L.CoutP * 32, (int8_t)0);
    h.wpop.assign((size_t)L.CoutP * 9, 0);
    for (int co = 0; co < Cout; ++co) {
        const uint64_t* row = packed + (size_t)co * nwords;
        for (int ci = 0; ci < Cin; ++ci) {
            const int word = ci < sC ? (ci >> 5) : L.cw0 + ((ci - sC) >> 5);
            const int bit = ci < sC ? (ci & 31) : ((ci - sC) & 31);
            for (int t = 0; t < 9; ++t) {
                const int k = ci * 9 + t;
                const bool plus = (row[k >> 6] >> (k & 63)) & 1ull;
                if (plus) {
                    h.wt[((size_t)co * 9 + t) * L.Kw + word] |= 1u << bit;
                    h.wpop[(size_t)co * 9 + t] += 1;
                }
                h.w8[(((size_t)word * 9 + t) * L.CoutP + co) * 32 + bit] = plus ? 1 : -1;
            }
        }
    }
    // tcgen05 blocks: per (channel block, word) the 9 taps' B operands in the
    // order the kernel stages them ([tap][16-byte K half][channel][16 bytes])
    // pooled layers keep four phase accumulators in TMEM: channel blocks of at most 128
    const int bn = pooled ? std::min(ws_bn(Cout), 128) : ws_bn(Cout), ncb = cdiv(Cout, bn);
    L.ubn = bn;
    auto block_layout = [&](int b, std::vector<int8_t>& w) {
        const int nb = cdiv(Cout, b);
        w.assign((size_t)nb * L.Kw * 9 * 2 * b * 16, (int8_t)0);
        for (int cb = 0; cb < nb; ++cb)
            for (int kw = 0; kw < L.Kw; ++kw)
                for (int t = 0; t < 9; ++t)
                    for (int hh = 0; hh < 2; ++hh)
                        for (int c = 0; c < b && cb * b + c < Cout; ++c)
                            memcpy(&w[((((size_t)cb * L.Kw + kw) * 9 + t) * 2 + hh) * b * 16 + (size_t)c * 16],
                                   &h.w8[(((size_t)kw * 9 + t) * L.CoutP + cb * b + c) * 32 + hh * 16], 16);
    };
    block_layout(bn, h.wu);
    block_layout(32, h.wus);  // small batches (launch_bconv)
    // the kind::mxf4 kernel: per (channel block, K step of two words) the 9
    // taps' B operands [tap][word of the step][channel][16 bytes], each
    // 16 bytes = 32 e2m1 nibbles (channel j of the word in byte j/2, low
    // nibble for even j: +1 -> 0x2, -1 -> 0xA, absent -> 0); channel blocks
    // of at most 128 (a 256-wide block leaves room for one tile per item)
    {
        const int KS = (L.Kw + 1) / 2, bn4 = std::min(bn, 128), ncb4 = cdiv(Cout, bn4);
        h.w4.assign((size_t)ncb4 * KS * 9 * 2 * bn4 * 16, (int8_t)0);
        for (int cb = 0; cb < ncb4; ++cb)
            for (int kw = 0; kw < L.Kw; ++kw)
                for (int t = 0; t < 9; ++t)
                    for (int c = 0; c < bn4 && cb * bn4 + c < Cout; ++c) {
                        const int8_t* src = &h.w8[(((size_t)kw * 9 + t) * L.CoutP + cb * bn4 + c) * 32];
                        int8_t* dst = &h.w4[((((size_t)cb * KS + kw / 2) * 9 + t) * 2 + (kw & 1)) * bn4 * 16 +
                                            (size_t)c * 16];
                        for (int j = 0; j < 32; ++j) {
                            const uint8_t nib = src[j] > 0 ? 0x2 : src[j] < 0 ? 0xA : 0x0;
                            dst[j >> 1] = (int8_t)((uint8_t)dst[j >> 1] | (uint8_t)(nib << ((j & 1) * 4)));
                        }
                    }
    }
    // 32-channel layers: the column taps of a kernel row stacked in N for
    // bconv_wsx_kernel ([word][dy][16-byte K half][dx][channel][16 bytes])
    h.wx.clear();
    if (bn == 32) {
        h.wx.assign((size_t)L.Kw * 3 * 2 * 3 * 32 * 16, (int8_t)0);
        for (int kw = 0; kw < L.Kw; ++kw)
            for (int dy = 0; dy < 3; ++dy)
                for (int hh = 0; hh < 2; ++hh)
                    for (int dx = 0; dx < 3; ++dx)
                        for (int c = 0; c < Cout; ++c)
                            memcpy(&h.wx[((((size_t)kw * 3 + dy) * 2 + hh) * 3 + dx) * 32 * 16 + (size_t)c * 16],
                                   &h.w8[(((size_t)kw * 9 + dy * 3 + dx) * L.CoutP + c) * 32 + hh * 16], 16);
    }
}

static void folds_of(const Act* a, int CoutP, std::vector<FoldIv>& v) {
    v.assign((size_t)CoutP, FoldIv{INT32_MAX, INT32_MIN, 0, 0});
    for (int c = 0; c < a->C; ++c) v[c] = to_iv(a->type[c], a->t[c], a->lo[c], a->hi[c]);
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Opt every kernel into the dynamic shared memory its largest tile needs.
// Done once per device (a context-level attribute), before any capture.
template <int BN, int TM, int TN, int KC>
static cudaError_t attr_bconv() {
    return cudaFuncSetAttribute(bconv3x3_kernel<BN, TM, TN, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)BconvCfg<BN, TM, TN, KC>::smem_bytes(512));
}
template <int BN, int MT, int EW = BNN_POOL_EPI_WARPS>
static cudaError_t attr_ws_pool() {
    return cudaFuncSetAttribute(bconv_ws_pool_kernel<BN, MT, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)WsPoolCfg<BN, MT, EW>::max_smem);
}
template <int BN, int MT, bool F4 = false, int EW = 8>
static cudaError_t attr_ws() {
    return cudaFuncSetAttribute(bconv_ws_kernel<BN, MT, F4, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)WsCfg<BN, MT, F4, EW>::max_smem);
}
template <int MT>
static cudaError_t attr_wsx() {
    return cudaFuncSetAttribute(bconv_wsx_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)WsxCfg<MT>::max_smem);
}
template <int BN>
static cudaError_t attr_bmma() {
    return cudaFuncSetAttribute(bconv_mma_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)BmmaCfg<BN>::smem_bytes(512));
}
template <int BN, int TM, int TN>
static cudaError_t attr_bconv_kc() {
    cudaError_t e;
    if ((e = attr_bconv<BN, TM, TN, 8>()) != cudaSuccess) return e;
    if ((e = attr_bconv<BN, TM, TN, 4>()) != cudaSuccess) return e;
    if ((e = attr_bconv<BN, TM, TN, 2>()) != cudaSuccess) return e;
    return attr_bconv<BN, TM, TN, 1>();
}
// stem weights in shared memory: up to 1024 bands x 32 channels; the
// bulk-copy kernel: weights and its ring, one CTA per SM
template <int CB>
static cudaError_t attr_stem() {
    const int smem = 1024 * CB * 4;
    constexpr int PXB = CB == 32 ? 2 : 4;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(stem_fold_kernel<CB, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(stem_fold_kernel<CB, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(stem_bulk_kernel<CB, PXB>, cudaFuncAttributeMaxDynamicSharedMemorySize, SB_SMEM)))
        return e;
    if constexpr (CB == 32) return cudaSuccess;
    else return cudaFuncSetAttribute(stem_fold_kernel<CB, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

static int set_kernel_attrs(int device) {
    static std::mutex mu;
    static bool done[64] = {false};
    std::lock_guard<std::mutex> g(mu);
    if (device >= 0 && device < 64 && done[device]) return BNN_OK;
    cudaError_t e;
    if ((e = attr_bconv_kc<32, 4, 4>()) != cudaSuccess || (e = attr_bconv_kc<64, 8, 4>()) != cudaSuccess ||
        (e = attr_bconv_kc<128, 8, 8>()) != cudaSuccess || (e = attr_bmma<32>()) != cudaSuccess ||
        (e = attr_bmma<64>()) != cudaSuccess || (e = attr_bmma<128>()) != cudaSuccess ||
        (e = attr_ws<32, 8>()) != cudaSuccess || (e = attr_ws<64, 4>()) != cudaSuccess ||
        (e = attr_ws<128, BNN_WS128_MT>()) != cudaSuccess || (e = attr_ws<256, BNN_WS256_MT>()) != cudaSuccess ||
        (e = attr_ws<32, BNN_F4_MT32, true>()) != cudaSuccess || (e = attr_ws<64, BNN_F4_MT64, true>()) != cudaSuccess ||
        (e = attr_ws<128, BNN_F4_MT128, true>()) != cudaSuccess ||
        (e = attr_ws<32, 8, false, 4>()) != cudaSuccess ||
        (e = attr_ws<64, BNN_F4_MT64, true, 4>()) != cudaSuccess ||
        (e = attr_ws_pool<32, 2>()) != cudaSuccess || (e = attr_ws_pool<64, 1>()) != cudaSuccess ||
        (e = attr_ws_pool<128, 1>()) != cudaSuccess || (e = attr_wsx<2>()) != cudaSuccess ||
        (e = attr_ws_pool<64, 1, 4>()) != cudaSuccess || (e = attr_ws<32, 1>()) != cudaSuccess ||
        (e = attr_ws_pool<32, 1>()) != cudaSuccess ||
        (e = cudaFuncSetAttribute(realin3x3_fold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  RI_HP * 260 * 4)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(realin_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RM_SMEM)) !=
            cudaSuccess ||
        (e = cudaFuncSetAttribute(realin_ws_kernel<0, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)RW_MAX_SMEM)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(realin_ws_kernel<32, 7>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)RW_MAX_SMEM)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(realin_dxn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RW_MAX_SMEM)) !=
            cudaSuccess ||
        (e = cudaFuncSetAttribute(realin_tx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TX_MAX_SMEM)) !=
            cudaSuccess ||
        (e = attr_stem<8>()) != cudaSuccess || (e = attr_stem<16>()) != cudaSuccess ||
        (e = attr_stem<32>()) != cudaSuccess)
        return set_error(BNN_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (device >= 0 && device < 64) done[device] = true;
    return BNN_OK;
}

// The reference's real fold on one float accumulator, with the device's
// operations and rounding (IEEE binary32, round to nearest, one fused
// multiply-add).
__attribute__((optimize("fp-contract=off"))) static int host_real_fold(float acc, const float* f) {
    const float o = f[0] * acc;
    float z = std::fmaf(f[1], o, f[2]);
    if (z < 0.0f) z = f[3] * z;
    return (z + f[4]) > 0.0f;
}
// finite floats <-> ordered integer keys (-0 and +0 share key 0)
static int64_t float_key(float x) {
    int32_t b;
    memcpy(&b, &x, 4);
    return b >= 0 ? (int64_t)b : -(int64_t)(b & 0x7fffffff);
}
static float key_float(int64_t k) {
    const uint32_t b = k >= 0 ? (uint32_t)k : ((uint32_t)(-k) | 0x80000000u);
    float x;
    memcpy(&x, &b, 4);
    return x;
}

// RwThr of one first-conv channel (f = alpha, A, B, slope, rsign): the fold
// is monotone in the accumulator (the channel is not exact), so one
// bisection over the ordered finite floats finds where it flips
static RwThr fold_threshold(const float* f, bool exact) {
    const long long BIG = 1ll << 62;
    RwThr t{BIG, 1, exact ? 1 : 0};
    if (exact) return t;
    const int64_t klo = float_key(-FLT_MAX), khi = float_key(FLT_MAX);
    const int flo = host_real_fold(-FLT_MAX, f), fhi = host_real_fold(FLT_MAX, f);
    if (flo == fhi) {
        t.C = flo ? -BIG : BIG;
        return t;
    }
    int64_t a = klo, b = khi;  // f(a) = flo, f(b) = fhi
    while (b - a > 1) {
        const int64_t mid = a + (b - a) / 2;
        if (host_real_fold(key_float(mid), f) == flo) a = mid;
        else b = mid;
    }
    auto clamp = [&](double v) { return v >= (double)BIG ? BIG : v <= -(double)BIG ? -BIG : (long long)v; };
    if (fhi) {  // increasing: 1 from tau = key_float(b) on
        t.sgn = 1;
        t.C = clamp(std::ceil((double)key_float(b) * 262144.0));
    } else {    // decreasing: 1 up to tau = key_float(a)
        t.sgn = -1;
        t.C = -clamp(std::floor((double)key_float(a) * 262144.0));
    }
    return t;
}

// upload everything to device d (called with d->mu held, device current)
static int dev_init(const Model* m, DevState* d) {
    Topology tp;
    int rc = topo(m, &tp);
    if (rc) return rc;
    if ((rc = set_kernel_attrs(d->device))) return rc;
    const Engine* E = eng(m);
    const bool stem = E->stem_c > 0;
    // first conv of a v1 model: tables of the exact, mma.sync and tcgen05
    // kernels. wsign is -1, 0 or +1 (checked at load) and goes in as is.
    std::vector<float> wf, rfold;
    std::vector<uint32_t> wfrag;
    std::vector<int> rexact;
    std::vector<int8_t> rwu, rxu;
    std::vector<RwThr> rthr;
    // stem of a v2 model: [slice][band][CB] weights and [channel][5] folds
    std::vector<float> sw, sfold;
    if (stem) {
        const Conv* sc = &E->stem_conv;
        const Act* sa = &E->stem_act;
        const int C = sc->Cout, Cin = sc->Cin;
        const int CB = C <= 8 ? 8 : C <= 16 ? 16 : 32, slices = cdiv(C, CB);
        d->st_CB = CB;
        d->st_slices = slices;
        sw.assign((size_t)slices * Cin * CB, 0.0f);
        sfold.assign((size_t)slices * CB * 5, 0.0f);
        for (int co = 0; co < C; ++co) {
            const int sl = co / CB, c = co % CB;
            for (int ci = 0; ci < Cin; ++ci)
                sw[((size_t)sl * Cin + ci) * CB + c] = (float)sc->wsign[(size_t)co * Cin + ci];
            sfold[co * 5 + 0] = sc->alpha[co];
            sfold[co * 5 + 1] = sa->A[co];
            sfold[co * 5 + 2] = sa->B[co];
            sfold[co * 5 + 3] = sa->slope[co];
            sfold[co * 5 + 4] = sa->rsign[co];
        }
    } else {
        const Conv* c1 = &m->enc_conv1[0];
        const Act* a1 = &m->enc_act1[0];
        const int Cin = c1->Cin, CoutR = c1->Cout, CoutRP = cdiv(CoutR, 32) * 32;
        d->ri_CinP = cdiv(Cin, 4) * 4;
        d->ri_CIP = d->ri_CinP + (((d->ri_CinP / 4) % 2 == 0) ? 4 : 0);
        wf.assign((size_t)CoutRP * 9 * d->ri_CinP, 0.0f);
        rfold.assign((size_t)CoutRP * 5, 0.0f);
        for (int co = 0; co < CoutR; ++co) {
            for (int ci = 0; ci < Cin; ++ci)
                for (int t = 0; t < 9; ++t)
                    wf[((size_t)co * 9 + t) * d->ri_CinP + ci] = (float)c1->wsign[((size_t)co * Cin + ci) * 9 + t];
            rfold[co * 5 + 0] = c1->alpha[co];
            rfold[co * 5 + 1] = a1->A[co];
            rfold[co * 5 + 2] = a1->B[co];
            rfold[co * 5 + 3] = a1->slope[co];
            rfold[co * 5 + 4] = a1->rsign[co];
        }
        // the same weights as int8 mma B fragments (realin_mma_kernel): for
        // channel group g, tap t, k-step kk, lane l = 4*gid + tig, n-tile nt:
        // b0 = bands kk*32 + tig*4 + 0..3 and b1 = bands kk*32 + 16 + tig*4 + 0..3
        // of channel g*32 + nt*8 + gid
        const int ngrp = cdiv(CoutR, 32);
        wfrag.assign((size_t)ngrp * 9 * 4 * 32 * 8, 0u);
        rexact.assign((size_t)CoutRP, 0);
        if (Cin <= RM_CINP) {
            for (int g = 0; g < ngrp; ++g)
                for (int t = 0; t < 9; ++t)
                    for (int kk = 0; kk < 4; ++kk)
                        for (int l = 0; l < 32; ++l)
                            for (int nt = 0; nt < 4; ++nt)
                                for (int h = 0; h < 2; ++h) {
                                    const int co = g * 32 + nt * 8 + (l >> 2);
                                    uint32_t word = 0;
                                    for (int i = 0; i < 4; ++i) {
                                        const int ci = kk * 32 + h * 16 + (l & 3) * 4 + i;
                                        int v = 0;
                                        if (co < CoutR && ci < Cin) v = c1->wsign[((size_t)co * Cin + ci) * 9 + t];
                                        word |= (uint32_t)(uint8_t)(int8_t)v << (8 * i);
                                    }
                                    wfrag[((((size_t)g * 9 + t) * 4 + kk) * 32 + l) * 8 + nt * 2 + h] = word;
                                }
        }
        // the same weights for realin_ws_kernel: [chunk][tap][16-band half][channel][16 bands]
        if (Cin <= RM_CINP && CoutR <= 32) {
            rwu.assign(RW_WBYTES, (int8_t)0);
            for (int kc = 0; kc < 4; ++kc)
                for (int t = 0; t < 9; ++t)
                    for (int h = 0; h < 2; ++h)
                        for (int co = 0; co < CoutR; ++co)
                            for (int i = 0; i < 16; ++i) {
                                const int ci = kc * 32 + h * 16 + i;
                                if (ci < Cin)
                                    rwu[((((size_t)kc * 9 + t) * 2 + h) * 32 + co) * 16 + i] =
                                        c1->wsign[((size_t)co * Cin + ci) * 9 + t];
                            }
        }
        // and for realin_dxn_kernel: [chunk][kernel row][16-band half][column tap * 32 + channel][16 bands]
        if (!rwu.empty()) {
            rxu.assign(RX_WBYTES, (int8_t)0);
            for (int kc = 0; kc < 4; ++kc)
                for (int t = 0; t < 9; ++t)
                    for (int h = 0; h < 2; ++h)
                        for (int co = 0; co < CoutR; ++co)
                            for (int i = 0; i < 16; ++i)
                                rxu[((((size_t)kc * 3 + t / 3) * 2 + h) * 96 + (t % 3) * 32 + co) * 16 + i] =
                                    rwu[((((size_t)kc * 9 + t) * 2 + h) * 32 + co) * 16 + i];
        }
        if (!rwu.empty()) {
            rthr.assign(32, RwThr{1ll << 62, 1, 0});
            for (int co = 0; co < CoutR; ++co) {
                long long s = 0;
                for (size_t k = 0; k < (size_t)Cin * 9; ++k) s += c1->wsign[(size_t)co * Cin * 9 + k];
                d->rw_wsum[co] = s;
            }
        }
        for (int co = 0; co < CoutR; ++co) {
            const float v[5] = {c1->alpha[co], a1->A[co], a1->B[co], a1->slope[co], a1->rsign[co]};
            bool ok = v[3] >= 0.0f;
            for (float f : v) ok = ok && std::isfinite(f);
            rexact[co] = ok ? 0 : 1;
            if (!rthr.empty()) rthr[co] = fold_threshold(v, !ok);
        }
        // realin_ws_kernel computes -Q for decreasing folds (the dxn / tx copies above keep the signs)
        if (BNN_RW_NEGW && !rwu.empty())
            for (int co = 0; co < CoutR; ++co)
                if (rthr[co].sgn < 0)
                    for (size_t blk = 0; blk < (size_t)4 * 9 * 2; ++blk)
                        for (int i = 0; i < 16; ++i) rwu[(blk * 32 + co) * 16 + i] = (int8_t)-rwu[(blk * 32 + co) * 16 + i];
    }
    // binary convs
    struct Item {
        BinLayer* L;
        const Conv* c;
        const Act* a;
        const Act* a2;
        int sC;
        HostBin h;
    };
    std::vector<Item> items;
    for (int i = 0; i < 4; ++i) {
        if (i > 0 || stem)
            items.push_back({&d->enc1[i], &m->enc_conv1[i], &m->enc_act1[i], nullptr, m->enc_conv1[i].Cin, {}});
        items.push_back({&d->enc2[i], &m->enc_conv2[i], &m->enc_act2_skip[i], &m->enc_act2_down[i],
                         m->enc_conv2[i].Cin, {}});
    }
    items.push_back({&d->bott1, &m->bott_conv1, &m->bott_act1, nullptr, m->bott_conv1.Cin, {}});
    items.push_back({&d->bott2, &m->bott_conv2, &m->bott_act2, nullptr, m->bott_conv2.Cin, {}});
    for (int i = 0; i < 4; ++i) {
        items.push_back({&d->dec1[i], &m->dec_conv1[i], &m->dec_act1[i], nullptr, tp.enc[3 - i], {}});
        items.push_back({&d->dec2[i], &m->dec_conv2[i], &m->dec_act2[i], nullptr, m->dec_conv2[i].Cin, {}});
    }
    size_t total = align256(wf.size() * 4) + align256(rfold.size() * 4) + align256(wfrag.size() * 4) +
                   align256(rexact.size() * 4) + align256(rwu.size()) + align256(rxu.size()) + align256(sw.size() * 4) +
                   align256(sfold.size() * 4);
    for (auto& it : items) {
        relayout_bin(it.c->packed, it.c->nwords, it.c->Cin, it.c->Cout, it.sC, *it.L, it.h, it.a2 != nullptr);
        folds_of(it.a, it.L->CoutP, it.h.fold);
        if (it.a2) folds_of(it.a2, it.L->CoutP, it.h.fold2);
        total += align256(it.h.wt.size() * 4) + align256(it.h.w8.size()) + align256(it.h.wu.size()) +
                 align256(it.h.wx.size()) + align256(it.h.w4.size()) + align256(it.h.wus.size()) +
                 align256(it.h.wpop.size() * 4) +
                 align256(it.h.fold.size() * sizeof(FoldIv)) + align256(it.h.fold2.size() * sizeof(FoldIv));
    }
    const size_t hw = (size_t)m->head_Cout * m->head_Cin;
    total += align256(hw * 4) + align256((size_t)m->head_Cout * 4);
    void* base = nullptr;
    if (dev_malloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_OOM, "cudaMalloc weights (%zu bytes) on device %d", total, d->device);
    }
    d->wbase = base;
    char* p = (char*)base;
    auto put = [&](const void* src, size_t bytes) -> void* {
        void* dst = p;
        if (bytes) cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
        p += align256(bytes);
        return dst;
    };
    d->ri_wf = (float*)put(wf.data(), wf.size() * 4);
    d->ri_fold = (float*)put(rfold.data(), rfold.size() * 4);
    d->rm_wfrag = (uint4*)put(wfrag.data(), wfrag.size() * 4);
    d->rm_exact = (int*)put(rexact.data(), rexact.size() * 4);
    d->rw_wu = rwu.empty() ? nullptr : (int8_t*)put(rwu.data(), rwu.size());
    d->rx_wu = rxu.empty() ? nullptr : (int8_t*)put(rxu.data(), rxu.size());
    d->rw_thr = rthr;
    d->st_w = sw.empty() ? nullptr : (float*)put(sw.data(), sw.size() * 4);
    d->st_fold = sfold.empty() ? nullptr : (float*)put(sfold.data(), sfold.size() * 4);
    for (auto& it : items) {
        it.L->wt = (uint32_t*)put(it.h.wt.data(), it.h.wt.size() * 4);
        it.L->w8 = (int8_t*)put(it.h.w8.data(), it.h.w8.size());
        it.L->wu = (int8_t*)put(it.h.wu.data(), it.h.wu.size());
        it.L->wx = it.h.wx.empty() ? nullptr : (int8_t*)put(it.h.wx.data(), it.h.wx.size());
        it.L->w4 = it.h.w4.empty() ? nullptr : (int8_t*)put(it.h.w4.data(), it.h.w4.size());
        it.L->wus = (int8_t*)put(it.h.wus.data(), it.h.wus.size());
        it.L->wpop = (int*)put(it.h.wpop.data(), it.h.wpop.size() * 4);
        it.L->fold = (FoldIv*)put(it.h.fold.data(), it.h.fold.size() * sizeof(FoldIv));
        it.L->fold2 = it.a2 ? (FoldIv*)put(it.h.fold2.data(), it.h.fold2.size() * sizeof(FoldIv)) : nullptr;
    }
    d->head_W = (float*)put(m->head_W, hw * 4);
    d->head_b = (float*)put(m->head_bias, (size_t)m->head_Cout * 4);
    CK(cudaGetLastError());
    CK(cudaStreamCreateWithFlags(&d->cs, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&d->h2d, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
    for (int s = 0; s < 2; ++s) {
        CK(cudaEventCreateWithFlags(&d->ev_in[s], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&d->ev_comp[s], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&d->ev_out[s], cudaEventDisableTiming));
    }
    CK(cudaEventCreateWithFlags(&d->ev_last, cudaEventDisableTiming));
    CK(cudaEventRecord(d->ev_last, d->cs));
    d->events = true;
    CK(cudaMallocHost((void**)&d->wt_host, 2 * sizeof(unsigned int)));
    d->wt_host[0] = d->wt_host[1] = 0u;
    return BNN_OK;
}

static int get_dev(const Model* m, int device, DevState** out) {
    Engine* E = (Engine*)m->engine;
    if (!E) return set_error(BNN_ERR_ARG, "model has no engine");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
        cudaGetLastError();
        return set_error(BNN_ERR_CUDA, "no CUDA device available");
    }
    if (device < 0 || device >= ndev) return set_error(BNN_ERR_ARG, "device %d out of range [0,%d)", device, ndev);
    DevState* d;
    {
        std::lock_guard<std::mutex> g(E->mu);
        auto& slot = E->devs[device];
        if (!slot) slot.reset(new DevState());
        d = slot.get();
    }
    std::lock_guard<std::mutex> g(d->mu);
    if (d->device < 0) {
        CK(cudaSetDevice(device));
        d->device = device;
        int rc = dev_init(m, d);
        if (rc) {
            dev_release(d);
            d->device = -1;
            d->wbase = nullptr;
            return rc;
        }
    }
    *out = d;
    return BNN_OK;
}

// -------------------------------------------------------------------
// activation arena
// -------------------------------------------------------------------
static int arena_reserve(const Model* m, DevState* d, int N, int H, int W) {
    Arena& a = d->ar;
    if (a.base && a.N >= N && a.H == H && a.W == W) return BNN_OK;
    Topology tp;
    topo(m, &tp);
    int Nn = std::max(N, a.H == H && a.W == W ? a.N : 0);
    size_t off = 0;
    std::vector<std::pair<uint32_t**, size_t>> plan;
    auto add = [&](uint32_t** slot, int h, int w, int c) {
        size_t bytes = (size_t)Nn * h * w * cw_of(c) * 4;
        plan.push_back({slot, off});
        off += align256(bytes + 4);
    };
    if (tp.stem) add(&a.stem, H, W, tp.stem);
    for (int i = 0; i < 4; ++i) {
        const int h = H >> i, w = W >> i;
        add(&a.enc_h[i], h, w, tp.enc[i]);
        add(&a.skip[i], h, w, tp.enc[i]);
        add(&a.down[i], h >> 1, w >> 1, tp.enc[i]);
    }
    add(&a.bott_h, H >> 4, W >> 4, m->bott_conv1.Cout);
    add(&a.bott_x, H >> 4, W >> 4, tp.bott);
    for (int i = 0; i < 4; ++i) {
        const int l = 3 - i;
        add(&a.dec_h[i], H >> l, W >> l, m->dec_conv1[i].Cout);
        add(&a.dec_x[i], H >> l, W >> l, tp.dec[i]);
    }
    // undecided-output list of the first conv: sized for ~1 in 64 outputs, at
    // least 64 K entries; beyond it the fix-up recomputes the whole batch
    const size_t outs = (size_t)Nn * H * W * m->enc_conv1[0].Cout;
    const int cap = tp.stem ? 0 : (int)std::min<size_t>(std::max<size_t>(outs / 64, 65536), (size_t)1 << 24);
    const size_t list_off = off;
    off += align256((size_t)cap * 16);
    const size_t ctl_off = off;
    off += 256;
    // graphs bake in arena pointers
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
    if (a.base) {
        CK(cudaEventSynchronize(d->ev_last));
        CK(cudaStreamSynchronize(d->cs));
        cudaFree(a.base);
        a.base = nullptr;
    }
    void* base = nullptr;
    if (dev_malloc(&base, off) != cudaSuccess) {
        cudaGetLastError();
        a.N = 0;
        return set_error(BNN_ERR_OOM, "cudaMalloc activation arena (%zu bytes)", off);
    }
    a.base = base;
    a.bytes = off;
    a.N = Nn; a.H = H; a.W = W;
    for (auto& pr : plan) *pr.first = (uint32_t*)((char*)base + pr.second);
    a.rm_list = (uint32_t*)((char*)base + list_off);
    a.rm_ctl = (unsigned int*)((char*)base + ctl_off);
    a.rm_cap = cap;
    return BNN_OK;
}

// -------------------------------------------------------------------
// launchers
// -------------------------------------------------------------------
// binary conv implementation: 0 = tcgen05 for non-pooled layers and mma.sync
// for pooled ones (default), 1 = XOR/POPC, 2 = mma.sync for every layer
static int g_bconv_kind = 0;

struct TileGeo {
    int TR, TC, TNI, tiles_x, tiles_y, tiles, HP;
};

static TileGeo tile_geo(int N, int H, int W, int BM) {
    TileGeo g;
    if (H * W <= BM) {
        g.TR = H; g.TC = W;
        g.TNI = std::max(1, std::min(BM / (H * W), 512 / ((H + 2) * (W + 2))));
        g.tiles_x = g.tiles_y = 1;
        g.tiles = cdiv(N, g.TNI);
    } else if (2 * W <= BM) {
        g.TC = W;
        g.TR = std::min(2 * (BM / (2 * W)), ((H + 1) / 2) * 2);
        g.TNI = 1;
        g.tiles_x = 1;
        g.tiles_y = cdiv(H, g.TR);
        g.tiles = N * g.tiles_y;
    } else {
        g.TR = 2; g.TC = BM / 2; g.TNI = 1;
        g.tiles_x = cdiv(W, g.TC);
        g.tiles_y = cdiv(H, 2);
        g.tiles = N * g.tiles_x * g.tiles_y;
    }
    g.HP = g.TNI * (g.TR + 2) * (g.TC + 2);
    return g;
}

template <int BN, int TM, int TN, int KC>
static int launch_bconv_t(BconvParams p, int N, cudaStream_t st) {
    using Cfg = BconvCfg<BN, TM, TN, KC>;
    TileGeo g = tile_geo(N, p.H, p.W, Cfg::BM);
    p.TR = g.TR; p.TC = g.TC; p.TNI = g.TNI; p.tiles_x = g.tiles_x; p.tiles_y = g.tiles_y; p.HP = g.HP;
    const size_t smem = Cfg::smem_bytes(g.HP);
    dim3 grid((unsigned)g.tiles, (unsigned)cdiv(p.Cout, BN));
    bconv3x3_kernel<BN, TM, TN, KC><<<grid, Cfg::NT, smem, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "bconv launch: %s", cudaGetErrorString(e));
    note_kernel("bconv3x3_kernel<%d,%d,%d,%d> (XOR+POPC)", BN, TM, TN, KC);
    return BNN_OK;
}

template <int BN, int TM, int TN>
static int launch_bconv_kc(BconvParams p, int N, cudaStream_t st) {
    const int Kw = p.Kw;
    if (Kw % 8 == 0) return launch_bconv_t<BN, TM, TN, 8>(p, N, st);
    if (Kw % 4 == 0) return launch_bconv_t<BN, TM, TN, 4>(p, N, st);
    if (Kw % 2 == 0) return launch_bconv_t<BN, TM, TN, 2>(p, N, st);
    return launch_bconv_t<BN, TM, TN, 1>(p, N, st);
}

template <int BN>
static int launch_bmma(BconvParams p, int N, cudaStream_t st) {
    using Cfg = BmmaCfg<BN>;
    TileGeo g = tile_geo(N, p.H, p.W, Cfg::BM);
    p.TR = g.TR; p.TC = g.TC; p.TNI = g.TNI; p.tiles_x = g.tiles_x; p.tiles_y = g.tiles_y; p.HP = g.HP;
    dim3 grid((unsigned)g.tiles, (unsigned)cdiv(p.Cout, BN));
    bconv_mma_kernel<BN><<<grid, Cfg::NT, Cfg::smem_bytes(g.HP), st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "bconv mma launch: %s", cudaGetErrorString(e));
    note_kernel("bconv_mma_kernel<%d> (mma.sync int8)", BN);
    return BNN_OK;
}


static int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// persistent tcgen05 kernel on the padded grid (non-pooled layers); returns
// BNN_ERR_UNSUPPORTED (and launches nothing) when the staging does not fit
template <int BN, int MT, bool F4 = false, int EW = 8>
static int launch_ws(BconvParams p, int N, cudaStream_t st) {
    using Cfg = WsCfg<BN, MT, F4, EW>;
    if (F4) {
        if (!p.w4) return BNN_ERR_UNSUPPORTED;
        p.wu = p.w4;
    }
    const long gk = std::max(1, 64 / (p.W + 1));
    const long Gw = gk * (p.W + 1) + 1;
    const long rows = (long)cdiv(N, gk) * (p.H + 1) + 1;
    const long ptot = (rows - 2) * Gw;  // output positions: grid rows 1 .. rows-2
    const long sp = ((Cfg::PI + 2 * Gw + 2) + 7) & ~7L;
    const long groups = (ptot + Cfg::PI - 1) / Cfg::PI;
    const long ncb = cdiv(p.Cout, BN);
    if (sp > Cfg::MAX_SP || groups * Cfg::PI + 2 * Gw + 2 >= (1L << 31) || groups * ncb >= (1L << 31))
        return BNN_ERR_UNSUPPORTED;
    const int ns = Cfg::stages((int)sp, (int)Gw, p.Cout);
    if (ns < 2) return BNN_ERR_UNSUPPORTED;
    p.gk = (int)gk; p.Gw = (int)Gw; p.HP = (int)sp;
    p.TR = (int)(groups * ncb); p.TC = (int)ncb; p.TNI = ns;
    // one CTA per SM (it allocates all of TMEM): never less than 116 KB
    const size_t smem = std::max<size_t>(
        (size_t)ns * Cfg::stage_bytes((int)sp) + Cfg::fixed_bytes((int)sp, (int)Gw, p.Cout), (size_t)116 * 1024);
    const int grid = (int)std::min<long>(groups * ncb, sm_count());
    cudaError_t e = launch_k(bconv_ws_kernel<BN, MT, F4, EW>, (unsigned)grid, Cfg::NT, smem, st, p);
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "bconv tcgen05 launch: %s", cudaGetErrorString(e));
    note_kernel("bconv_ws_kernel<%d,%d,%s,%d> (tcgen05 %s)", BN, MT, F4 ? "e2m1" : "i8", EW,
                F4 ? "kind::mxf4" : "kind::i8");
    return BNN_OK;
}

// 32-channel non-pooled layers with the column taps in N (bconv_wsx_kernel);
// BNN_ERR_UNSUPPORTED (nothing launched) when the staging does not fit
template <int MT>
static int launch_wsx(BconvParams p, int N, cudaStream_t st) {
    using Cfg = WsxCfg<MT>;
    if (!p.wx || p.Cout > 32) return BNN_ERR_UNSUPPORTED;
    const long gk = std::max(1, 64 / (p.W + 1));
    const long Gw = gk * (p.W + 1) + 1;
    const long rows = (long)cdiv(N, gk) * (p.H + 1) + 1;
    const long ptot = (rows - 2) * Gw;  // output positions: grid rows 1 .. rows-2
    const long sp = Cfg::sp_of((int)std::min<long>(Gw, 1L << 20));
    const long groups = (ptot + Cfg::PIV - 1) / Cfg::PIV;
    if (sp > Cfg::MAX_SP || groups * Cfg::PIV + 2 * Gw + 130 >= (1L << 31) || groups >= (1L << 31))
        return BNN_ERR_UNSUPPORTED;
    const int ns = Cfg::stages((int)sp, (int)Gw, p.Cout);
    if (ns < 2) return BNN_ERR_UNSUPPORTED;
    p.gk = (int)gk; p.Gw = (int)Gw; p.HP = (int)sp;
    p.TR = (int)groups; p.TC = 1; p.TNI = ns;
    p.wu = p.wx;
    const size_t smem = std::max<size_t>(
        (size_t)ns * Cfg::stage_bytes((int)sp) + Cfg::fixed_bytes((int)sp, (int)Gw, p.Cout), (size_t)116 * 1024);
    const int grid = (int)std::min<long>(groups, sm_count());
    bconv_wsx_kernel<MT><<<grid, Cfg::NT, smem, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "bconv tcgen05 (taps in N) launch: %s", cudaGetErrorString(e));
    note_kernel("bconv_wsx_kernel<%d> (tcgen05 kind::i8, column taps in N)", MT);
    return BNN_OK;
}

// the pooled layers' polyphase kernel (even H and W, no concat input)
template <int BN, int MT, int EW = BNN_POOL_EPI_WARPS>
static int launch_ws_pool(BconvParams p, int N, cudaStream_t st) {
    using Cfg = WsPoolCfg<BN, MT, EW>;
    if ((p.H & 1) || (p.W & 1) || p.cw1 != 0 || !p.fold2) return BNN_ERR_UNSUPPORTED;
    const long H2 = p.H / 2, W2 = p.W / 2;
    const long gk = std::max(1L, 64 / (W2 + 1));
    const long Gw = gk * (W2 + 1) + 1;
    const long rows = (long)cdiv(N, gk) * (H2 + 1) + 1;
    const long ptot = (rows - 2) * Gw;
    const long sp = ((Cfg::PI + 2 * Gw + 2) + 7) & ~7L;
    const long groups = (ptot + Cfg::PI - 1) / Cfg::PI;
    const long ncb = cdiv(p.Cout, BN);
    if (Gw > Cfg::MAX_GW || sp > Cfg::MAX_SP || groups * Cfg::PI + 2 * Gw + 2 >= (1L << 31) ||
        groups * ncb >= (1L << 31) || (size_t)N * p.H * p.W >= ((size_t)1 << 31))
        return BNN_ERR_UNSUPPORTED;
    const int ns = Cfg::stages((int)sp, (int)Gw, p.Cout);
    if (ns < 2) return BNN_ERR_UNSUPPORTED;
    p.gk = (int)gk; p.Gw = (int)Gw; p.HP = (int)sp;
    p.TR = (int)(groups * ncb); p.TC = (int)ncb; p.TNI = ns;
    const size_t smem = std::max<size_t>(
        (size_t)ns * Cfg::stage_bytes((int)sp) + Cfg::fixed_bytes((int)sp, (int)Gw, p.Cout), (size_t)116 * 1024);
    const int grid = (int)std::min<long>(groups * ncb, sm_count());
    cudaError_t e = launch_k(bconv_ws_pool_kernel<BN, MT, EW>, (unsigned)grid, Cfg::NT, smem, st, p);
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "bconv tcgen05 pooled launch: %s", cudaGetErrorString(e));
    note_kernel("bconv_ws_pool_kernel<%d,%d,%d> (tcgen05 kind::i8, polyphase 2x2 pool)", BN, MT, EW);
    return BNN_OK;
}

// below this many padded-grid positions (N*(H+1)*(W+1)) a layer runs in
// 32-channel blocks of 128-position items: a small batch then spreads over
// many CTAs instead of streaming the whole layer through one or two
constexpr long kSmallPositions = 16384;

static int launch_bconv(BconvParams p, int N, cudaStream_t st) {
    const bool tc = g_bconv_kind == 0 || g_bconv_kind >= 3;
    if (g_bconv_kind == 0 && p.wus && (long)N * (p.H + 1) * (p.W + 1) < kSmallPositions) {
        BconvParams q = p;
        q.wu = p.wus;
        q.ubn = 32;
        const int rc = p.out2 ? launch_ws_pool<32, 1>(q, N, st) : launch_ws<32, 1>(q, N, st);
        if (rc != BNN_ERR_UNSUPPORTED) return rc;
    }
    if (tc && p.out2 && p.wu) {
        int rc = BNN_ERR_UNSUPPORTED;
        switch (p.ubn) {
            case 32: rc = launch_ws_pool<32, 2>(p, N, st); break;
            // 10 producer warps at 64 channels (enc2.conv2 0.138 vs 0.155 ms); 6 at 32 and 128 (faster there)
            case 64: rc = launch_ws_pool<64, 1, 4>(p, N, st); break;
            case 128: rc = launch_ws_pool<128, 1>(p, N, st); break;
        }
        if (rc != BNN_ERR_UNSUPPORTED) return rc;
    }
    // e2m1 MMAs where they measured faster than int8 (4096 32x32 patches):
    // 64- and 128-channel layers with at least 2 input words (dec3.conv1
    // 0.084 vs 0.118 ms, dec2.conv1 0.131 vs 0.169, enc3.conv1 0.046 vs
    // 0.048, dec2.conv2 0.076 vs 0.077), 256-channel layers with at least 8,
    // in 128-channel blocks (dec4.conv1 0.103 vs 0.119, dec4.conv2 0.051 vs
    // 0.054, bott.conv2 0.056 vs 0.061); one input word (enc2.conv1 0.074 vs
    // 0.060) and the 32-channel layers (dec1.conv1 0.278 vs 0.209) stay int8;
    // kind 5 takes e2m1 for every non-pooled layer
    const bool f4 = (g_bconv_kind == 0 && (p.ubn == 64 || p.ubn == 128) && p.Kw >= 2) ||
                    (g_bconv_kind == 0 && p.ubn == 256 && p.Kw >= 8) || g_bconv_kind == 5;
    if (f4 && !p.out2 && p.w4) {
        int rc = BNN_ERR_UNSUPPORTED;
        switch (p.ubn) {
            case 32: rc = launch_ws<32, BNN_F4_MT32, true>(p, N, st); break;
            case 64:
                rc = p.cw1 > 0 ? launch_ws<64, BNN_F4_MT64, true, 4>(p, N, st) : launch_ws<64, BNN_F4_MT64, true>(p, N, st);
                break;
            case 128: rc = launch_ws<128, BNN_F4_MT128, true>(p, N, st); break;
            case 256: rc = launch_ws<128, BNN_F4_MT128, true>(p, N, st); break;  // 128-channel blocks
        }
        if (rc != BNN_ERR_UNSUPPORTED) return rc;
    }
    if (tc && !p.out2 && p.wu) {
        int rc = BNN_ERR_UNSUPPORTED;
        switch (p.ubn) {
            case 32:
                if (g_bconv_kind == 3) rc = launch_wsx<2>(p, N, st);
                // a decoder conv1 (concat input) stages two sources: 10 producer warps
                // (dec1.conv1 0.22 vs 0.27 ms); 6 elsewhere (4 epilogue warps measured slower there)
                if (rc == BNN_ERR_UNSUPPORTED)
                    rc = p.cw1 > 0 ? launch_ws<32, 8, false, 4>(p, N, st) : launch_ws<32, 8>(p, N, st);
                break;
            case 64: rc = launch_ws<64, 4>(p, N, st); break;
            case 128: rc = launch_ws<128, BNN_WS128_MT>(p, N, st); break;
            case 256: rc = launch_ws<256, BNN_WS256_MT>(p, N, st); break;
        }
        if (rc != BNN_ERR_UNSUPPORTED) return rc;
    }
    if (tc || g_bconv_kind == 2) {
        if (p.Cout <= 32) return launch_bmma<32>(p, N, st);
        if (p.Cout <= 64) return launch_bmma<64>(p, N, st);
        return launch_bmma<128>(p, N, st);
    }
    if (p.Cout <= 32) return launch_bconv_kc<32, 4, 4>(p, N, st);
    if (p.Cout <= 64) return launch_bconv_kc<64, 8, 4>(p, N, st);
    return launch_bconv_kc<128, 8, 8>(p, N, st);
}

// one binary conv layer of the forward
static int run_bin(const BinLayer& L, const uint32_t* in0, const uint32_t* in1, int h1, int w1, int N, int H,
                   int W, uint32_t* out, uint32_t* out2, int32_t* P, int32_t* P2, cudaStream_t st) {
    if (N <= 0 || H <= 0 || W <= 0) return BNN_OK;
    BconvParams p{};
    p.in0 = in0; p.in1 = in1; p.cw0 = L.cw0; p.cw1 = L.cw1; p.Kw = L.Kw;
    p.N = N; p.H = H; p.W = W;
    p.h1 = h1; p.w1 = w1;
    // reference up_cat (csrc/bnn_model.c:130-148): offset d/2 when the skip is larger
    const int upH = 2 * h1, upW = 2 * w1;
    p.oh = H > upH ? (H - upH) / 2 : 0;
    p.ow = W > upW ? (W - upW) / 2 : 0;
    p.cH = std::min(upH, H);
    p.cW = std::min(upW, W);
    p.Cin = L.Cin; p.Cout = L.Cout; p.cwo = cw_of(L.Cout);
    p.wt = L.wt; p.wpop = L.wpop; p.w8 = L.w8; p.CoutP = L.CoutP; p.fold = L.fold; p.fold2 = out2 ? L.fold2 : nullptr;
    p.wu = L.wu; p.ubn = L.ubn; p.wx = L.wx; p.w4 = L.w4; p.wus = L.wus;
    if ((g_bconv_kind != 1 && !L.w8) || (g_bconv_kind == 1 && (!L.wt || !L.wpop)) || !L.fold)
        return set_error(BNN_ERR_ARG, "binary conv layer has no weights for the selected kernel");
    p.out = out; p.out2 = out2; p.P = P; p.P2 = P2;
    return launch_bconv(p, N, st);
}

static int run_realin_exact(DevState* d, const Model* m, const float* x, int N, int H, int W, uint32_t* out,
                            float* dbg, cudaStream_t st) {
    if (N <= 0) return BNN_OK;
    RealinParams p{};
    p.x = x; p.wf = d->ri_wf; p.fold = d->ri_fold; p.out = out; p.dbg = dbg;
    p.N = N; p.Cin = m->enc_conv1[0].Cin; p.CinP = d->ri_CinP; p.CIP = d->ri_CIP;
    p.H = H; p.W = W; p.Cout = m->enc_conv1[0].Cout; p.cwo = cw_of(p.Cout);
    p.tiles_x = cdiv(W, RI_TC); p.tiles_y = cdiv(H, RI_TR);
    const size_t smem = (size_t)RI_HP * p.CIP * 4;
    cudaError_t e;
    dim3 grid((unsigned)((size_t)N * p.tiles_x * p.tiles_y), (unsigned)cdiv(p.Cout, 32));
    realin3x3_fold_kernel<<<grid, 128, smem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "realin launch: %s", cudaGetErrorString(e));
    return BNN_OK;
}

// e2 / T of realin_mma_kernel for a full window (the largest taps count):
// g(Cin-1) + g(8) * (1 + g(Cin-1)), g(n) = n u / (1 - n u), u = 2^-24,
// padded by 2^-30 relative and rounded up to float
static float first_conv_c9(int Cin) {
    const double u = std::ldexp(1.0, -24);
    auto g = [&](int n) { return n * u / (1.0 - n * u); };
    const double c = (g(Cin - 1) + g(8) * (1.0 + g(Cin - 1))) * (1.0 + std::ldexp(1.0, -30));
    float f = (float)c;
    if ((double)f < c) f = std::nextafter(f, 1.0f);
    return f;
}

// Coefficients of the tighter per-position bound of realin_ws_kernel. The
// reference sums a tap's bands sequentially (csrc/bnn_conv_realin.c:66-116):
// s_1 = y_1 exactly, s_k = fl(s_{k-1} + y_k), y = x*w exact (w = +-1 or 0),
// so its error is at most sum_{k>=2} u |s_{k-1} + y_k| with
// |s_{k-1} + y_k| <= (1 + gamma(n)) sum_{i<=k} |y_i|: at most
// u (1 + gamma(n)) sum_b (n - b)|x_b| over bands b = 0..n-1 (band b enters
// n - b of the partial sums at most). The nine tap sums add gamma(8) times
// sum_t |s_t| <= gamma(8) (1 + gamma(n)) sum_t sum_b |x_b|. Both rounded up,
// with the same 2^-30 margin as first_conv_c9.
static void first_conv_cab(int Cin, float* ca, float* cb) {
    const double u = std::ldexp(1.0, -24);
    auto g = [&](int n) { return n * u / (1.0 - n * u); };
    const double m = 1.0 + std::ldexp(1.0, -30);
    const double a = u * (1.0 + g(Cin)) * m, b = g(8) * (1.0 + g(Cin)) * m;
    float fa = (float)a, fb = (float)b;
    if ((double)fa < a) fa = std::nextafter(fa, 1.0f);
    if ((double)fb < b) fb = std::nextafter(fb, 1.0f);
    *ca = fa;
    *cb = fb;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependency on libcuda)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)f;
        cudaGetLastError();
    });
    return fn;
}

// input [N][C][H][W] f32 as a 4-D TMA map with a (bx, by, bc, 1) box
static bool first_conv_tmap(const float* x, int N, int C, int H, int W, CUtensorMap* tm, int bx = RM_BX,
                            int by = RM_BY, int bc = RM_BC) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn || (W % 4) != 0 || ((uintptr_t)x & 15)) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)C, (cuuint64_t)N};
    const cuuint64_t strides[3] = {(cuuint64_t)W * 4, (cuuint64_t)H * W * 4, (cuuint64_t)C * H * W * 4};
    const cuuint32_t box[4] = {(cuuint32_t)bx, (cuuint32_t)by, (cuuint32_t)bc, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D map over the flattened image (H*W, C, N) for realin_dxn_kernel: box
// (npos, 32, 1), an item's staged rows as one contiguous run per band
static bool first_conv_tmap3(const float* x, int N, int C, int H, int W, int npos, CUtensorMap* tm) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn || (W % 4) != 0 || ((uintptr_t)x & 15) || npos > 256) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)H * W, (cuuint64_t)C, (cuuint64_t)N};
    const cuuint64_t strides[2] = {(cuuint64_t)H * W * 4, (cuuint64_t)C * H * W * 4};
    const cuuint32_t box[3] = {(cuuint32_t)npos, 32, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)x, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool first_conv_fast_ok(const Model* m, int N, int H, int W) {
    return m->enc_conv1[0].Cin <= RM_CINP && (W % 4) == 0 && (size_t)N * H * W < ((size_t)1 << 31) &&
           encode_tiled() != nullptr;
}

// first conv implementation: 0 = tcgen05 realin_ws_kernel where the shape
// allows (default), 1 = mma.sync, 2 = tcgen05 realin_dxn_kernel (column taps
// in N) where W divides 32, realin_ws_kernel for other widths. Measured on
// 4096 32x32 patches: realin_ws 1.29 ms, realin_dxn 1.35 ms (with the fix-up).
static int g_first_kind = 0;

// realin_ws_kernel geometry for (H, W); false if the shape does not fit it
struct RwGeo {
    int R, Wp, SP, NS, NB;
    size_t smem;
};
// rmax: at most this many rows per item (a small batch takes short items, so
// that more CTAs share it)
#ifndef BNN_RW_RCAP
#define BNN_RW_RCAP (1 << 30)  // rows per first-conv item, at most (A/B builds)
#endif
static bool rw_geometry(int H, int W, RwGeo* g, int rmax = 1 << 30) {
    if ((W % 4) != 0 || W > RW_MT * 128 - 1) return false;
    g->Wp = W + 1;
    g->NB = RW_NB;
    // every output row inside the tiles
    g->R = std::min(std::min(H, rmax), std::min(BNN_RW_RCAP, (RW_MT * 128 - W) / g->Wp + 1));
    g->SP = rw_sp(W);
    if (g->R < 1 || g->SP > RW_MAX_SP || g->R + 2 > 256) return false;
    const size_t fixed = rw_fixed_bytes(W, g->R, g->SP);
    if (fixed + 2 * rw_stage_bytes(g->SP) > RW_MAX_SMEM) return false;
    g->NS = (int)std::min<size_t>(4, (RW_MAX_SMEM - fixed) / rw_stage_bytes(g->SP));
    g->smem = std::max<size_t>(fixed + (size_t)g->NS * rw_stage_bytes(g->SP), (size_t)116 * 1024);
    return true;
}

#ifndef BNN_RX_MINNS
#define BNN_RX_MINNS 2  // stages kept before input boxes are added
#endif
// realin_dxn_kernel geometry: W divides 32, an item = 128 / W whole rows;
// two stages, then as many input boxes as fit (5 at W = 32, 6 below), then
// stages again up to 4
static bool rx_geometry(int W, RwGeo* g) {
    if (W < 4 || W > 32 || (32 % W) != 0) return false;
    g->R = 128 / W;
    g->Wp = W;
    g->SP = rx_sp(W);
    const size_t stage = rx_stage_bytes(W);
    int nb = RX_MAXNB;
    while (nb > 2 && rx_fixed_bytes(W, nb) + BNN_RX_MINNS * stage > RW_MAX_SMEM) --nb;
    const size_t fixed = rx_fixed_bytes(W, nb);
    if (fixed + 2 * stage > RW_MAX_SMEM) return false;
    g->NB = nb;
    g->NS = (int)std::min<size_t>(4, (RW_MAX_SMEM - fixed) / stage);
    g->smem = std::max<size_t>(fixed + (size_t)g->NS * stage, (size_t)116 * 1024);
    return true;
}

// first conv -> bit plane: int8 tensor cores decided by the error bound, then
// the exact fix-up of undecided outputs (a memset and 2 kernels)
// realin_tx_kernel: R rows of R*Wp <= TX_TO outputs, one N = TX_N tile per item
static bool tx_geometry(int H, int W, RwGeo* g) {
    if ((W % 4) != 0) return false;
    g->Wp = W + 1;
    g->NB = RW_NB;
    g->R = std::min(H, TX_TO / g->Wp);
    g->SP = (2 * g->Wp + TX_N + 7) & ~7;
    if (g->R < 1 || g->SP > TX_MAX_SP) return false;
    const size_t fixed = tx_fixed_bytes(W, g->R, g->SP);
    if (fixed + 2 * tx_stage_bytes(g->SP) > TX_MAX_SMEM) return false;
    g->NS = (int)std::min<size_t>(4, (TX_MAX_SMEM - fixed) / tx_stage_bytes(g->SP));
    g->smem = std::max<size_t>(fixed + (size_t)g->NS * tx_stage_bytes(g->SP), (size_t)116 * 1024);
    return true;
}

// fix-up grid: one warp per 16 pixels of the batch, at most 8 blocks per SM
// (the kernel strides over its list; a small batch needs few blocks)
static unsigned fixup_blocks(int N, int H, int W) {
    const long px = (long)N * H * W;
    return (unsigned)std::max<long>(1, std::min<long>(148 * 8, (px + 16 * FIX_WARPS - 1) / (16 * FIX_WARPS)));
}

static int run_realin_fast(DevState* d, const Model* m, const float* x, int N, int H, int W, uint32_t* out,
                           cudaStream_t st) {
    if (N <= 0) return BNN_OK;
    Arena& a = d->ar;
    CUtensorMap tm;
    RwGeo geo{};
    const int Cin = m->enc_conv1[0].Cin, Cout = m->enc_conv1[0].Cout;
    const bool dxn = g_first_kind == 2 && d->rx_wu && rx_geometry(W, &geo);
    const bool tx = !dxn && g_first_kind == 3 && d->rx_wu && tx_geometry(H, W, &geo);
    // rows per item: as many as the tiles hold, fewer when that leaves most SMs idle
    const int rmax = std::max(1, cdiv((long)N * H, std::max(1, sm_count() / 2)));
    if (g_first_kind != 1 && d->rw_wu && d->rw_thr.size() == 32 && Cout <= 32 && Cin <= RM_CINP &&
        (dxn || tx || rw_geometry(H, W, &geo, rmax)) &&
        (dxn ? first_conv_tmap3(x, N, Cin, H, W, rx_npos(W), &tm) : first_conv_tmap(x, N, Cin, H, W, &tm, W, geo.R + 2, 32))) {
        CK(cudaMemsetAsync(a.rm_ctl, 0, 3 * sizeof(unsigned int), st));
        RealinWsParams p{};
        p.wu = (dxn || tx) ? d->rx_wu : d->rw_wu; p.out = out;
        for (int c = 0; c < 32; ++c) {
            p.thrC[c] = d->rw_thr[c].C;
            p.thr_neg |= (uint32_t)(d->rw_thr[c].sgn < 0) << c;
            p.thr_exact |= (uint32_t)(d->rw_thr[c].exact != 0) << c;
            // realin_ws_kernel's plane 0 carries +64 per element (every staged
            // position, padding included): its sums exceed the exact ones by
            // 64 * 2^16 * (the channel's weight sum), for the fold's test on Q or -Q
            if (BNN_RW_UP0 && !dxn && !tx)
                p.thrC[c] += (d->rw_thr[c].sgn < 0 ? -1 : 1) * (d->rw_wsum[c] << 22);
        }
        p.list = a.rm_list; p.ctl = a.rm_ctl; p.cap = a.rm_cap;
        p.N = N; p.Cin = Cin; p.H = H; p.W = W; p.Cout = Cout; p.cwo = cw_of(Cout);
        p.R = geo.R; p.Wp = geo.Wp; p.SP = geo.SP; p.NS = geo.NS; p.NB = geo.NB; p.KC = cdiv(Cin, 32);
        p.ipi = cdiv(H, geo.R);
        p.n_items = N * p.ipi;
        p.c9 = first_conv_c9(Cin);
        first_conv_cab(Cin, &p.ca, &p.cb);
        const int grid = std::min(p.n_items, sm_count());
        cudaError_t e;
        if (dxn) {
            realin_dxn_kernel<<<grid, RX_NT, geo.smem, st>>>(tm, p);
            e = cudaGetLastError();
        } else if (tx) {
            realin_tx_kernel<<<grid, TX_NT, geo.smem, st>>>(tm, p);
            e = cudaGetLastError();
        } else if (W == 32 && geo.R == 7) {  // the benchmark's 32-wide patches in 7-row items: geometry compiled in
            e = launch_k(realin_ws_kernel<32, 7>, (unsigned)grid, RW_NT, geo.smem, st, tm, p);
        } else {
            e = launch_k(realin_ws_kernel<0, 0>, (unsigned)grid, RW_NT, geo.smem, st, tm, p);
        }
        if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "realin tcgen05 launch: %s", cudaGetErrorString(e));
        RealinFixParams f{x, d->ri_wf, d->ri_fold, out, a.rm_list, a.rm_ctl, a.rm_cap, N, Cin, d->ri_CinP, H, W,
                          Cout, p.cwo};
        e = launch_k(realin_fixup_kernel, (unsigned)fixup_blocks(N, H, W), FIX_WARPS * 32, 0, st, f);
        if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "realin fixup launch: %s", cudaGetErrorString(e));
        return BNN_OK;
    }
    if (!first_conv_tmap(x, N, m->enc_conv1[0].Cin, H, W, &tm))
        return run_realin_exact(d, m, x, N, H, W, out, nullptr, st);
    CK(cudaMemsetAsync(a.rm_ctl, 0, 3 * sizeof(unsigned int), st));
    RealinMmaParams p{};
    p.wfrag = d->rm_wfrag; p.fold = d->ri_fold; p.exact_ch = d->rm_exact; p.out = out;
    p.list = a.rm_list; p.ctl = a.rm_ctl; p.cap = a.rm_cap;
    p.N = N; p.Cin = m->enc_conv1[0].Cin; p.H = H; p.W = W; p.Cout = m->enc_conv1[0].Cout; p.cwo = cw_of(p.Cout);
    p.tiles_x = cdiv(W, RM_TC); p.tiles_y = cdiv(H, RM_TR);
    p.c9 = first_conv_c9(p.Cin);
    dim3 grid((unsigned)((size_t)N * p.tiles_x * p.tiles_y), (unsigned)cdiv(p.Cout, 32));
    realin_mma_kernel<<<grid, 256, RM_SMEM, st>>>(tm, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "realin mma launch: %s", cudaGetErrorString(e));
    RealinFixParams f{x, d->ri_wf, d->ri_fold, out, a.rm_list, a.rm_ctl, a.rm_cap, N, p.Cin, d->ri_CinP, H, W,
                      p.Cout, p.cwo};
    realin_fixup_kernel<<<fixup_blocks(N, H, W), FIX_WARPS * 32, 0, st>>>(f);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "realin fixup launch: %s", cudaGetErrorString(e));
    return BNN_OK;
}

static int run_first_conv(DevState* d, const Model* m, const float* x, int N, int H, int W, uint32_t* out,
                          cudaStream_t st) {
    if (first_conv_fast_ok(m, N, H, W)) return run_realin_fast(d, m, x, N, H, W, out, st);
    return run_realin_exact(d, m, x, N, H, W, out, nullptr, st);
}

// v2 stem: bands -> bit plane [N][H][W][cw(stem_c)]; dbg (optional) gets
// the conv output alpha*acc as [N][stem_c][H][W]
static int run_stem(DevState* d, const Model* m, const float* x, int N, int H, int W, uint32_t* out, float* dbg,
                    cudaStream_t st) {
    if (N <= 0) return BNN_OK;
    const Engine* E = eng(m);
    StemParams p{};
    p.x = x; p.w = d->st_w; p.fold = d->st_fold; p.out = out; p.dbg = dbg;
    p.Cin = E->stem_conv.Cin; p.HW = H * W; p.Cout = E->stem_c; p.cwo = cw_of(p.Cout);
    const int CB = d->st_CB;
    const uintptr_t xa = (uintptr_t)x;
    // default (measured on B200, 4096 patches of 32x32x120): stems up to 16
    // channels run the register-streamed kernel (8 ch: 0.33 ms = 92% of HBM;
    // 16 ch: 0.44 ms), wider ones the bulk-copy kernel (32 ch: 0.93 ms vs
    // 1.25 ms) where rows are 16-byte aligned and its ring fits;
    // set_first_conv_kernel(1) swaps the two
    const bool want_bulk = (CB == 32) == (g_first_kind != 1);
    {
        const int PXb = CB == 32 ? 2 : 4;
        const int nst = sb_stages(p.Cin, CB, PXb);
        const long long pixels = (long long)N * p.HW;
        const long long items = (pixels + SB_NC * PXb - 1) / (SB_NC * PXb);
        if (want_bulk && p.HW % 4 == 0 && p.HW >= 256 && xa % 16 == 0 && nst >= 2 && items < (1ll << 31)) {
            p.groups = pixels / 4;
            const size_t smem = (size_t)sb_wbytes(p.Cin, CB) + (size_t)nst * sb_stage_bytes(PXb) + 2 * SB_MAXST * 8;
            const dim3 grid((unsigned)std::min<long long>(items, sm_count()), (unsigned)d->st_slices);
            if (CB == 8) stem_bulk_kernel<8, 4><<<grid, SB_NT, smem, st>>>(p, (int)items, nst);
            else if (CB == 16) stem_bulk_kernel<16, 4><<<grid, SB_NT, smem, st>>>(p, (int)items, nst);
            else stem_bulk_kernel<32, 2><<<grid, SB_NT, smem, st>>>(p, (int)items, nst);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "stem launch: %s", cudaGetErrorString(e));
            return BNN_OK;
        }
    }
    // PX pixels per thread: they share one patch (PX | H*W) and one aligned
    // vector load; at most 64 accumulators per thread
    int PX = (p.HW % 4 == 0 && xa % 16 == 0) ? 4 : (p.HW % 2 == 0 && xa % 8 == 0) ? 2 : 1;
    if (CB == 32 && PX == 4) PX = 2;
    p.groups = (long long)N * p.HW / PX;
    const size_t smem = (size_t)p.Cin * CB * 4;
    const dim3 grid((unsigned)cdiv(p.groups, 256), (unsigned)d->st_slices);
#define STEM_LAUNCH(cb, px) stem_fold_kernel<cb, px><<<grid, 256, smem, st>>>(p)
    if (CB == 8) { if (PX == 4) STEM_LAUNCH(8, 4); else if (PX == 2) STEM_LAUNCH(8, 2); else STEM_LAUNCH(8, 1); }
    else if (CB == 16) { if (PX == 4) STEM_LAUNCH(16, 4); else if (PX == 2) STEM_LAUNCH(16, 2); else STEM_LAUNCH(16, 1); }
    else { if (PX == 2) STEM_LAUNCH(32, 2); else STEM_LAUNCH(32, 1); }
#undef STEM_LAUNCH
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "stem launch: %s", cudaGetErrorString(e));
    return BNN_OK;
}

static int run_head(DevState* d, const Model* m, const uint32_t* in, int N, int H, int W, float* out,
                    cudaStream_t st) {
    if (N <= 0) return BNN_OK;
    HeadParams p{in, d->head_W, d->head_b, out, N, H, W, m->head_Cin, cw_of(m->head_Cin), m->head_Cout};
    const size_t total = (size_t)N * H * W;
    if (total >= ((size_t)1 << 31)) return set_error(BNN_ERR_ARG, "N*H*W = %zu: at most 2^31 - 1 pixels", total);
    unsigned blocks = (unsigned)std::max<size_t>(1, std::min<size_t>((total + 511) / 512, 148 * 8));
    const cudaError_t e = p.Cin == 32 && p.ncls == 3
                              ? launch_k(head1x1_c32_kernel<3>, blocks, 256, 0, st, p)  // weights in registers
                              : launch_k(head1x1_kernel, blocks, 256, 0, st, p);
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "head launch: %s", cudaGetErrorString(e));
    return BNN_OK;
}

// -------------------------------------------------------------------
// the forward: 19 launches in the reference's order (+1 for the first conv's
// fix-up; a v2 model: stem, 18 binary convs, head)
// -------------------------------------------------------------------
struct Dbg {  // optional debug outputs of one forward (device pointers)
    float* realin = nullptr;
    uint32_t* realin_bits = nullptr;  // scratch for the exact kernel that produces `realin`
    int32_t* P[18] = {nullptr};     // binary convs' P in forward order (18 with a v2 stem)
    int32_t* Pd[4] = {nullptr};
};

struct ProfCtx {
    Profiler* prof = nullptr;
    cudaStream_t st = nullptr;
    std::vector<std::tuple<std::string, const char*, double, cudaEvent_t, cudaEvent_t>> marks;
    cudaEvent_t last = nullptr;
    void begin(const std::string& label, const char* optype, double work) {
        if (!prof) return;
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, st);
        marks.emplace_back(label, optype, work, a, b);
    }
    void end() {
        if (!prof) return;
        cudaEventRecord(std::get<4>(marks.back()), st);
    }
    int finish() {
        if (!prof) return BNN_OK;
        CK(cudaStreamSynchronize(st));
        for (auto& mk : marks) {
            float ms = 0;
            cudaEventElapsedTime(&ms, std::get<3>(mk), std::get<4>(mk));
            prof->add(std::get<0>(mk), std::get<1>(mk), std::get<2>(mk), ms);
            cudaEventDestroy(std::get<3>(mk));
            cudaEventDestroy(std::get<4>(mk));
        }
        marks.clear();
        return BNN_OK;
    }
};

static int forward_launches(const Model* m, DevState* d, const float* x, int N, int H, int W, float* logits,
                            cudaStream_t st, const Dbg* dbg, ProfCtx* pc) {
    // small batches: dependent launches (the flag is reset on every return)
    struct PdlScope {
        explicit PdlScope(bool on) { t_pdl = on; }
        ~PdlScope() { t_pdl = false; }
    } pdl_scope(pdl_enabled() && (double)N * H * W <= kPdlPixels);
    static const char* EN[4] = {"enc1", "enc2", "enc3", "enc4"};
    static const char* DN[4] = {"dec4", "dec3", "dec2", "dec1"};
    Arena& a = d->ar;
    int rc;
    const double NHW = (double)N * H * W;
    auto work = [&](const BinLayer& L, int h, int w) { return (double)N * h * w * L.Cout * (double)L.Cin * 9.0; };
    int li = 0;
    const Engine* E = eng(m);
    if (E->stem_c) {
        // v2: stem (exact fp32 order in the production kernel itself), then
        // enc1.conv1 binary like the other levels
        if (pc) pc->begin("stem.conv+act", "conv_real", NHW * E->stem_c * E->stem_conv.Cin);
        rc = run_stem(d, m, x, N, H, W, a.stem, dbg ? dbg->realin : nullptr, st);
        if (pc) pc->end();
        if (rc) return rc;
        if (pc) pc->begin("enc1.conv1+act1", "bconv", work(d->enc1[0], H, W));
        rc = run_bin(d->enc1[0], a.stem, nullptr, 0, 0, N, H, W, a.enc_h[0], nullptr, dbg ? dbg->P[li] : nullptr,
                     nullptr, st);
        if (pc) pc->end();
        if (rc) return rc;
        ++li;
    } else {
        if (pc) pc->begin("enc1.conv1+act1", "conv_real", NHW * m->enc_conv1[0].Cout * m->enc_conv1[0].Cin * 9.0);
        // the stage dump's float output of the first conv comes from the exact
        // kernel; the bit plane used downstream is always the production path's
        if (dbg && dbg->realin) rc = run_realin_exact(d, m, x, N, H, W, dbg->realin_bits, dbg->realin, st);
        else rc = BNN_OK;
        if (!rc) rc = run_first_conv(d, m, x, N, H, W, a.enc_h[0], st);
        if (pc) pc->end();
        if (rc) return rc;
    }
    for (int i = 0; i < 4; ++i) {
        const int h = H >> i, w = W >> i;
        if (i > 0) {
            if (pc) pc->begin(std::string(EN[i]) + ".conv1+act1", "bconv", work(d->enc1[i], h, w));
            rc = run_bin(d->enc1[i], a.down[i - 1], nullptr, 0, 0, N, h, w, a.enc_h[i], nullptr,
                         dbg ? dbg->P[li] : nullptr, nullptr, st);
            if (pc) pc->end();
            if (rc) return rc;
            ++li;
        }
        if (pc) pc->begin(std::string(EN[i]) + ".conv2+skip+pool+down", "bconv", work(d->enc2[i], h, w));
        rc = run_bin(d->enc2[i], a.enc_h[i], nullptr, 0, 0, N, h, w, a.skip[i], a.down[i],
                     dbg ? dbg->P[li] : nullptr, dbg ? dbg->Pd[i] : nullptr, st);
        if (pc) pc->end();
        if (rc) return rc;
        ++li;
    }
    const int h4 = H >> 4, w4 = W >> 4;
    if (pc) pc->begin("bott.conv1+act1", "bconv", work(d->bott1, h4, w4));
    rc = run_bin(d->bott1, a.down[3], nullptr, 0, 0, N, h4, w4, a.bott_h, nullptr, dbg ? dbg->P[li] : nullptr,
                 nullptr, st);
    if (pc) pc->end();
    if (rc) return rc;
    ++li;
    if (pc) pc->begin("bott.conv2+act2", "bconv", work(d->bott2, h4, w4));
    rc = run_bin(d->bott2, a.bott_h, nullptr, 0, 0, N, h4, w4, a.bott_x, nullptr, dbg ? dbg->P[li] : nullptr,
                 nullptr, st);
    if (pc) pc->end();
    if (rc) return rc;
    ++li;
    const uint32_t* xprev = a.bott_x;
    int hp = h4, wp = w4;
    for (int i = 0; i < 4; ++i) {
        const int l = 3 - i, h = H >> l, w = W >> l;
        if (pc) pc->begin(std::string(DN[i]) + ".upcat+conv1+act1", "bconv", work(d->dec1[i], h, w));
        rc = run_bin(d->dec1[i], a.skip[l], xprev, hp, wp, N, h, w, a.dec_h[i], nullptr,
                     dbg ? dbg->P[li] : nullptr, nullptr, st);
        if (pc) pc->end();
        if (rc) return rc;
        ++li;
        if (pc) pc->begin(std::string(DN[i]) + ".conv2+act2", "bconv", work(d->dec2[i], h, w));
        rc = run_bin(d->dec2[i], a.dec_h[i], nullptr, 0, 0, N, h, w, a.dec_x[i], nullptr,
                     dbg ? dbg->P[li] : nullptr, nullptr, st);
        if (pc) pc->end();
        if (rc) return rc;
        ++li;
        xprev = a.dec_x[i];
        hp = h; wp = w;
    }
    if (pc) pc->begin("head", "head", NHW * m->head_Cout * m->head_Cin);
    rc = run_head(d, m, a.dec_x[3], N, H, W, logits, st);
    if (pc) pc->end();
    return rc;
}

static int check_hw(int N, int H, int W) {
    if (N < 0) return set_error(BNN_ERR_ARG, "N = %d", N);
    // below 16 an encoder level is one pixel wide, where the reference's
    // maxpool_P writes past its H/2 = 0 output (bnn_maxpool.c:29-30): the
    // reference has no defined result there, so it is refused here.
    if (H < 16 || W < 16) return set_error(BNN_ERR_ARG, "H=%d W=%d: the v1 forward needs H, W >= 16", H, W);
    if ((size_t)H * W > ((size_t)1 << 28)) return set_error(BNN_ERR_ARG, "H*W too large");
    return BNN_OK;
}

// forward on device buffers; graph replay unless profiling / debugging
static int forward_device(const Model* m, DevState* d, const float* x, int N, int H, int W, float* logits,
                          cudaStream_t user, const Dbg* dbg) {
    int rc = arena_reserve(m, d, N, H, W);
    if (rc) return rc;
    Engine* E = (Engine*)m->engine;
    if (N == 0) return BNN_OK;
    // the activation arena is shared by every forward on this device: work
    // enqueued on different streams is ordered through ev_last
    CK(cudaStreamWaitEvent(user, d->ev_last, 0));
    if ((rc = poison_arena(d->ar.base, d->ar.bytes, user))) return rc;
    if (E->prof.on || dbg) {
        ProfCtx pc;
        ProfCtx* ppc = nullptr;
        if (E->prof.on) { pc.prof = &E->prof; pc.st = user; ppc = &pc; }
        rc = forward_launches(m, d, x, N, H, W, logits, user, dbg, ppc);
        if (rc) return rc;
        CK(cudaEventRecord(d->ev_last, user));
        return ppc ? ppc->finish() : BNN_OK;
    }
    GraphKey key{N, H, W, x, logits};
    auto it = d->graphs.find(key);
    if (it == d->graphs.end()) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(d->cs, cudaStreamCaptureModeThreadLocal));
        rc = forward_launches(m, d, x, N, H, W, logits, d->cs, nullptr, nullptr);
        cudaError_t e = cudaStreamEndCapture(d->cs, &g);
        if (rc) { if (g) cudaGraphDestroy(g); return rc; }
        if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
        if (d->graphs.size() > 64) {
            for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
            d->graphs.clear();
        }
        it = d->graphs.emplace(key, ex).first;
    }
    CK(cudaGraphLaunch(it->second, user));
    CK(cudaEventRecord(d->ev_last, user));
    return BNN_OK;
}

static int current_device(int* dev) {
    if (cudaGetDevice(dev) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_CUDA, "no CUDA device available");
    }
    return BNN_OK;
}

// Bounded device waits that gave up during a synchronous call. The device
// counter (g_bnn_wait_timeouts) is read on the call's stream before its
// first launch (slot 0) and after its last (slot 1) into pinned host words:
// no extra synchronisation, and work queued by other calls before this one
// is not counted against it.
static int wait_mark(DevState* d, cudaStream_t s, int slot) {
    CK(cudaMemcpyFromSymbolAsync(&d->wt_host[slot], g_bnn_wait_timeouts, sizeof(unsigned int), 0,
                                 cudaMemcpyDeviceToHost, s));
    return BNN_OK;
}
// test hook (BNN_FAULT_WAIT): a wait that gives up, queued on stream s
static int inject_wait(cudaStream_t s) {
    if (g_fail_wait.exchange(0) == 0) return BNN_OK;
    wait_probe_kernel<<<1, 1, 0, s>>>(1 << 12, nullptr);
    CK(cudaGetLastError());
    return BNN_OK;
}
// once the stream that carried both marks has been synchronised
static int wait_verdict(const DevState* d) {
    const unsigned int n = d->wt_host[1] - d->wt_host[0];
    if (n)
        return set_error(BNN_ERR_CUDA,
                         "%u bounded device wait(s) gave up on device %d during this call: its outputs are not valid",
                         n, d->device);
    return BNN_OK;
}

// pipelined host batch on one device: chunks of `chunk` patches, H2D of the
// next chunk and D2H of the previous one overlap the current forward
static int host_batch_on(const Model* m, int device, const float* in, int N, int H, int W, float* out, int chunk) {
    CK(cudaSetDevice(device));
    DevState* d = nullptr;
    int rc = get_dev(m, device, &d);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(d->mu);
    const size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    const int C = std::max(1, std::min(chunk, N));
    if (d->pcap < (size_t)C || d->pbands != m->n_bands || d->pclasses != m->n_classes || d->pH != H || d->pW != W) {
        CK(cudaDeviceSynchronize());
        for (int s = 0; s < 2; ++s) {
            cudaFree(d->pin[s]); cudaFree(d->pout[s]);
            d->pin[s] = d->pout[s] = nullptr;
        }
        d->pcap = 0;
        for (int s = 0; s < 2; ++s) {
            if (dev_malloc(&d->pin[s], (size_t)C * ip * 4) != cudaSuccess ||
                dev_malloc(&d->pout[s], (size_t)C * op * 4) != cudaSuccess) {
                cudaGetLastError();
                return set_error(BNN_ERR_OOM, "cudaMalloc staging (%d patches)", C);
            }
        }
        d->pcap = (size_t)C; d->pbands = m->n_bands; d->pclasses = m->n_classes; d->pH = H; d->pW = W;
    }
    const int nch = cdiv(N, C);
    // on an error after work was queued, let the queued copies finish before
    // returning: the caller may release its host buffers at once
    struct Drain {
        DevState* d;
        bool armed = true;
        ~Drain() {
            if (!armed) return;
            cudaStreamSynchronize(d->h2d);
            cudaStreamSynchronize(d->cs);
            cudaStreamSynchronize(d->d2h);
            cudaGetLastError();
        }
    } drain{d};
    if ((rc = wait_mark(d, d->cs, 0))) return rc;
    for (int k = 0; k < nch; ++k) {
        const int s = k & 1;
        const int lo = k * C, n = std::min(C, N - lo);
        if (k >= 2) CK(cudaStreamWaitEvent(d->h2d, d->ev_comp[s], 0));  // slot free for input
        CK(cudaMemcpyAsync(d->pin[s], in + (size_t)lo * ip, (size_t)n * ip * 4, cudaMemcpyHostToDevice, d->h2d));
        CK(cudaEventRecord(d->ev_in[s], d->h2d));
        CK(cudaStreamWaitEvent(d->cs, d->ev_in[s], 0));
        if (k >= 2) CK(cudaStreamWaitEvent(d->cs, d->ev_out[s], 0));  // output slot drained
        rc = forward_device(m, d, d->pin[s], n, H, W, d->pout[s], d->cs, nullptr);
        if (rc) return rc;
        CK(cudaEventRecord(d->ev_comp[s], d->cs));
        CK(cudaStreamWaitEvent(d->d2h, d->ev_comp[s], 0));
        CK(cudaMemcpyAsync(out + (size_t)lo * op, d->pout[s], (size_t)n * op * 4, cudaMemcpyDeviceToHost, d->d2h));
        CK(cudaEventRecord(d->ev_out[s], d->d2h));
    }
    if ((rc = inject_wait(d->cs)) || (rc = wait_mark(d, d->cs, 1))) return rc;
    drain.armed = false;
    CK(cudaStreamSynchronize(d->d2h));
    CK(cudaStreamSynchronize(d->cs));
    return wait_verdict(d);
}

// device buffer of at least `n` floats, kept in *buf / *cap across calls
static int grow(float** buf, size_t* cap, size_t n, const char* what) {
    if (*cap >= n) return BNN_OK;
    cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    if (dev_malloc(buf, n * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_OOM, "cudaMalloc %s (%zu bytes)", what, n * sizeof(float));
    }
    *cap = n;
    return BNN_OK;
}

// tiles per forward of the patched path
static constexpr int kSceneChunk = 4096;

// Patched forward of a [bands][H][W] scene on device d: chunks of PxP tiles
// gathered from the cube, the batched forward (graph replay), the in-scene
// part of their logits stitched into [classes][H][W]. Called with d->mu held.
static int scene_device(const Model* m, DevState* d, const float* cube, int H, int W, int P, float* logits,
                        cudaStream_t st) {
    const int tx = cdiv(W, P), ty = cdiv(H, P), nt = tx * ty;
    const int C = std::min(nt, kSceneChunk);
    const size_t in_per = (size_t)m->n_bands * P * P, out_per = (size_t)m->n_classes * P * P;
    int rc;
    if ((rc = grow(&d->tin, &d->tcap, (size_t)C * in_per, "scene tiles"))) return rc;
    if ((rc = grow(&d->tout, &d->tcap_out, (size_t)C * out_per, "scene tile logits"))) return rc;
    for (int t0 = 0; t0 < nt; t0 += C) {
        const int n = std::min(C, nt - t0);
        const size_t gin = (size_t)n * m->n_bands * P * (((W | P) & 3) == 0 ? P / 4 : P);
        tile_gather_kernel<<<(unsigned)std::min<size_t>((gin + 255) / 256, 148 * 32), 256, 0, st>>>(
            cube, m->n_bands, H, W, P, tx, t0, n, d->tin);
        CK(cudaGetLastError());
        if ((rc = forward_device(m, d, d->tin, n, P, P, d->tout, st, nullptr))) return rc;
        const size_t gout = (size_t)n * m->n_classes * P * (((W | P) & 3) == 0 ? P / 4 : P);
        tile_stitch_kernel<<<(unsigned)std::min<size_t>((gout + 255) / 256, 148 * 32), 256, 0, st>>>(
            d->tout, m->n_classes, H, W, P, tx, t0, n, logits);
        CK(cudaGetLastError());
    }
    return BNN_OK;
}

// patched forward of scene rows [y0, y1) of a host cube on one device: the
// slab in (one strided copy), scene_device, the logits slab out
static int scene_host_on(const Model* m, int device, const float* in, int H, int W, int y0, int y1, int P,
                         float* out) {
    CK(cudaSetDevice(device));
    DevState* d = nullptr;
    int rc = get_dev(m, device, &d);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(d->mu);
    const int Hs = y1 - y0;
    const size_t plane = (size_t)Hs * W;
    if ((rc = grow(&d->scube, &d->scube_cap, (size_t)m->n_bands * plane, "scene slab"))) return rc;
    if ((rc = grow(&d->slog, &d->slog_cap, (size_t)m->n_classes * plane, "scene logits"))) return rc;
    if ((rc = wait_mark(d, d->cs, 0))) return rc;
    CK(cudaMemcpy2DAsync(d->scube, plane * 4, in + (size_t)y0 * W, (size_t)H * W * 4, plane * 4, m->n_bands,
                         cudaMemcpyHostToDevice, d->cs));
    if ((rc = scene_device(m, d, d->scube, Hs, W, P, d->slog, d->cs))) return rc;
    CK(cudaMemcpy2DAsync(out + (size_t)y0 * W, (size_t)H * W * 4, d->slog, plane * 4, plane * 4, m->n_classes,
                         cudaMemcpyDeviceToHost, d->cs));
    if ((rc = inject_wait(d->cs)) || (rc = wait_mark(d, d->cs, 1))) return rc;
    CK(cudaStreamSynchronize(d->cs));
    return wait_verdict(d);
}

}  // namespace bnn

using namespace bnn;

// ===================================================================
// C ABI
// ===================================================================
BNN_API int bnn_forward_device(const Model* m, int device, const float* d_input, int N, int H, int W,
                               float* d_logits, void* stream) {
    if (!m) return set_error(BNN_ERR_ARG, "model is NULL");
    int rc = check_hw(N, H, W);
    if (rc) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_ARG, "cannot select device %d", device);
    }
    DevState* d = nullptr;
    rc = get_dev(m, device, &d);
    if (!rc) {
        std::lock_guard<std::mutex> g(d->mu);
        rc = forward_device(m, d, d_input, N, H, W, d_logits, (cudaStream_t)stream, nullptr);
    }
    cudaSetDevice(prev);
    return rc;
}

BNN_API int bnn_forward_batch(const Model* m, const float* input, int N, int H, int W, float* logits) {
    if (!m || (!input && N > 0) || (!logits && N > 0)) return set_error(BNN_ERR_ARG, "NULL argument");
    int rc = check_hw(N, H, W);
    if (rc) return rc;
    if (N == 0) return BNN_OK;
    Engine* E = (Engine*)m->engine;
    std::vector<int> devs;
    {
        std::lock_guard<std::mutex> g(E->mu);
        devs = E->devices;
    }
    int prev = 0;
    if (devs.empty()) {
        if ((rc = current_device(&prev))) return rc;
        devs.push_back(prev);
    } else {
        cudaGetDevice(&prev);
    }
    const size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    const int nd = (int)devs.size();
    if (nd == 1) {
        rc = host_batch_on(m, devs[0], input, N, H, W, logits, E->chunk);
        cudaSetDevice(prev);
        return rc;
    }
    std::vector<int> st(nd, BNN_OK);
    std::vector<std::string> msg(nd);
    std::vector<std::thread> th;
    const int fail = g_fail_shard.exchange(-1);  // test hook (BNN_FAULT_SHARD)
    for (int r = 0; r < nd; ++r) {
        const int lo = (int)((long)N * r / nd), hi = (int)((long)N * (r + 1) / nd);
        th.emplace_back([&, r, lo, hi]() {
            if (r == fail)
                st[r] = set_error(BNN_ERR_CUDA, "shard %d: injected host-thread failure", r);
            else if (hi > lo)
                st[r] = host_batch_on(m, devs[r], input + (size_t)lo * ip, hi - lo, H, W, logits + (size_t)lo * op,
                                      E->chunk);
            if (st[r]) msg[r] = bnn_last_error();
        });
    }
    for (auto& t : th) t.join();
    cudaSetDevice(prev);
    for (int r = 0; r < nd; ++r)
        if (st[r]) return set_error(st[r], "device %d: %s", devs[r], msg[r].c_str());
    return BNN_OK;
}

BNN_API int bnn_forward_patched(const Model* m, const float* input, int H, int W, float* logits, int P) {
    if (!m || !input || !logits) return set_error(BNN_ERR_ARG, "NULL argument");
    if (H <= 0 || W <= 0) return set_error(BNN_ERR_ARG, "scene %dx%d", H, W);
    int rc = check_hw(1, P, P);  // every tile is a PxP forward
    if (rc) return rc;
    Engine* E = (Engine*)m->engine;
    std::vector<int> devs;
    {
        std::lock_guard<std::mutex> g(E->mu);
        devs = E->devices;
    }
    int prev = 0;
    if (devs.empty()) {
        if ((rc = current_device(&prev))) return rc;
        devs.push_back(prev);
    } else {
        cudaGetDevice(&prev);
    }
    const int ty = cdiv(H, P), nd = std::min((int)devs.size(), ty);
    std::vector<int> st(nd, BNN_OK);
    std::vector<std::string> msg(nd);
    std::vector<std::thread> th;
    for (int r = 0; r < nd; ++r) {
        const int r0 = (int)((long)ty * r / nd), r1 = (int)((long)ty * (r + 1) / nd);
        auto job = [&, r, r0, r1]() {
            st[r] = scene_host_on(m, devs[r], input, H, W, r0 * P, std::min(r1 * P, H), P, logits);
            if (st[r]) msg[r] = bnn_last_error();
        };
        if (nd == 1) job();
        else th.emplace_back(job);
    }
    for (auto& t : th) t.join();
    cudaSetDevice(prev);
    for (int r = 0; r < nd; ++r)
        if (st[r]) return nd == 1 ? st[r] : set_error(st[r], "device %d: %s", devs[r], msg[r].c_str());
    return BNN_OK;
}

BNN_API int bnn_forward_patched_device(const Model* m, int device, const float* d_cube, int H, int W, int P,
                                       float* d_logits, void* stream) {
    if (!m || !d_cube || !d_logits) return set_error(BNN_ERR_ARG, "NULL argument");
    if (H <= 0 || W <= 0) return set_error(BNN_ERR_ARG, "scene %dx%d", H, W);
    int rc = check_hw(1, P, P);
    if (rc) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_ARG, "cannot select device %d", device);
    }
    DevState* d = nullptr;
    rc = get_dev(m, device, &d);
    if (!rc) {
        std::lock_guard<std::mutex> g(d->mu);
        rc = scene_device(m, d, d_cube, H, W, P, d_logits, (cudaStream_t)stream);
    }
    cudaSetDevice(prev);
    return rc;
}

BNN_API void bnn_forward(const Model* m, const float* input, int H, int W, float* logits) {
    int dev = 0;
    int rc = current_device(&dev);
    if (!rc) rc = check_hw(1, H, W);
    if (!rc) rc = host_batch_on(m, dev, input, 1, H, W, logits, 1);
    if (rc) {
        fprintf(stderr, "%s\n", bnn_last_error());
        exit(1);
    }
}

BNN_API int bnn_set_bconv_kernel(int kind) {
    if (kind < 0 || kind > 5)
        return set_error(BNN_ERR_ARG,
                         "bconv kernel kind %d (0 = tcgen05 int8 + e2m1 where faster, 1 = popc, 2 = mma.sync, "
                         "3 = tcgen05 int8 with the column taps in N at 32 channels, 4 = tcgen05 int8, "
                         "5 = tcgen05 e2m1 for every non-pooled layer)", kind);
    g_bconv_kind = kind;
    return BNN_OK;
}

BNN_API int bnn_set_first_conv_kernel(int kind) {
    if (kind < 0 || kind > 3)
        return set_error(BNN_ERR_ARG,
                         "first conv kernel kind %d (0 = tcgen05, 1 = mma.sync, 2 = tcgen05 column taps in N, "
                         "3 = tcgen05 weights in M, positions in N)", kind);
    g_first_kind = kind;
    return BNN_OK;
}

BNN_API int bnn_set_arena_poison(int byte) {
    if (byte < -1 || byte > 255) return set_error(BNN_ERR_ARG, "poison byte %d (-1 = off, 0..255)", byte);
    g_poison = byte;
    return BNN_OK;
}

BNN_API int bnn_arena_poison(void) { return arena_poison_byte(); }

BNN_API int bnn_device_error(int device, unsigned int* wait_timeouts) {
    if (!wait_timeouts) return set_error(BNN_ERR_ARG, "NULL argument");
    int prev = 0;
    cudaGetDevice(&prev);
    CK(cudaSetDevice(device));
    cudaError_t e = cudaMemcpyFromSymbol(wait_timeouts, g_bnn_wait_timeouts, sizeof(unsigned int));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "read device error counter: %s", cudaGetErrorString(e));
    return BNN_OK;
}

BNN_API int bnn_wait_probe(int device, int rounds, int* gave_up, unsigned int* timeouts) {
    if (rounds < 1 || rounds > (1 << 22)) return set_error(BNN_ERR_ARG, "rounds %d outside [1, 2^22]", rounds);
    int prev = 0;
    cudaGetDevice(&prev);
    CK(cudaSetDevice(device));
    int* d = nullptr;
    int h[2] = {0, 0};
    int rc = BNN_OK;
    if (cudaMalloc(&d, 2 * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        rc = set_error(BNN_ERR_OOM, "cudaMalloc probe flags");
    }
    if (!rc) {
        wait_probe_kernel<<<1, 1>>>(rounds, d);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpy(h, d, sizeof h, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = set_error(BNN_ERR_CUDA, "wait probe: %s", cudaGetErrorString(e));
        cudaFree(d);
    }
    if (!rc && timeouts && cudaMemcpyFromSymbol(timeouts, g_bnn_wait_timeouts, sizeof(unsigned int)) != cudaSuccess)
        rc = set_error(BNN_ERR_CUDA, "read device error counter");
    if (!rc && gave_up) *gave_up = h[0] && h[1];
    cudaSetDevice(prev);
    return rc;
}

BNN_API int bnn_debug_inject_fault(int kind, int arg) {
    switch (kind) {
        case 0:
            g_fail_alloc = 0; g_fail_wait = 0; g_fail_shard = -1;
            return BNN_OK;
        case BNN_FAULT_ALLOC:
            if (arg < 1) return set_error(BNN_ERR_ARG, "allocation index %d (1 = the next one)", arg);
            g_fail_alloc = arg;
            return BNN_OK;
        case BNN_FAULT_WAIT:
            g_fail_wait = 1;
            return BNN_OK;
        case BNN_FAULT_SHARD:
            if (arg < 0) return set_error(BNN_ERR_ARG, "shard %d", arg);
            g_fail_shard = arg;
            return BNN_OK;
    }
    return set_error(BNN_ERR_ARG, "fault kind %d", kind);
}

BNN_API const char* bnn_bconv_last_kernel(void) { return g_last_kernel; }

BNN_API int bnn_set_devices(Model* m, const int* devices, int n) {
    if (!m || n < 0 || (n > 0 && !devices)) return set_error(BNN_ERR_ARG, "bad arguments");
    int ndev = 0;
    if (n > 0 && (cudaGetDeviceCount(&ndev) != cudaSuccess)) {
        cudaGetLastError();
        return set_error(BNN_ERR_CUDA, "no CUDA device available");
    }
    for (int i = 0; i < n; ++i) {
        if (devices[i] < 0 || devices[i] >= ndev) return set_error(BNN_ERR_ARG, "device %d out of range", devices[i]);
        for (int j = 0; j < i; ++j)
            if (devices[j] == devices[i]) return set_error(BNN_ERR_ARG, "device %d listed twice", devices[i]);
    }
    Engine* E = (Engine*)m->engine;
    std::lock_guard<std::mutex> g(E->mu);
    E->devices.assign(devices, devices + n);
    return BNN_OK;
}

BNN_API int bnn_get_devices(const Model* m, int* devices, int cap) {
    if (!m) return set_error(BNN_ERR_ARG, "model is NULL");
    Engine* E = (Engine*)m->engine;
    std::lock_guard<std::mutex> g(E->mu);
    for (int i = 0; i < (int)E->devices.size() && i < cap; ++i) devices[i] = E->devices[i];
    return (int)E->devices.size();
}

BNN_API int bnn_set_chunk(Model* m, int patches) {
    if (!m || patches < 1) return set_error(BNN_ERR_ARG, "chunk must be >= 1");
    ((Engine*)m->engine)->chunk = patches;
    return BNN_OK;
}

BNN_API int bnn_forward_launches(const Model* m, int N, int H, int W) {
    if (!m || N <= 0 || H < 16 || W < 16) return 0;
    if (eng(m)->stem_c) return 20;                    // stem + 18 binary convs + head
    return first_conv_fast_ok(m, N, H, W) ? 20 : 19;  // + the first conv's fix-up kernel
}

BNN_API int bnn_first_conv_device(const Model* m, int device, const float* d_input, int N, int H, int W,
                                  uint32_t* d_bits, int exact, unsigned int* undecided, void* stream) {
    if (!m || !d_input || !d_bits) return set_error(BNN_ERR_ARG, "NULL argument");
    int rc = check_hw(N, H, W);
    if (rc) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_ARG, "cannot select device %d", device);
    }
    DevState* d = nullptr;
    rc = get_dev(m, device, &d);
    if (!rc) {
        std::lock_guard<std::mutex> g(d->mu);
        cudaStream_t st = (cudaStream_t)stream;
        rc = arena_reserve(m, d, N, H, W);
        if (!rc) {
            cudaStreamWaitEvent(st, d->ev_last, 0);
            rc = poison_arena(d->ar.base, d->ar.bytes, st);
        }
        if (!rc) {
            const bool stem = eng(m)->stem_c > 0;
            const bool fast = !stem && !exact && first_conv_fast_ok(m, N, H, W);
            rc = stem   ? run_stem(d, m, d_input, N, H, W, d_bits, nullptr, st)
                 : fast ? run_realin_fast(d, m, d_input, N, H, W, d_bits, st)
                        : run_realin_exact(d, m, d_input, N, H, W, d_bits, nullptr, st);
            if (!rc) cudaEventRecord(d->ev_last, st);
            if (!rc && undecided) {
                unsigned int ctl[3] = {0, 0, 0};
                if (fast && cudaMemcpyAsync(ctl, d->ar.rm_ctl, sizeof ctl, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                    rc = set_error(BNN_ERR_CUDA, "D2H ctl");
                if (!rc && cudaStreamSynchronize(st) != cudaSuccess)
                    rc = set_error(BNN_ERR_CUDA, "first conv: %s", cudaGetErrorString(cudaGetLastError()));
                *undecided = ctl[1] ? 0xffffffffu : ctl[2];
            }
        }
    }
    cudaSetDevice(prev);
    return rc;
}

// ---------------- profiler ----------------
BNN_API int bnn_profile_enable(Model* m, int on) {
    if (!m) return set_error(BNN_ERR_ARG, "model is NULL");
    ((Engine*)m->engine)->prof.on = on != 0;
    return BNN_OK;
}
BNN_API void bnn_profile_reset(Model* m) {
    if (!m) return;
    Profiler& P = ((Engine*)m->engine)->prof;
    std::lock_guard<std::mutex> g(P.mu);
    P.recs.clear();
}
BNN_API int bnn_profile_count(const Model* m) {
    if (!m) return 0;
    Profiler& P = ((Engine*)m->engine)->prof;
    std::lock_guard<std::mutex> g(P.mu);
    return (int)P.recs.size();
}
BNN_API int bnn_profile_get(const Model* m, int i, const char** label, const char** optype, double* work, double* ms,
                            int* calls) {
    if (!m) return set_error(BNN_ERR_ARG, "model is NULL");
    Profiler& P = ((Engine*)m->engine)->prof;
    std::lock_guard<std::mutex> g(P.mu);
    if (i < 0 || i >= (int)P.recs.size()) return set_error(BNN_ERR_ARG, "profile index %d", i);
    const auto& r = P.recs[i];
    if (label) *label = r.label.c_str();
    if (optype) *optype = r.optype.c_str();
    if (work) *work = r.work;
    if (ms) *ms = r.ms;
    if (calls) *calls = r.calls;
    return BNN_OK;
}
// same two tables as the reference's prof_report (csrc/bnn_prof.c:42-77)
BNN_API void bnn_profile_report(const Model* m, void* file) {
    if (!m) return;
    FILE* o = file ? (FILE*)file : stderr;
    Profiler& P = ((Engine*)m->engine)->prof;
    std::lock_guard<std::mutex> g(P.mu);
    if (P.recs.empty()) return;
    double tot = 0;
    for (auto& r : P.recs) tot += r.ms;
    fprintf(o, "\n# per-op (execution order, device time summed over calls)\n");
    fprintf(o, "%-26s %-10s %6s %12s %10s %7s %10s\n", "layer", "op", "calls", "work", "ms", "%", "Gwork/s");
    for (auto& r : P.recs)
        fprintf(o, "%-26s %-10s %6d %12.4g %10.4f %6.2f %10.1f\n", r.label.c_str(), r.optype.c_str(), r.calls, r.work,
                r.ms, tot > 0 ? 100.0 * r.ms / tot : 0.0, r.ms > 0 ? r.work / (r.ms * 1e6) : 0.0);
    fprintf(o, "\n# roll-up by op type\n");
    fprintf(o, "%-10s %6s %12s %10s %7s\n", "op", "calls", "work", "ms", "%");
    std::vector<std::string> seen;
    for (auto& r : P.recs)
        if (std::find(seen.begin(), seen.end(), r.optype) == seen.end()) seen.push_back(r.optype);
    for (auto& s : seen) {
        double ms = 0, w = 0;
        int c = 0;
        for (auto& r : P.recs)
            if (r.optype == s) { ms += r.ms; w += r.work; c += r.calls; }
        fprintf(o, "%-10s %6d %12.4g %10.4f %6.2f\n", s.c_str(), c, w, ms, tot > 0 ? 100.0 * ms / tot : 0.0);
    }
    fprintf(o, "# total per-op: %.4f ms\n", tot);
}

// ---------------- stage dump ----------------
BNN_API int bnn_forward_stages(const Model* m, const float* input, int H, int W, float* logits, bnn_stage_cb cb,
                               void* ctx) {
    if (!m || !input || !logits) return set_error(BNN_ERR_ARG, "NULL argument");
    int rc = check_hw(1, H, W);
    if (rc) return rc;
    int dev = 0;
    if ((rc = current_device(&dev))) return rc;
    DevState* d = nullptr;
    if ((rc = get_dev(m, dev, &d))) return rc;
    std::lock_guard<std::mutex> g(d->mu);
    if ((rc = arena_reserve(m, d, 1, H, W))) return rc;
    Topology tp;
    topo(m, &tp);
    const size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    const int stc = tp.stem;
    // binary-conv layer geometry in forward order (enc1.conv1 is one of them
    // only behind a v2 stem)
    struct LG { std::string name; int C, h, w; const BinLayer* L; };
    static const char* EN[4] = {"enc1", "enc2", "enc3", "enc4"};
    static const char* DN[4] = {"dec4", "dec3", "dec2", "dec1"};
    std::vector<LG> lg;
    for (int i = 0; i < 4; ++i) {
        if (i > 0 || stc) lg.push_back({std::string(EN[i]) + ".conv1.P", d->enc1[i].Cout, H >> i, W >> i, &d->enc1[i]});
        lg.push_back({std::string(EN[i]) + ".conv2.P", d->enc2[i].Cout, H >> i, W >> i, &d->enc2[i]});
    }
    lg.push_back({"bottleneck.conv1.P", d->bott1.Cout, H >> 4, W >> 4, &d->bott1});
    lg.push_back({"bottleneck.conv2.P", d->bott2.Cout, H >> 4, W >> 4, &d->bott2});
    for (int i = 0; i < 4; ++i) {
        lg.push_back({std::string(DN[i]) + ".conv1.P", d->dec1[i].Cout, H >> (3 - i), W >> (3 - i), &d->dec1[i]});
        lg.push_back({std::string(DN[i]) + ".conv2.P", d->dec2[i].Cout, H >> (3 - i), W >> (3 - i), &d->dec2[i]});
    }
    const int nl = (int)lg.size();
    size_t words = 0;
    std::vector<size_t> poff(nl), pdoff(4);
    for (int k = 0; k < nl; ++k) { poff[k] = words; words += (size_t)lg[k].C * lg[k].h * lg[k].w + 1; }
    for (int i = 0; i < 4; ++i) { pdoff[i] = words; words += (size_t)tp.enc[i] * (H >> (i + 1)) * (W >> (i + 1)) + 1; }
    const size_t ri_words = (size_t)(stc ? stc : m->enc_conv1[0].Cout) * H * W;
    const size_t rb_words = (size_t)H * W * cw_of(m->enc_conv1[0].Cout);
    void* buf = nullptr;
    if (dev_malloc(&buf, (words + ri_words + ip + op + rb_words) * 4) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_OOM, "cudaMalloc stage buffers");
    }
    int32_t* P = (int32_t*)buf;
    float* dri = (float*)(P + words);
    float* din = dri + ri_words;
    float* dout = din + ip;
    Dbg dbg;
    dbg.realin = dri;
    dbg.realin_bits = (uint32_t*)(dout + op);
    for (int k = 0; k < nl; ++k) dbg.P[k] = P + poff[k];
    for (int i = 0; i < 4; ++i) dbg.Pd[i] = P + pdoff[i];
    rc = BNN_OK;
    auto fail = [&](int code) { cudaFree(buf); return code; };
    if (cudaMemcpy(din, input, ip * 4, cudaMemcpyHostToDevice) != cudaSuccess) return fail(set_error(BNN_ERR_CUDA, "H2D"));
    if ((rc = poison_arena(d->ar.base, d->ar.bytes, d->cs))) return fail(rc);
    rc = forward_launches(m, d, din, 1, H, W, dout, d->cs, &dbg, nullptr);
    if (rc) return fail(rc);
    if (cudaStreamSynchronize(d->cs) != cudaSuccess) return fail(set_error(BNN_ERR_CUDA, "forward: %s", cudaGetErrorString(cudaGetLastError())));
    std::vector<int32_t> hP(words);
    std::vector<float> hri(ri_words);
    cudaMemcpy(hP.data(), P, words * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hri.data(), dri, ri_words * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(logits, dout, op * 4, cudaMemcpyDeviceToHost);
    // activations: unpack bit planes from the arena
    Arena& a = d->ar;
    auto bits_to_i8 = [&](const uint32_t* dbits, int C, int h, int w, std::vector<int8_t>& o) {
        const int cw = cw_of(C);
        std::vector<uint32_t> hb((size_t)h * w * cw);
        cudaMemcpy(hb.data(), dbits, hb.size() * 4, cudaMemcpyDeviceToHost);
        o.assign((size_t)C * h * w, 0);
        for (int c = 0; c < C; ++c)
            for (int px = 0; px < h * w; ++px)
                o[(size_t)c * h * w + px] = ((hb[(size_t)px * cw + (c >> 5)] >> (c & 31)) & 1u) ? 1 : -1;
    };
    std::vector<int8_t> act;
    char nm[64];
    int k = 0;
    std::vector<std::vector<int8_t>> skips(4);
    for (int i = 0; i < 4; ++i) {
        const int h = H >> i, w = W >> i;
        if (i == 0 && !stc) {
            cb(ctx, "enc1.conv1.out", 2, m->enc_conv1[0].Cout, H, W, hri.data());
        } else {
            if (i == 0) {
                cb(ctx, "stem.conv.out", 2, stc, H, W, hri.data());
                bits_to_i8(a.stem, stc, H, W, act);
                cb(ctx, "stem.act", 0, stc, H, W, act.data());
            }
            cb(ctx, lg[k].name.c_str(), 1, lg[k].C, h, w, hP.data() + poff[k]);
            ++k;
        }
        bits_to_i8(a.enc_h[i], tp.enc[i], h, w, act);
        snprintf(nm, sizeof nm, "%s.act1", EN[i]);
        cb(ctx, nm, 0, tp.enc[i], h, w, act.data());
        cb(ctx, lg[k].name.c_str(), 1, lg[k].C, h, w, hP.data() + poff[k]);
        ++k;
        bits_to_i8(a.skip[i], tp.enc[i], h, w, skips[i]);
        snprintf(nm, sizeof nm, "%s.act2_skip", EN[i]);
        cb(ctx, nm, 0, tp.enc[i], h, w, skips[i].data());
        snprintf(nm, sizeof nm, "%s.pool.P", EN[i]);
        cb(ctx, nm, 1, tp.enc[i], h >> 1, w >> 1, hP.data() + pdoff[i]);
        bits_to_i8(a.down[i], tp.enc[i], h >> 1, w >> 1, act);
        snprintf(nm, sizeof nm, "%s.act2_down", EN[i]);
        cb(ctx, nm, 0, tp.enc[i], h >> 1, w >> 1, act.data());
    }
    const int h4 = H >> 4, w4 = W >> 4;
    cb(ctx, lg[k].name.c_str(), 1, lg[k].C, h4, w4, hP.data() + poff[k]); ++k;
    bits_to_i8(a.bott_h, d->bott1.Cout, h4, w4, act);
    cb(ctx, "bottleneck.act1", 0, d->bott1.Cout, h4, w4, act.data());
    cb(ctx, lg[k].name.c_str(), 1, lg[k].C, h4, w4, hP.data() + poff[k]); ++k;
    std::vector<int8_t> xprev;
    bits_to_i8(a.bott_x, tp.bott, h4, w4, xprev);
    cb(ctx, "bottleneck.act2", 0, tp.bott, h4, w4, xprev.data());
    int xC = tp.bott, hp = h4, wp = w4;
    for (int i = 0; i < 4; ++i) {
        const int l = 3 - i, h = H >> l, w = W >> l, sC = tp.enc[l];
        // the reference's concat tensor (0 where the upsample does not reach)
        std::vector<int8_t> cat((size_t)(sC + xC) * h * w, 0);
        memcpy(cat.data(), skips[l].data(), (size_t)sC * h * w);
        const int cH = std::min(2 * hp, h), cW = std::min(2 * wp, w);
        const int oh = h > 2 * hp ? (h - 2 * hp) / 2 : 0, ow = w > 2 * wp ? (w - 2 * wp) / 2 : 0;
        for (int c = 0; c < xC; ++c)
            for (int y = 0; y < cH; ++y)
                for (int x = 0; x < cW; ++x)
                    cat[((size_t)(sC + c) * h + oh + y) * w + ow + x] = xprev[((size_t)c * hp + y / 2) * wp + x / 2];
        snprintf(nm, sizeof nm, "%s.cat", DN[i]);
        cb(ctx, nm, 0, sC + xC, h, w, cat.data());
        cb(ctx, lg[k].name.c_str(), 1, lg[k].C, h, w, hP.data() + poff[k]); ++k;
        bits_to_i8(a.dec_h[i], d->dec1[i].Cout, h, w, act);
        snprintf(nm, sizeof nm, "%s.act1", DN[i]);
        cb(ctx, nm, 0, d->dec1[i].Cout, h, w, act.data());
        cb(ctx, lg[k].name.c_str(), 1, lg[k].C, h, w, hP.data() + poff[k]); ++k;
        bits_to_i8(a.dec_x[i], tp.dec[i], h, w, xprev);
        snprintf(nm, sizeof nm, "%s.act2", DN[i]);
        cb(ctx, nm, 0, tp.dec[i], h, w, xprev.data());
        xC = tp.dec[i]; hp = h; wp = w;
    }
    cb(ctx, "logits", 2, m->n_classes, H, W, logits);
    cudaFree(buf);
    return BNN_OK;
}

// ---------------- standalone fused layer (isolated-kernel benchmark) ----------------
struct bnn_bconv_layer {
    int device;
    BinLayer L;
    void* base;
};

BNN_API int bnn_bconv_layer_create(int device, int Cin, int Cout, const uint64_t* packed, const int32_t* type,
                                   const int32_t* t, const int32_t* lo, const int32_t* hi, const int32_t* ptype,
                                   const int32_t* pt, const int32_t* plo, const int32_t* phi, bnn_bconv_layer** out) {
    if (!out || !packed || !type || !t || !lo || !hi || Cin <= 0 || Cout <= 0)
        return set_error(BNN_ERR_ARG, "bad arguments");
    *out = nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    CK(cudaSetDevice(device));
    int arc = set_kernel_attrs(device);
    if (arc) { cudaSetDevice(prev); return arc; }
    auto* Lh = new (std::nothrow) bnn_bconv_layer();
    if (!Lh) return set_error(BNN_ERR_OOM, "OOM");
    Lh->device = device;
    HostBin h;
    relayout_bin(packed, (9 * Cin + 63) / 64, Cin, Cout, Cin, Lh->L, h, ptype != nullptr);
    Act a{0, Cout, (int32_t*)type, (int32_t*)t, (int32_t*)lo, (int32_t*)hi, nullptr, nullptr, nullptr, nullptr};
    folds_of(&a, Lh->L.CoutP, h.fold);
    const bool pool = ptype && pt && plo && phi;
    if (pool) {
        Act a2{0, Cout, (int32_t*)ptype, (int32_t*)pt, (int32_t*)plo, (int32_t*)phi, nullptr, nullptr, nullptr, nullptr};
        folds_of(&a2, Lh->L.CoutP, h.fold2);
    }
    size_t total = align256(h.wt.size() * 4) + align256(h.w8.size()) + align256(h.wu.size()) +
                   align256(h.wx.size()) + align256(h.w4.size()) + align256(h.wus.size()) +
                   align256(h.wpop.size() * 4) +
                   2 * align256(h.fold.size() * sizeof(FoldIv));
    if (dev_malloc(&Lh->base, total) != cudaSuccess) {
        cudaGetLastError();
        delete Lh;
        cudaSetDevice(prev);
        return set_error(BNN_ERR_OOM, "cudaMalloc layer");
    }
    char* p = (char*)Lh->base;
    auto put = [&](const void* src, size_t bytes) -> void* {
        void* dst = p;
        if (bytes) cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
        p += align256(bytes);
        return dst;
    };
    Lh->L.wt = (uint32_t*)put(h.wt.data(), h.wt.size() * 4);
    Lh->L.w8 = (int8_t*)put(h.w8.data(), h.w8.size());
    Lh->L.wu = (int8_t*)put(h.wu.data(), h.wu.size());
    Lh->L.wx = h.wx.empty() ? nullptr : (int8_t*)put(h.wx.data(), h.wx.size());
    Lh->L.w4 = h.w4.empty() ? nullptr : (int8_t*)put(h.w4.data(), h.w4.size());
    Lh->L.wus = (int8_t*)put(h.wus.data(), h.wus.size());
    Lh->L.wpop = (int*)put(h.wpop.data(), h.wpop.size() * 4);
    Lh->L.fold = (FoldIv*)put(h.fold.data(), h.fold.size() * sizeof(FoldIv));
    Lh->L.fold2 = pool ? (FoldIv*)put(h.fold2.data(), h.fold2.size() * sizeof(FoldIv)) : nullptr;
    cudaError_t e = cudaGetLastError();
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaFree(Lh->base);
        delete Lh;
        return set_error(BNN_ERR_CUDA, "layer upload: %s", cudaGetErrorString(e));
    }
    *out = Lh;
    return BNN_OK;
}

BNN_API int bnn_bconv_layer_run(const bnn_bconv_layer* Lh, const uint32_t* d_in, int N, int H, int W, uint32_t* d_out,
                                uint32_t* d_out_pool, int32_t* d_P, int32_t* d_Ppool, void* stream) {
    if (!Lh || !d_in || !d_out || N < 0 || H < 1 || W < 1) return set_error(BNN_ERR_ARG, "bad arguments");
    if ((d_out_pool || d_Ppool) && !Lh->L.fold2) return set_error(BNN_ERR_ARG, "layer has no pooled fold");
    int prev = 0;
    cudaGetDevice(&prev);
    CK(cudaSetDevice(Lh->device));
    int rc = run_bin(Lh->L, d_in, nullptr, 0, 0, N, H, W, d_out, d_out_pool, d_P, d_Ppool, (cudaStream_t)stream);
    cudaSetDevice(prev);
    return rc;
}

BNN_API void bnn_bconv_layer_destroy(bnn_bconv_layer* Lh) {
    if (!Lh) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(Lh->device);
    cudaFree(Lh->base);
    cudaSetDevice(prev);
    delete Lh;
}

// ---------------- helpers ----------------
BNN_API int bnn_synth_device(int device, uint32_t seed, uint32_t first, int N, int bands, int H, int W, float* d_out,
                             void* stream) {
    if (N < 0 || bands <= 0 || H <= 0 || W <= 0 || (!d_out && N > 0)) return set_error(BNN_ERR_ARG, "bad arguments");
    if (N == 0) return BNN_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    CK(cudaSetDevice(device));
    const size_t per = (size_t)bands * H * W, total = per * N;
    synth_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(seed, first, per, total, d_out);
    cudaError_t e = cudaGetLastError();
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "synth launch: %s", cudaGetErrorString(e));
    return BNN_OK;
}

BNN_API int bnn_pack_act_device(const int8_t* d_a, int N, int C, int H, int W, uint32_t* d_bits, void* stream) {
    if (N < 0 || C <= 0 || H <= 0 || W <= 0) return set_error(BNN_ERR_ARG, "bad arguments");
    if (N == 0) return BNN_OK;
    pack_act_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(d_a, N, C, H, W, d_bits);
    CK(cudaGetLastError());
    return BNN_OK;
}

BNN_API int bnn_unpack_act_device(const uint32_t* d_bits, int N, int C, int H, int W, int8_t* d_a, void* stream) {
    if (N < 0 || C <= 0 || H <= 0 || W <= 0) return set_error(BNN_ERR_ARG, "bad arguments");
    if (N == 0) return BNN_OK;
    unpack_act_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(d_bits, N, C, H, W, d_a);
    CK(cudaGetLastError());
    return BNN_OK;
}

// ---------------- host-pointer kernel shims ----------------
namespace bnn {
// the device give-up counter read synchronously (the host-pointer shims
// synchronise the device anyway)
static int read_wait_counter(unsigned int* v) {
    CK(cudaMemcpyFromSymbol(v, g_bnn_wait_timeouts, sizeof(unsigned int)));
    return BNN_OK;
}
// after the device was synchronised: the call's verdict from the counter
// read before it (w0)
static int sync_wait_verdict(unsigned int w0) {
    unsigned int w1 = w0;
    int rc = read_wait_counter(&w1);
    if (rc) return rc;
    if (w1 != w0)
        return set_error(BNN_ERR_CUDA, "%u bounded device wait(s) gave up during this call: its outputs are not valid",
                         w1 - w0);
    return BNN_OK;
}
}  // namespace bnn

BNN_API int bnn_gpu_bconv_dispatch(const int8_t* a, const uint64_t* packed_w, int32_t* P, int Cin, int H, int W,
                                   int Cout, int kh, int kw, int pad, int stride) {
    if (kh != 3 || kw != 3 || stride != 1 || (pad != 0 && pad != 1))
        return set_error(BNN_ERR_UNSUPPORTED, "bconv %dx%d pad %d stride %d: only 3x3 stride 1 pad 0/1", kh, kw, pad,
                         stride);
    if (!a || !packed_w || !P || Cin <= 0 || Cout <= 0 || H <= 0 || W <= 0) return set_error(BNN_ERR_ARG, "bad arguments");
    const int Ho = H + 2 * pad - 2, Wo = W + 2 * pad - 2;
    if (Ho <= 0 || Wo <= 0) return BNN_OK;
    std::vector<int32_t> zeros(Cout, 0);
    bnn_bconv_layer* L = nullptr;
    int rc;
    int dev = 0;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = bnn_bconv_layer_create(dev, Cin, Cout, packed_w, zeros.data(), zeros.data(), zeros.data(), zeros.data(),
                                     nullptr, nullptr, nullptr, nullptr, &L)))
        return rc;
    const int cw = cw_of(Cin);
    const size_t na = (size_t)Cin * H * W, nbits = (size_t)H * W * cw, nP = (size_t)Cout * H * W;
    void* buf = nullptr;
    if (dev_malloc(&buf, na + 16 + nbits * 4 + (size_t)H * W * cw_of(Cout) * 4 + nP * 4) != cudaSuccess) {
        cudaGetLastError();
        bnn_bconv_layer_destroy(L);
        return set_error(BNN_ERR_OOM, "cudaMalloc");
    }
    int8_t* da = (int8_t*)buf;
    uint32_t* dbits = (uint32_t*)((char*)buf + ((na + 15) & ~(size_t)15));
    uint32_t* dout = dbits + nbits;
    int32_t* dP = (int32_t*)(dout + (size_t)H * W * cw_of(Cout));
    unsigned int w0 = 0;
    rc = read_wait_counter(&w0);
    if (!rc && cudaMemcpy(da, a, na, cudaMemcpyHostToDevice) != cudaSuccess) rc = set_error(BNN_ERR_CUDA, "H2D");
    if (!rc) rc = bnn_pack_act_device(da, 1, Cin, H, W, dbits, nullptr);
    if (!rc) rc = bnn_bconv_layer_run(L, dbits, 1, H, W, dout, nullptr, dP, nullptr, nullptr);
    if (!rc) rc = inject_wait(nullptr);
    if (!rc && cudaDeviceSynchronize() != cudaSuccess)
        rc = set_error(BNN_ERR_CUDA, "bconv: %s", cudaGetErrorString(cudaGetLastError()));
    if (!rc) rc = sync_wait_verdict(w0);
    if (!rc) {
        std::vector<int32_t> full(nP);
        cudaMemcpy(full.data(), dP, nP * 4, cudaMemcpyDeviceToHost);
        // pad 0 = the interior of the pad-1 result (every tap in bounds there)
        for (int co = 0; co < Cout; ++co)
            for (int y = 0; y < Ho; ++y)
                for (int x = 0; x < Wo; ++x)
                    P[((size_t)co * Ho + y) * Wo + x] = full[((size_t)co * H + y + 1 - pad) * W + x + 1 - pad];
    }
    cudaFree(buf);
    bnn_bconv_layer_destroy(L);
    return rc;
}

BNN_API int bnn_gpu_conv_realin(const float* x, const int8_t* wsign, const float* alpha, float* out, int Cin, int H,
                                int W, int Cout, int kh, int kw, int pad, int stride) {
    if (kh != 3 || kw != 3 || pad != 1 || stride != 1)
        return set_error(BNN_ERR_UNSUPPORTED, "realin %dx%d pad %d stride %d: only 3x3 pad 1 stride 1", kh, kw, pad,
                         stride);
    if (!x || !wsign || !alpha || !out || Cin <= 0 || Cin > 256 || Cout <= 0 || H <= 0 || W <= 0)
        return set_error(BNN_ERR_ARG, "bad arguments");
    int rc, dev = 0;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = set_kernel_attrs(dev))) return rc;
    DevState d;  // a throwaway state holding only the first-conv tables
    d.device = dev;
    const int CoutP = cdiv(Cout, 32) * 32;
    d.ri_CinP = cdiv(Cin, 4) * 4;
    d.ri_CIP = d.ri_CinP + (((d.ri_CinP / 4) % 2 == 0) ? 4 : 0);
    std::vector<float> wf((size_t)CoutP * 9 * d.ri_CinP, 0.0f), fold((size_t)CoutP * 5, 0.0f);
    for (int co = 0; co < Cout; ++co) {
        for (int ci = 0; ci < Cin; ++ci)
            for (int t = 0; t < 9; ++t) wf[((size_t)co * 9 + t) * d.ri_CinP + ci] = (float)wsign[((size_t)co * Cin + ci) * 9 + t];
        fold[co * 5] = alpha[co];
        fold[co * 5 + 1] = 1.0f;  // identity fold; only the conv output is returned
    }
    Model mm;
    memset(&mm, 0, sizeof mm);
    mm.enc_conv1[0].Cin = Cin;
    mm.enc_conv1[0].Cout = Cout;
    const size_t nx = (size_t)Cin * H * W, no = (size_t)Cout * H * W, nb = (size_t)H * W * cw_of(Cout);
    void* buf = nullptr;
    const size_t bytes = (wf.size() + fold.size() + nx + no + nb) * 4;
    if (dev_malloc(&buf, bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_OOM, "cudaMalloc");
    }
    d.ri_wf = (float*)buf;
    d.ri_fold = d.ri_wf + wf.size();
    float* dx = d.ri_fold + fold.size();
    float* dout = dx + nx;
    uint32_t* dbits = (uint32_t*)(dout + no);
    rc = BNN_OK;
    if (cudaMemcpy(d.ri_wf, wf.data(), wf.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d.ri_fold, fold.data(), fold.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dx, x, nx * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = set_error(BNN_ERR_CUDA, "H2D");
    if (!rc) rc = run_realin_exact(&d, &mm, dx, 1, H, W, dbits, dout, nullptr);
    if (!rc && cudaDeviceSynchronize() != cudaSuccess)
        rc = set_error(BNN_ERR_CUDA, "realin: %s", cudaGetErrorString(cudaGetLastError()));
    if (!rc && cudaMemcpy(out, dout, no * 4, cudaMemcpyDeviceToHost) != cudaSuccess) rc = set_error(BNN_ERR_CUDA, "D2H");
    cudaFree(buf);
    d.device = -1;  // nothing else to release
    return rc;
}

// ===================================================================
// Allocation-free bconv_dispatch.
//
// For callers that must not allocate device memory: processes whose GPU
// memory is fixed up front by an allocator or memory budget of their own (an
// extra cudaMalloc can fail there, or fragment the pool), and latency-bound
// loops that cannot afford the device-wide synchronisation cudaFree implies.
// bnn_gpu_bconv_dispatch stages its operands in cudaMalloc'd buffers; this
// variant carves the same buffers out of one file-scope static device array
// of BNN_NOALLOC_SCRATCH_BYTES, which every GPU that loads the library holds
// until the process exits.
// ===================================================================
namespace bnn {

static constexpr size_t kNoAllocScratch = BNN_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratch];

static std::mutex g_noalloc_mu;
static bool g_noalloc_attrs[64];  // kernel attributes set on this device

// On every call, with the call's device current: the array's name in host
// code is only a host-side stand-in, so its device address comes from
// cudaGetSymbolAddress (looked up each time, so a device reset or a new
// primary context never leaves a stale address behind). The kernels'
// shared-memory attributes are set once per device, on its first call.
static int noalloc_scratch(int dev, unsigned char** out) {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (dev < 0 || dev >= 64) return set_error(BNN_ERR_ARG, "device %d out of range for the static scratch", dev);
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
        cudaGetLastError();
        return set_error(BNN_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    }
    if (!g_noalloc_attrs[dev]) {
        int rc = set_kernel_attrs(dev);
        if (rc) return rc;
        g_noalloc_attrs[dev] = true;
    }
    *out = (unsigned char*)p;
    return BNN_OK;
}

// kidx-ordered weights (bit ci*9+t of row co) -> tap-major words + per-tap
// popcounts (XOR/POPC kernel) and +-1 int8 rows (tensor-core kernel), one
// thread per (co, tap); rows co >= Cout and channels >= Cin are written as
// zero, so nothing in the shared array has to be cleared first.
__global__ void noalloc_relayout_kernel(const uint64_t* packed, int nwords, int Cin, int Cout, int CoutP, int Kw,
                                        uint32_t* wt, int8_t* w8, int* wpop, FoldIv* fold) {
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= CoutP * 9) return;
    const int co = g / 9, t = g - co * 9;
    int pop = 0;
    for (int w = 0; w < Kw; ++w) {
        uint32_t word = 0u;
        if (co < Cout)
            for (int b = 0; b < 32; ++b) {
                const int ci = w * 32 + b;
                if (ci >= Cin) break;
                const int k = ci * 9 + t;
                if ((packed[(size_t)co * nwords + (k >> 6)] >> (k & 63)) & 1ull) word |= 1u << b;
            }
        wt[(size_t)g * Kw + w] = word;
        int8_t* row8 = w8 + (((size_t)w * 9 + t) * CoutP + co) * 32;
        for (int b = 0; b < 32; ++b) row8[b] = (co < Cout && w * 32 + b < Cin) ? (((word >> b) & 1u) ? 1 : -1) : 0;
        pop += __popc(word);
    }
    wpop[g] = pop;
    if (t == 0) fold[co] = FoldIv{0, 0, 0, 0};  // P is the output; the fold is unused
}

// P [Cout][H][W] (pad-1 geometry) -> interior [Cout][H-2][W-2] for pad 0
__global__ void noalloc_crop_kernel(const int32_t* P, int Cout, int H, int W, int32_t* out) {
    const int Ho = H - 2, Wo = W - 2;
    const size_t total = (size_t)Cout * Ho * Wo;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const int x = (int)(g % Wo), y = (int)((g / Wo) % Ho);
        const size_t c = g / ((size_t)Wo * Ho);
        out[g] = P[(c * H + y + 1) * W + x + 1];
    }
}

}  // namespace bnn

BNN_API int bnn_gpu_bconv_dispatch_noalloc(const int8_t* a, const uint64_t* packed_w, int32_t* P, int Cin, int H,
                                           int W, int Cout, int kh, int kw, int pad, int stride) {
    if (kh != 3 || kw != 3 || stride != 1 || (pad != 0 && pad != 1))
        return set_error(BNN_ERR_UNSUPPORTED, "bconv %dx%d pad %d stride %d: only 3x3 stride 1 pad 0/1", kh, kw, pad,
                         stride);
    if (!a || !packed_w || !P || Cin <= 0 || Cout <= 0 || H <= 0 || W <= 0) return set_error(BNN_ERR_ARG, "bad arguments");
    const int Ho = H + 2 * pad - 2, Wo = W + 2 * pad - 2;
    if (Ho <= 0 || Wo <= 0) return BNN_OK;
    int rc, dev = 0;
    // layout of the static scratch for this call (256-byte aligned regions)
    const int nwords = (9 * Cin + 63) / 64, Kw = cw_of(Cin), CoutP = cdiv(Cout, 128) * 128;
    const size_t n_a = (size_t)Cin * H * W, n_pk = (size_t)Cout * nwords * 8, n_bits = (size_t)H * W * Kw * 4,
                 n_wt = (size_t)CoutP * 9 * Kw * 4, n_w8 = (size_t)Kw * 9 * CoutP * 32, n_pop = (size_t)CoutP * 9 * 4,
                 n_fold = (size_t)CoutP * sizeof(FoldIv),
                 n_out = (size_t)H * W * cw_of(Cout) * 4, n_P = (size_t)Cout * H * W * 4,
                 n_crop = pad == 0 ? (size_t)Cout * Ho * Wo * 4 : 0;
    const size_t need = align256(n_a) + align256(n_pk) + align256(n_bits) + align256(n_wt) + align256(n_w8) +
                        align256(n_pop) +
                        align256(n_fold) + align256(n_out) + align256(n_P) + align256(n_crop);
    if (need > kNoAllocScratch)
        return set_error(BNN_ERR_ARG,
                         "bconv Cin=%d H=%d W=%d Cout=%d needs %zu bytes of scratch, above the %zu-byte static array",
                         Cin, H, W, Cout, need, kNoAllocScratch);
    if ((rc = current_device(&dev))) return rc;
    unsigned char* base = nullptr;
    if ((rc = noalloc_scratch(dev, &base))) return rc;
    unsigned char* p = base;
    auto take = [&](size_t bytes) { unsigned char* r = p; p += align256(bytes); return r; };
    int8_t* da = (int8_t*)take(n_a);
    uint64_t* dpk = (uint64_t*)take(n_pk);
    uint32_t* dbits = (uint32_t*)take(n_bits);
    BinLayer L;
    L.Cin = Cin; L.Cout = Cout; L.CoutP = CoutP; L.cw0 = Kw; L.cw1 = 0; L.Kw = Kw; L.sC = Cin;
    L.wt = (uint32_t*)take(n_wt);
    L.w8 = (int8_t*)take(n_w8);
    L.wpop = (int*)take(n_pop);
    L.fold = (FoldIv*)take(n_fold);
    L.fold2 = nullptr;
    uint32_t* dout = (uint32_t*)take(n_out);
    int32_t* dP = (int32_t*)take(n_P);
    int32_t* dcrop = (int32_t*)take(n_crop);
    // every region below is fully rewritten by this call before it is read
    unsigned int w0 = 0;
    if ((rc = read_wait_counter(&w0))) return rc;
    CK(cudaMemcpy(da, a, n_a, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dpk, packed_w, n_pk, cudaMemcpyHostToDevice));
    noalloc_relayout_kernel<<<cdiv((long)CoutP * 9, 128), 128>>>(dpk, nwords, Cin, Cout, CoutP, Kw, L.wt, L.w8, L.wpop,
                                                                 L.fold);
    CK(cudaGetLastError());
    pack_act_kernel<<<148 * 4, 256>>>(da, 1, Cin, H, W, dbits);
    CK(cudaGetLastError());
    if ((rc = run_bin(L, dbits, nullptr, 0, 0, 1, H, W, dout, nullptr, dP, nullptr, nullptr))) return rc;
    const int32_t* src = dP;
    if (pad == 0) {
        noalloc_crop_kernel<<<148 * 4, 256>>>(dP, Cout, H, W, dcrop);
        CK(cudaGetLastError());
        src = dcrop;
    }
    if ((rc = inject_wait(nullptr))) return rc;
    CK(cudaMemcpy(P, src, (size_t)Cout * Ho * Wo * 4, cudaMemcpyDeviceToHost));
    return sync_wait_verdict(w0);
}
