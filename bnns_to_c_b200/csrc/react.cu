// react.cu - the v3 ReActNet real-highway engine (csrc/bnn_model_react.c)
// behind the drop-in include/bnn_model_react.h.
//
// Per patch the forward is the reference's (:395-441) on the whole image
// (its enc1 / dec1 row strips give the same values): for each block, unit1
// = projection of the input (+ the input's tap bits), binary conv1 on the
// tap, epilogue (+ the result's tap bits for conv2); unit2 = binary conv2,
// then the skip and pooled-down epilogues (encoder) or the block output
// (bottleneck, decoder); decoders read their concat (skip + nearest
// upsample) in place. Binary convs run on the v1 engine's tcgen05 kernels
// through bnn_bconv_layer_* with their exact P written out; the float work
// is react_kernels.cuh. Activations stay in one device arena per (N, H, W);
// repeated device forwards replay a captured CUDA graph.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include <cuda_runtime.h>

#include "common.h"
#include "react_kernels.cuh"
#include "../../include/bnn_model_react.h"

namespace bnn {

namespace {

#define RCK(call)                                                                                  \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) return set_error(BNN_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }
inline int cw_of(int c) { return (c + 31) >> 5; }
inline size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

const char* BN[9] = {"enc1", "enc2", "enc3", "enc4", "bottleneck", "dec4", "dec3", "dec2", "dec1"};

// device copies of one block's float parameters
struct RBlockDev {
    float *proj = nullptr;   // [slices][Cin][16]
    float *tap1 = nullptr, *tap2 = nullptr;
    float *A1 = nullptr, *Bm1 = nullptr, *pw1 = nullptr;
    float *Aa = nullptr, *Bma = nullptr, *pwa = nullptr;
    float *Ab = nullptr, *Bmb = nullptr, *pwb = nullptr;
    bnn_bconv_layer *conv1 = nullptr, *conv2 = nullptr;
    int Cin = 0, Cout = 0;
};

// activations of one block at (N, h, w)
struct RBuf {
    float *res = nullptr, *h1 = nullptr, *out = nullptr, *down = nullptr, *c1 = nullptr;
    uint32_t *t1 = nullptr, *t2 = nullptr;
    int32_t *P1 = nullptr, *P2 = nullptr;
    int h = 0, w = 0;
};

struct GraphKeyR {
    int N, H, W;
    const void *in, *out;
    bool operator<(const GraphKeyR& o) const { return std::tie(N, H, W, in, out) < std::tie(o.N, o.H, o.W, o.in, o.out); }
};

struct RDev {
    int device = -1;
    std::mutex mu;
    void* wbase = nullptr;
    RBlockDev blk[9];
    float *c3w = nullptr, *c3a = nullptr;  // enc1 conv: [Cout/16][Cin][9][16], alpha
    float *headW = nullptr, *headb = nullptr;
    // arena
    void* abase = nullptr;
    size_t abytes = 0;
    int aN = 0, aH = 0, aW = 0;
    RBuf buf[9];
    uint32_t* scratch = nullptr;           // the binary convs' (unused) bit outputs
    cudaStream_t cs = nullptr;
    cudaEvent_t ev_last = nullptr;
    std::map<GraphKeyR, cudaGraphExec_t> graphs;
    // host batches: two device staging slots, copies on their own streams
    float *pin[2] = {nullptr, nullptr}, *pout[2] = {nullptr, nullptr};
    size_t pcap = 0, pin_floats = 0, pout_floats = 0;
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t ev_in[2] = {nullptr, nullptr}, ev_comp[2] = {nullptr, nullptr}, ev_out[2] = {nullptr, nullptr};
};

struct RProfiler {
    struct Rec {
        std::string label, optype;
        double work = 0, ms = 0;
        int calls = 0;
    };
    bool on = false;
    std::vector<Rec> recs;
    std::mutex mu;
};

struct REngine {
    std::mutex mu;
    std::map<int, std::unique_ptr<RDev>> devs;
    RProfiler prof;
};

const BlockR& block_of(const ModelR* m, int b) { return b < 4 ? m->enc[b] : b == 4 ? m->bott : m->dec[b - 5]; }

void rdev_release(RDev* d) {
    if (!d || d->device < 0) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(d->device);
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
    if (d->cs) cudaStreamSynchronize(d->cs);
    for (auto& b : d->blk) {
        bnn_bconv_layer_destroy(b.conv1);
        bnn_bconv_layer_destroy(b.conv2);
        b.conv1 = b.conv2 = nullptr;
    }
    if (d->h2d) cudaStreamSynchronize(d->h2d);
    if (d->d2h) cudaStreamSynchronize(d->d2h);
    cudaFree(d->wbase);
    cudaFree(d->abase);
    for (int k = 0; k < 2; ++k) {
        cudaFree(d->pin[k]);
        cudaFree(d->pout[k]);
        if (d->ev_in[k]) cudaEventDestroy(d->ev_in[k]);
        if (d->ev_comp[k]) cudaEventDestroy(d->ev_comp[k]);
        if (d->ev_out[k]) cudaEventDestroy(d->ev_out[k]);
    }
    if (d->ev_last) cudaEventDestroy(d->ev_last);
    if (d->cs) cudaStreamDestroy(d->cs);
    if (d->h2d) cudaStreamDestroy(d->h2d);
    if (d->d2h) cudaStreamDestroy(d->d2h);
    cudaSetDevice(prev);
}

// upload the model to device d (d->mu held, device current)
int rdev_init(const ModelR* m, RDev* d) {
    std::vector<std::pair<std::vector<float>, float**>> up;  // host array -> device slot
    auto add = [&](std::vector<float> v, float** slot) { up.emplace_back(std::move(v), slot); };
    auto vec = [](const float* p, int n) { return std::vector<float>(p, p + n); };
    auto epi = [&](const EpiR& e, float** A, float** Bm, float** pw) {
        std::vector<float> bm(e.C);
        for (int c = 0; c < e.C; ++c) bm[c] = e.B[c] + e.move1[c];  // fp32, once per channel (as the reference)
        add(vec(e.A, e.C), A);
        add(bm, Bm);
        add(vec(e.prelu_w, e.C), pw);
    };
    for (int b = 0; b < 9; ++b) {
        const BlockR& B = block_of(m, b);
        RBlockDev& D = d->blk[b];
        D.Cin = B.conv1.Cin;
        D.Cout = B.conv1.Cout;
        const int sl = cdiv(D.Cout, react::PROJ_CB);
        std::vector<float> pj((size_t)sl * D.Cin * react::PROJ_CB, 0.0f);
        for (int co = 0; co < D.Cout; ++co)
            for (int ci = 0; ci < D.Cin; ++ci)
                pj[((size_t)(co / react::PROJ_CB) * D.Cin + ci) * react::PROJ_CB + co % react::PROJ_CB] =
                    B.proj1.W[(size_t)co * D.Cin + ci];
        add(pj, &D.proj);
        if (!B.input_real) add(vec(B.tap1.rsign, B.tap1.C), &D.tap1);
        add(vec(B.tap2.rsign, B.tap2.C), &D.tap2);
        epi(B.epi1, &D.A1, &D.Bm1, &D.pw1);
        epi(B.epi_a, &D.Aa, &D.Bma, &D.pwa);
        if (B.is_down) epi(B.epi_b, &D.Ab, &D.Bmb, &D.pwb);
    }
    {
        const ConvR& c1 = m->enc[0].conv1;
        const int nb = cdiv(c1.Cout, 16);
        std::vector<float> w((size_t)nb * c1.Cin * 9 * 16, 0.0f);
        for (int co = 0; co < c1.Cout; ++co)
            for (int ci = 0; ci < c1.Cin; ++ci)
                for (int t = 0; t < 9; ++t)
                    w[(((size_t)(co / 16) * c1.Cin + ci) * 9 + t) * 16 + co % 16] =
                        (float)c1.wsign[((size_t)co * c1.Cin + ci) * 9 + t];
        add(w, &d->c3w);
        add(vec(c1.alpha, c1.Cout), &d->c3a);
    }
    add(vec(m->head_W, m->head_Cout * m->head_Cin), &d->headW);
    add(vec(m->head_bias, m->head_Cout), &d->headb);
    size_t total = 0;
    for (auto& u : up) total += al256(u.first.size() * 4 + 4);
    if (cudaMalloc(&d->wbase, total) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_OOM, "cudaMalloc ReAct weights (%zu bytes)", total);
    }
    char* p = (char*)d->wbase;
    for (auto& u : up) {
        RCK(cudaMemcpy(p, u.first.data(), u.first.size() * 4, cudaMemcpyHostToDevice));
        *u.second = (float*)p;
        p += al256(u.first.size() * 4 + 4);
    }
    // binary convs: the v1 engine's layers, constant folds (their bit output
    // is not used; P is)
    for (int b = 0; b < 9; ++b) {
        const BlockR& B = block_of(m, b);
        const ConvR* cs[2] = {&B.conv1, &B.conv2};
        bnn_bconv_layer** slots[2] = {&d->blk[b].conv1, &d->blk[b].conv2};
        for (int k = 0; k < 2; ++k) {
            if (k == 0 && B.input_real) continue;
            const int C = cs[k]->Cout;
            std::vector<int32_t> zero(C, 0);
            int rc = bnn_bconv_layer_create(d->device, cs[k]->Cin, C, cs[k]->packed, zero.data(), zero.data(),
                                            zero.data(), zero.data(), nullptr, nullptr, nullptr, nullptr, slots[k]);
            if (rc) return rc;
        }
    }
    RCK(cudaFuncSetAttribute(react::conv3_tma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)react::C4Cfg<64>::SMEM));
    RCK(cudaFuncSetAttribute(react::conv3_tma_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)react::C4Cfg<32>::SMEM));
    {
        const int sm = react::PROJ_MAX_CIN * react::PROJ_CB * 4;
#define PROJ_ATTR(px, cat, tap)                                                                             \
    RCK(cudaFuncSetAttribute(react::proj_tap_kernel<px, cat, tap, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             sm));                                                                                  \
    RCK(cudaFuncSetAttribute(react::proj_tap_kernel<px, cat, tap, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm))
        PROJ_ATTR(1, false, false); PROJ_ATTR(1, false, true); PROJ_ATTR(1, true, true);
#undef PROJ_ATTR
        const int sa = sm + react::PROJ_D * 256 * 16;
#define PROJ_ATTR_A(cat, tap)                                                                                  \
    RCK(cudaFuncSetAttribute(react::proj_async_kernel<cat, tap, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             sa));                                                                             \
    RCK(cudaFuncSetAttribute(react::proj_async_kernel<cat, tap, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, sa))
        PROJ_ATTR_A(false, false); PROJ_ATTR_A(false, true); PROJ_ATTR_A(true, true);
#undef PROJ_ATTR_A
    }
    RCK(cudaStreamCreateWithFlags(&d->cs, cudaStreamNonBlocking));
    RCK(cudaStreamCreateWithFlags(&d->h2d, cudaStreamNonBlocking));
    RCK(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
    for (int k = 0; k < 2; ++k) {
        RCK(cudaEventCreateWithFlags(&d->ev_in[k], cudaEventDisableTiming));
        RCK(cudaEventCreateWithFlags(&d->ev_comp[k], cudaEventDisableTiming));
        RCK(cudaEventCreateWithFlags(&d->ev_out[k], cudaEventDisableTiming));
        RCK(cudaEventRecord(d->ev_comp[k], d->cs));
        RCK(cudaEventRecord(d->ev_out[k], d->cs));
    }
    RCK(cudaEventCreateWithFlags(&d->ev_last, cudaEventDisableTiming));
    RCK(cudaEventRecord(d->ev_last, d->cs));
    return BNN_OK;
}

int get_rdev(const ModelR* m, int device, RDev** out) {
    REngine* E = (REngine*)m->engine;
    if (!E) return set_error(BNN_ERR_ARG, "model has no engine");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
        cudaGetLastError();
        return set_error(BNN_ERR_CUDA, "no CUDA device available");
    }
    if (device < 0 || device >= ndev) return set_error(BNN_ERR_ARG, "device %d out of range [0,%d)", device, ndev);
    RDev* d;
    {
        std::lock_guard<std::mutex> g(E->mu);
        auto& slot = E->devs[device];
        if (!slot) slot.reset(new RDev());
        d = slot.get();
    }
    std::lock_guard<std::mutex> g(d->mu);
    if (d->device < 0) {
        RCK(cudaSetDevice(device));
        d->device = device;
        int rc = rdev_init(m, d);
        if (rc) {
            rdev_release(d);
            d->device = -1;
            d->wbase = d->abase = nullptr;
            for (auto& b : d->blk) b = RBlockDev();
            d->cs = nullptr;
            d->ev_last = nullptr;
            d->aN = d->aH = d->aW = 0;
            return rc;
        }
    }
    *out = d;
    return BNN_OK;
}

// arena for N patches of H x W (d->mu held)
int arena(const ModelR* m, RDev* d, int N, int H, int W) {
    if (d->abase && d->aN >= N && d->aH == H && d->aW == W) return BNN_OK;
    const int Nn = std::max(N, d->aH == H && d->aW == W ? d->aN : 0);
    size_t off = 0;
    std::vector<std::pair<void**, size_t>> plan;
    auto take = [&](void** slot, size_t bytes) {
        plan.push_back({slot, off});
        off += al256(bytes + 16);
    };
    size_t scratch = 0;
    for (int b = 0; b < 9; ++b) {
        const int l = b < 4 ? b : b == 4 ? 4 : 8 - b;  // resolution level
        const int h = H >> l, w = W >> l;
        const size_t px = (size_t)Nn * h * w;
        const RBlockDev& D = d->blk[b];
        RBuf& B = d->buf[b];
        B.h = h;
        B.w = w;
        take((void**)&B.res, px * D.Cout * 4);
        take((void**)&B.h1, px * D.Cout * 4);
        take((void**)&B.out, px * D.Cout * 4);
        take((void**)&B.t2, px * cw_of(D.Cout) * 4);
        take((void**)&B.P2, px * D.Cout * 4);
        if (b == 0) take((void**)&B.c1, px * D.Cout * 4);
        else {
            take((void**)&B.t1, px * cw_of(D.Cin) * 4);
            take((void**)&B.P1, px * D.Cout * 4);
        }
        if (b < 4) take((void**)&B.down, (size_t)Nn * (h / 2) * (w / 2) * D.Cout * 4);
        scratch = std::max(scratch, px * cw_of(D.Cout) * 4);
    }
    take((void**)&d->scratch, scratch);
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
    if (d->abase) {
        RCK(cudaEventSynchronize(d->ev_last));
        cudaFree(d->abase);
        d->abase = nullptr;
    }
    if (cudaMalloc(&d->abase, off) != cudaSuccess) {
        cudaGetLastError();
        d->aN = 0;
        return set_error(BNN_ERR_OOM, "cudaMalloc ReAct arena (%zu bytes)", off);
    }
    for (auto& pr : plan) *pr.first = (char*)d->abase + pr.second;
    d->abytes = off;
    d->aN = Nn;
    d->aH = H;
    d->aW = W;
    return BNN_OK;
}

// the arena filled with BNN_ARENA_POISON's byte before a forward (debug;
// every launch must write what it later reads)
static int poison(RDev* d, cudaStream_t s) {
    const int b = arena_poison_byte();
    if (b < 0 || !d->abase) return BNN_OK;
    if (cudaMemsetAsync(d->abase, b, d->abytes, s) != cudaSuccess)
        return set_error(BNN_ERR_CUDA, "arena poison: %s", cudaGetErrorString(cudaGetLastError()));
    return BNN_OK;
}

struct RProf {
    RProfiler* prof = nullptr;
    cudaStream_t st = nullptr;
    std::vector<std::tuple<std::string, const char*, double, cudaEvent_t, cudaEvent_t>> marks;
    void begin(const std::string& l, const char* op, double work) {
        if (!prof) return;
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, st);
        marks.emplace_back(l, op, work, a, b);
    }
    void end() {
        if (prof) cudaEventRecord(std::get<4>(marks.back()), st);
    }
    int finish() {
        if (!prof) return BNN_OK;
        RCK(cudaStreamSynchronize(st));
        std::lock_guard<std::mutex> g(prof->mu);
        for (auto& mk : marks) {
            float ms = 0;
            cudaEventElapsedTime(&ms, std::get<3>(mk), std::get<4>(mk));
            bool found = false;
            for (auto& r : prof->recs)
                if (r.label == std::get<0>(mk)) { r.work += std::get<2>(mk); r.ms += ms; r.calls++; found = true; break; }
            if (!found) prof->recs.push_back({std::get<0>(mk), std::get<1>(mk), std::get<2>(mk), ms, 1});
            cudaEventDestroy(std::get<3>(mk));
            cudaEventDestroy(std::get<4>(mk));
        }
        marks.clear();
        return BNN_OK;
    }
};

typedef CUresult (*EncodeTiledFnR)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point
EncodeTiledFnR encode_tiled_r() {
    static EncodeTiledFnR fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFnR)f;
        cudaGetLastError();
    });
    return fn;
}

// the enc1 input as a 4-D map (W, H, bands, patches), box = one stage of
// conv3_tma_kernel<TC>; false where TMA cannot address it (W % 4, alignment)
bool conv3_tmap(const float* x, int N, int C, int H, int W, int TC, CUtensorMap* tm) {
    EncodeTiledFnR fn = encode_tiled_r();
    if (!fn || W % 4 || ((uintptr_t)x & 15)) return false;
    const int bx = TC + 8, by = 128 / (TC / 4) + 2;
    const cuuint64_t dims[4] = {(cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)C, (cuuint64_t)N};
    const cuuint64_t strides[3] = {(cuuint64_t)W * 4, (cuuint64_t)H * W * 4, (cuuint64_t)C * H * W * 4};
    const cuuint32_t box[4] = {(cuuint32_t)bx, (cuuint32_t)by, (cuuint32_t)react::C4_CK, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// conv kernel choice (A/B): 0 = TMA-staged where it applies, 1 = the
// thread-staged kernel
int g_conv3_kind = 0;

int launched(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return BNN_OK;
}

int run_proj(const RBlockDev& D, const float* x0, int c0, const float* x1, int c1, int h1, int w1, int N, int H,
             int W, bool blocked, float* out, uint32_t* bits, cudaStream_t st) {
    react::ProjParams p{};
    p.x0 = x0; p.x1 = x1; p.c0 = c0; p.c1 = c1; p.h1 = h1; p.w1 = w1;
    const int upH = 2 * h1, upW = 2 * w1;
    p.oh = H > upH ? (H - upH) / 2 : 0;
    p.ow = W > upW ? (W - upW) / 2 : 0;
    p.cH = std::min(upH, H);
    p.cW = std::min(upW, W);
    p.N = N; p.H = H; p.W = W; p.Cin = D.Cin; p.Cout = D.Cout;
    p.w = D.proj;
    const int HW = H * W;
    p.nfull = blocked ? HW - HW % 8 : HW;  // proj_blk's pixel blocks of 8 vs react_proj_1x1
    p.out = out;
    p.rsign = bits ? D.tap1 : nullptr;
    p.bits = bits;
    // 4 pixels of one row per thread when rows split evenly and the plain
    // input is 16-byte aligned
    const bool v4 = W % 4 == 0 && ((uintptr_t)x0 & 15) == 0;
    const int PX = v4 ? 4 : 1;
    const dim3 grid(cdiv((long long)N * HW / PX, 256), cdiv(D.Cout, react::PROJ_CB));
    const size_t smem = (size_t)D.Cin * react::PROJ_CB * 4;
    const size_t smem_a = smem + (size_t)react::PROJ_D * 256 * 16;  // + the cp.async slots
    const bool all_fused = p.nfull == HW;
#define PROJ_LAUNCH(cat, tap)                                                                              \
    do {                                                                                                   \
        if (v4) {                                                                                          \
            if (all_fused) react::proj_async_kernel<cat, tap, 1><<<grid, 256, smem_a, st>>>(p);             \
            else react::proj_async_kernel<cat, tap, 0><<<grid, 256, smem_a, st>>>(p);                      \
        } else {                                                                                           \
            if (all_fused) react::proj_tap_kernel<1, cat, tap, 1><<<grid, 256, smem, st>>>(p);              \
            else react::proj_tap_kernel<1, cat, tap, 0><<<grid, 256, smem, st>>>(p);                       \
        }                                                                                                  \
    } while (0)
    if (x1) PROJ_LAUNCH(true, true);
    else if (bits) PROJ_LAUNCH(false, true);
    else PROJ_LAUNCH(false, false);
#undef PROJ_LAUNCH
    return launched("proj");
}

int run_epi(const int32_t* P, const float* v, const float* res, float* out, const float* A, const float* Bm,
            const float* pw, const float* rsign, uint32_t* bits, int N, int C, int HW, cudaStream_t st) {
    react::EpiParams p{P, v, res, out, A, Bm, pw, rsign, bits, N, C, HW};
    const bool v4 = HW % 4 == 0 && (((uintptr_t)(P ? (const void*)P : (const void*)v) | (uintptr_t)res |
                                      (uintptr_t)out) & 15) == 0;
    const unsigned chunks = (unsigned)cdiv(C, 32);
    if (v4) react::epi_kernel<4><<<dim3(cdiv((long long)N * HW / 4, 256), chunks), 256, 0, st>>>(p);
    else react::epi_kernel<1><<<dim3(cdiv((long long)N * HW, 256), chunks), 256, 0, st>>>(p);
    return launched("epilogue");
}

int run_bconv(const bnn_bconv_layer* L, const uint32_t* in, int N, int h, int w, int32_t* P, uint32_t* scratch,
              cudaStream_t st) {
    return bnn_bconv_layer_run(L, in, N, h, w, scratch, nullptr, P, nullptr, st);
}

// one forward of N patches (x, logits on the device)
int forward_launches(const ModelR* m, RDev* d, const float* x, int N, int H, int W, float* logits, cudaStream_t st,
                     RProf* pc) {
    int rc;
    auto beg = [&](int b, const char* what, const char* op, double work) {
        if (pc && pc->prof) pc->begin(std::string(BN[b]) + "." + what, op, work);
    };
    auto end = [&]() { if (pc && pc->prof) pc->end(); };
    const float* xin = x;  // input of the current block
    int xc = m->n_bands, xh = H, xw = W;
    for (int b = 0; b < 9; ++b) {
        const BlockR& B = block_of(m, b);
        RBlockDev& D = d->blk[b];
        RBuf& Q = d->buf[b];
        const int h = Q.h, w = Q.w, HW = h * w;
        const double px = (double)N * HW;
        const bool blocked = D.Cout % 8 == 0;
        // ---- unit1
        if (b == 0) {
            beg(b, "proj", "proj", px * D.Cout * D.Cin);
            rc = run_proj(D, xin, D.Cin, nullptr, 0, 0, 0, N, h, w, blocked, Q.res, nullptr, st);
            end();
            if (rc) return rc;
            react::Conv3Params c{xin, d->c3w, d->c3a, Q.c1, N, D.Cin, h, w, D.Cout, cdiv(w, react::C3_TC),
                                 cdiv(h, react::C3_TR)};
            beg(b, "conv1", "conv_real", px * D.Cout * D.Cin * 9.0);
            const int TC = w >= 64 ? 64 : 32;
            CUtensorMap tm;
            if (blocked && g_conv3_kind == 0 && conv3_tmap(xin, N, D.Cin, h, w, TC, &tm)) {
                react::Conv3Params c4 = c;
                c4.tiles_x = cdiv(w, TC);
                c4.tiles_y = cdiv(h, 512 / TC);
                const dim3 grid(N * c4.tiles_x * c4.tiles_y, cdiv(D.Cout, 16));
                if (TC == 64)
                    react::conv3_tma_kernel<64><<<grid, 128, react::C4Cfg<64>::SMEM, st>>>(tm, c4);
                else
                    react::conv3_tma_kernel<32><<<grid, 128, react::C4Cfg<32>::SMEM, st>>>(tm, c4);
            } else if (blocked) {
                react::conv3_blk_kernel<<<dim3(N * c.tiles_x * c.tiles_y, cdiv(D.Cout, 16)), 128, 0, st>>>(c);
            } else {
                react::conv3_naive_kernel<<<cdiv((long long)N * HW * cdiv(D.Cout, 4), 128), 128, 0, st>>>(c);
            }
            rc = launched("conv3");
            end();
            if (rc) return rc;
            beg(b, "epi1", "epi", px * D.Cout);
            rc = run_epi(nullptr, Q.c1, Q.res, Q.h1, D.A1, D.Bm1, D.pw1, D.tap2, Q.t2, N, D.Cout, HW, st);
            end();
            if (rc) return rc;
        } else {
            const bool dec = b >= 5;
            const RBuf* skip = dec ? &d->buf[8 - b] : nullptr;  // dec4 <- enc4 (b=5 -> 3) ...
            beg(b, dec ? "upcat+proj" : "proj", "proj", px * D.Cout * D.Cin);
            if (dec)
                rc = run_proj(D, skip->out, d->blk[8 - b].Cout, xin, xc, xh, xw, N, h, w, blocked, Q.res, Q.t1, st);
            else
                rc = run_proj(D, xin, D.Cin, nullptr, 0, 0, 0, N, h, w, blocked, Q.res, Q.t1, st);
            end();
            if (rc) return rc;
            beg(b, "conv1", "bconv", px * D.Cout * D.Cin * 9.0);
            rc = run_bconv(D.conv1, Q.t1, N, h, w, Q.P1, d->scratch, st);
            end();
            if (rc) return rc;
            beg(b, "epi1", "epi", px * D.Cout);
            rc = run_epi(Q.P1, nullptr, Q.res, Q.h1, D.A1, D.Bm1, D.pw1, D.tap2, Q.t2, N, D.Cout, HW, st);
            end();
            if (rc) return rc;
        }
        // ---- unit2
        beg(b, "conv2", "bconv", px * D.Cout * D.Cout * 9.0);
        rc = run_bconv(D.conv2, Q.t2, N, h, w, Q.P2, d->scratch, st);
        end();
        if (rc) return rc;
        if (B.is_down) {
            react::SkipPoolParams sp{Q.P2, Q.h1, Q.out, Q.down, D.Aa, D.Bma, D.pwa, D.Ab, D.Bmb, D.pwb,
                                     N, D.Cout, h, w};
            beg(b, "skip+pool+down", "epi", px * D.Cout);
            react::skip_pool_kernel<<<dim3(cdiv((long long)N * ((h + 1) / 2) * ((w + 1) / 2), 256),
                                           (unsigned)cdiv(D.Cout, 16)),
                                      256, 0, st>>>(sp);
            rc = launched("skip / pool epilogue");
            end();
            if (rc) return rc;
            xin = Q.down; xc = D.Cout; xh = h / 2; xw = w / 2;
        } else {
            beg(b, "epi2", "epi", px * D.Cout);
            rc = run_epi(Q.P2, nullptr, Q.h1, Q.out, D.Aa, D.Bma, D.pwa, nullptr, nullptr, N, D.Cout, HW, st);
            end();
            if (rc) return rc;
            xin = Q.out; xc = D.Cout; xh = h; xw = w;
        }
    }
    react::HeadParams hp{xin, d->headW, d->headb, logits, N, m->head_Cin, m->head_Cout, H * W};
    if (pc && pc->prof) pc->begin("head", "head", (double)N * H * W * m->head_Cout * m->head_Cin);
    const bool hv4 = (H * W) % 4 == 0 && (((uintptr_t)xin | (uintptr_t)logits) & 15) == 0;
    const unsigned hg = (unsigned)cdiv((long long)N * H * W / (hv4 ? 4 : 1), 256);
    if (hv4 && m->head_Cout == 3) react::head_kernel<4, 3><<<hg, 256, 0, st>>>(hp);
    else if (hv4) react::head_kernel<4, react::HEADR_MAXC><<<hg, 256, 0, st>>>(hp);
    else react::head_kernel<1, react::HEADR_MAXC><<<hg, 256, 0, st>>>(hp);
    rc = launched("head");
    end();
    return rc;
}

int check_hw(const ModelR* m, int N, int H, int W) {
    if (N < 0) return set_error(BNN_ERR_ARG, "N = %d", N);
    // below 16 a pooled level is empty and the reference's 2x2 max-pools
    // read past their input (csrc/bnn_react_opt.c:48, (H-2)/2+1 = 1 at H = 1)
    if (H < 16 || W < 16) return set_error(BNN_ERR_ARG, "H=%d W=%d: the ReAct forward needs H, W >= 16", H, W);
    if ((long long)N * H * W >= (1ll << 31)) return set_error(BNN_ERR_ARG, "N*H*W too large");
    if (m->head_Cout > react::HEADR_MAXC) return set_error(BNN_ERR_UNSUPPORTED, "n_classes > %d", react::HEADR_MAXC);
    return BNN_OK;
}

int forward_device(const ModelR* m, RDev* d, const float* x, int N, int H, int W, float* logits, cudaStream_t user) {
    int rc = arena(m, d, N, H, W);
    if (rc || N == 0) return rc;
    REngine* E = (REngine*)m->engine;
    RCK(cudaStreamWaitEvent(user, d->ev_last, 0));
    if ((rc = poison(d, user))) return rc;
    if (E->prof.on) {
        RProf pc;
        pc.prof = &E->prof;
        pc.st = user;
        if ((rc = forward_launches(m, d, x, N, H, W, logits, user, &pc))) return rc;
        RCK(cudaEventRecord(d->ev_last, user));
        return pc.finish();
    }
    GraphKeyR key{N, H, W, x, logits};
    auto it = d->graphs.find(key);
    if (it == d->graphs.end()) {
        cudaGraph_t g = nullptr;
        RCK(cudaStreamBeginCapture(d->cs, cudaStreamCaptureModeThreadLocal));
        rc = forward_launches(m, d, x, N, H, W, logits, d->cs, nullptr);
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
    RCK(cudaGraphLaunch(it->second, user));
    RCK(cudaEventRecord(d->ev_last, user));
    return BNN_OK;
}

int current_device(int* dev) {
    if (cudaGetDevice(dev) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_CUDA, "no CUDA device available");
    }
    return BNN_OK;
}

// host batch on the current device: chunks through two device staging
// slots, host->device copies on one stream, forwards on the compute stream,
// device->host copies on a third, so chunk i's compute overlaps chunk i+1's
// upload and chunk i-1's download (end to end this is bound by the host link)
int host_batch(const ModelR* m, const float* in, int N, int H, int W, float* out) {
    int rc = check_hw(m, N, H, W);
    if (rc || N == 0) return rc;
    int dev = 0;
    if ((rc = current_device(&dev))) return rc;
    RDev* d = nullptr;
    if ((rc = get_rdev(m, dev, &d))) return rc;
    std::lock_guard<std::mutex> g(d->mu);
    RCK(cudaSetDevice(dev));
    const size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    // chunk: about 64 MB of input, at least 1 patch, at most N
    const int chunk = (int)std::max<size_t>(1, std::min<size_t>((size_t)N, ((size_t)64 << 20) / (ip * 4)));
    if (d->pcap < (size_t)chunk || d->pin_floats != ip || d->pout_floats != op) {
        RCK(cudaStreamSynchronize(d->h2d));
        RCK(cudaStreamSynchronize(d->d2h));
        RCK(cudaStreamSynchronize(d->cs));
        for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
        d->graphs.clear();
        for (int k = 0; k < 2; ++k) {
            cudaFree(d->pin[k]);
            cudaFree(d->pout[k]);
            d->pin[k] = d->pout[k] = nullptr;
        }
        d->pcap = 0;
        for (int k = 0; k < 2; ++k)
            if (cudaMalloc(&d->pin[k], ip * chunk * 4) != cudaSuccess ||
                cudaMalloc(&d->pout[k], op * chunk * 4) != cudaSuccess) {
                cudaGetLastError();
                return set_error(BNN_ERR_OOM, "cudaMalloc ReAct staging");
            }
        d->pcap = chunk;
        d->pin_floats = ip;
        d->pout_floats = op;
    }
    int i = 0;
    for (int s0 = 0; s0 < N && !rc; s0 += chunk, ++i) {
        const int n = std::min(chunk, N - s0), k = i & 1;
        // slot k's input is free once its previous forward ran; its output
        // once its previous download ran
        if (cudaStreamWaitEvent(d->h2d, d->ev_comp[k], 0) != cudaSuccess ||
            cudaMemcpyAsync(d->pin[k], in + ip * s0, ip * n * 4, cudaMemcpyHostToDevice, d->h2d) != cudaSuccess ||
            cudaEventRecord(d->ev_in[k], d->h2d) != cudaSuccess || cudaStreamWaitEvent(d->cs, d->ev_in[k], 0) != cudaSuccess ||
            cudaStreamWaitEvent(d->cs, d->ev_out[k], 0) != cudaSuccess) {
            rc = set_error(BNN_ERR_CUDA, "H2D: %s", cudaGetErrorString(cudaGetLastError()));
            break;
        }
        if ((rc = forward_device(m, d, d->pin[k], n, H, W, d->pout[k], d->cs))) break;
        if (cudaEventRecord(d->ev_comp[k], d->cs) != cudaSuccess || cudaStreamWaitEvent(d->d2h, d->ev_comp[k], 0) != cudaSuccess ||
            cudaMemcpyAsync(out + op * s0, d->pout[k], op * n * 4, cudaMemcpyDeviceToHost, d->d2h) != cudaSuccess ||
            cudaEventRecord(d->ev_out[k], d->d2h) != cudaSuccess)
            rc = set_error(BNN_ERR_CUDA, "D2H: %s", cudaGetErrorString(cudaGetLastError()));
    }
    cudaError_t e1 = cudaStreamSynchronize(d->d2h), e2 = cudaStreamSynchronize(d->cs), e3 = cudaStreamSynchronize(d->h2d);
    if (!rc && (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess))
        rc = set_error(BNN_ERR_CUDA, "ReAct forward: %s", cudaGetErrorString(cudaGetLastError()));
    return rc;
}

}  // namespace

void* react_engine_create() { return new (std::nothrow) REngine(); }

void react_engine_destroy(void* e) {
    REngine* E = (REngine*)e;
    if (!E) return;
    for (auto& kv : E->devs) rdev_release(kv.second.get());
    delete E;
}

}  // namespace bnn

using namespace bnn;

BNN_API int bnn_forward_react_batch(const ModelR* m, const float* input, int N, int H, int W, float* logits) {
    if (!m || !input || !logits) return set_error(BNN_ERR_ARG, "NULL argument");
    return host_batch(m, input, N, H, W, logits);
}

BNN_API int bnn_forward_react_device(const ModelR* m, int device, const float* d_input, int N, int H, int W,
                                     float* d_logits, void* stream) {
    if (!m || !d_input || !d_logits) return set_error(BNN_ERR_ARG, "NULL argument");
    int rc = check_hw(m, N, H, W);
    if (rc) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_ARG, "cannot select device %d", device);
    }
    RDev* d = nullptr;
    rc = get_rdev(m, device, &d);
    if (!rc) {
        std::lock_guard<std::mutex> g(d->mu);
        rc = forward_device(m, d, d_input, N, H, W, d_logits, (cudaStream_t)stream);
    }
    cudaSetDevice(prev);
    return rc;
}

BNN_API void bnn_forward_react(const ModelR* m, const float* input, int H, int W, float* logits) {
    if (bnn_forward_react_batch(m, input, 1, H, W, logits) != BNN_OK) {
        fprintf(stderr, "%s\n", bnn_last_error());
        exit(1);
    }
}

// the reference's tiler (csrc/bnn_model_react.c:454-476): zero-padded PxP
// tiles, each a standalone forward, stitched; all tiles in one batch
BNN_API int bnn_forward_react_patched_ex(const ModelR* m, const float* input, int H, int W, float* logits, int P) {
    if (!m || !input || !logits) return set_error(BNN_ERR_ARG, "NULL argument");
    if (P < 16 || P % 16 || H <= 0 || W <= 0)
        return set_error(BNN_ERR_ARG, "H=%d W=%d P=%d: P must be a multiple of 16", H, W, P);
    const int nb = m->n_bands, ncl = m->n_classes, ty = cdiv(H, P), tx = cdiv(W, P), nt = ty * tx;
    std::vector<float> tin((size_t)nt * nb * P * P, 0.0f), tout((size_t)nt * ncl * P * P);
    for (int a = 0; a < ty; ++a)
        for (int b = 0; b < tx; ++b) {
            const int py = a * P, px = b * P, ph = std::min(P, H - py), pw = std::min(P, W - px);
            float* t = tin.data() + (size_t)(a * tx + b) * nb * P * P;
            for (int c = 0; c < nb; ++c)
                for (int y = 0; y < ph; ++y)
                    memcpy(t + ((size_t)c * P + y) * P, input + ((size_t)c * H + py + y) * W + px, (size_t)pw * 4);
        }
    int rc = bnn_forward_react_batch(m, tin.data(), nt, P, P, tout.data());
    if (rc) return rc;
    for (int a = 0; a < ty; ++a)
        for (int b = 0; b < tx; ++b) {
            const int py = a * P, px = b * P, ph = std::min(P, H - py), pw = std::min(P, W - px);
            const float* t = tout.data() + (size_t)(a * tx + b) * ncl * P * P;
            for (int c = 0; c < ncl; ++c)
                for (int y = 0; y < ph; ++y)
                    memcpy(logits + ((size_t)c * H + py + y) * W + px, t + ((size_t)c * P + y) * P, (size_t)pw * 4);
        }
    return BNN_OK;
}

BNN_API void bnn_forward_react_patched(const ModelR* m, const float* input, int H, int W, float* logits, int P) {
    if (bnn_forward_react_patched_ex(m, input, H, W, logits, P) != BNN_OK) {
        fprintf(stderr, "%s\n", bnn_last_error());
        exit(1);
    }
}

static std::vector<float> read_cube(const ModelR* m, FILE* f, int H, int W) {
    std::vector<float> x((size_t)m->n_bands * H * W);
    if (!f || fseek(f, 0, SEEK_SET) != 0 || fread(x.data(), 4, x.size(), f) != x.size()) {
        fprintf(stderr, "file_reader: short read of the [%d,%d,%d] cube\n", m->n_bands, H, W);
        exit(1);
    }
    return x;
}

// the file forms read the cube and run the in-memory forwards (the
// reference streams strips to bound host memory; the values are the same)
BNN_API void bnn_forward_react_file(const ModelR* m, FILE* in_f, int H, int W, float* logits) {
    std::vector<float> x = read_cube(m, in_f, H, W);
    bnn_forward_react(m, x.data(), H, W, logits);
}

BNN_API void bnn_forward_react_patched_file(const ModelR* m, FILE* f, int H, int W, float* logits, int P) {
    std::vector<float> x = read_cube(m, f, H, W);
    bnn_forward_react_patched(m, x.data(), H, W, logits, P);
}

BNN_API int bnn_forward_react_stages(const ModelR* m, const float* input, int H, int W, float* logits,
                                     bnn_stage_cb cb, void* ctx) {
    if (!m || !input || !logits || !cb) return set_error(BNN_ERR_ARG, "NULL argument");
    int rc = check_hw(m, 1, H, W);
    if (rc) return rc;
    int dev = 0;
    if ((rc = current_device(&dev))) return rc;
    RDev* d = nullptr;
    if ((rc = get_rdev(m, dev, &d))) return rc;
    std::lock_guard<std::mutex> g(d->mu);
    if ((rc = arena(m, d, 1, H, W))) return rc;
    const size_t ip = (size_t)m->n_bands * H * W, op = (size_t)m->n_classes * H * W;
    float *din = nullptr, *dout = nullptr;
    int8_t* d8 = nullptr;
    size_t maxc = 0;
    for (int b = 0; b < 9; ++b) maxc = std::max(maxc, (size_t)std::max(d->blk[b].Cin, d->blk[b].Cout) * d->buf[b].h * d->buf[b].w);
    if (cudaMalloc(&din, ip * 4) != cudaSuccess || cudaMalloc(&dout, op * 4) != cudaSuccess ||
        cudaMalloc(&d8, maxc) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(din);
        cudaFree(dout);
        return set_error(BNN_ERR_OOM, "cudaMalloc stage buffers");
    }
    auto fail = [&](int code) { cudaFree(din); cudaFree(dout); cudaFree(d8); return code; };
    if (cudaMemcpy(din, input, ip * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(set_error(BNN_ERR_CUDA, "H2D"));
    if ((rc = poison(d, d->cs))) return fail(rc);
    if ((rc = forward_launches(m, d, din, 1, H, W, dout, d->cs, nullptr))) return fail(rc);
    if (cudaStreamSynchronize(d->cs) != cudaSuccess)
        return fail(set_error(BNN_ERR_CUDA, "ReAct forward: %s", cudaGetErrorString(cudaGetLastError())));
    std::vector<char> host;
    auto fl = [&](const char* blk, const char* st, const float* dp, int C, int h, int w) {
        host.resize((size_t)C * h * w * 4);
        cudaMemcpy(host.data(), dp, host.size(), cudaMemcpyDeviceToHost);
        cb(ctx, (std::string(blk) + "." + st).c_str(), 2, C, h, w, host.data());
    };
    auto in32 = [&](const char* blk, const char* st, const int32_t* dp, int C, int h, int w) {
        host.resize((size_t)C * h * w * 4);
        cudaMemcpy(host.data(), dp, host.size(), cudaMemcpyDeviceToHost);
        cb(ctx, (std::string(blk) + "." + st).c_str(), 1, C, h, w, host.data());
    };
    auto bits = [&](const char* blk, const char* st, const uint32_t* dp, int C, int h, int w) {
        react::unpack_bits_kernel<<<std::max(1, std::min(cdiv((long long)C * h * w, 256), 148 * 8)), 256, 0, d->cs>>>(
            dp, 1, C, h * w, d8);
        cudaStreamSynchronize(d->cs);
        host.resize((size_t)C * h * w);
        cudaMemcpy(host.data(), d8, host.size(), cudaMemcpyDeviceToHost);
        cb(ctx, (std::string(blk) + "." + st).c_str(), 0, C, h, w, host.data());
    };
    for (int b = 0; b < 9; ++b) {
        const RBlockDev& D = d->blk[b];
        const RBuf& Q = d->buf[b];
        const int h = Q.h, w = Q.w;
        fl(BN[b], "proj", Q.res, D.Cout, h, w);
        if (b == 0) fl(BN[b], "conv1.out", Q.c1, D.Cout, h, w);
        else {
            bits(BN[b], "tap1", Q.t1, D.Cin, h, w);
            in32(BN[b], "conv1.P", Q.P1, D.Cout, h, w);
        }
        fl(BN[b], "h1", Q.h1, D.Cout, h, w);
        bits(BN[b], "tap2", Q.t2, D.Cout, h, w);
        in32(BN[b], "conv2.P", Q.P2, D.Cout, h, w);
        if (b < 4) {
            fl(BN[b], "skip", Q.out, D.Cout, h, w);
            fl(BN[b], "down", Q.down, D.Cout, h / 2, w / 2);
        } else {
            fl(BN[b], "h2", Q.out, D.Cout, h, w);
        }
    }
    cudaMemcpy(logits, dout, op * 4, cudaMemcpyDeviceToHost);
    cb(ctx, "logits", 2, m->n_classes, H, W, logits);
    return fail(BNN_OK);
}

BNN_API int bnn_react_profile_enable(ModelR* m, int on) {
    if (!m || !m->engine) return set_error(BNN_ERR_ARG, "NULL model");
    ((REngine*)m->engine)->prof.on = on != 0;
    return BNN_OK;
}

BNN_API void bnn_react_profile_reset(ModelR* m) {
    if (!m || !m->engine) return;
    REngine* E = (REngine*)m->engine;
    std::lock_guard<std::mutex> g(E->prof.mu);
    E->prof.recs.clear();
}

BNN_API int bnn_react_profile_count(const ModelR* m) {
    if (!m || !m->engine) return 0;
    REngine* E = (REngine*)m->engine;
    std::lock_guard<std::mutex> g(E->prof.mu);
    return (int)E->prof.recs.size();
}

BNN_API int bnn_react_profile_get(const ModelR* m, int i, const char** label, const char** optype, double* work,
                                  double* ms, int* calls) {
    if (!m || !m->engine) return set_error(BNN_ERR_ARG, "NULL model");
    REngine* E = (REngine*)m->engine;
    std::lock_guard<std::mutex> g(E->prof.mu);
    if (i < 0 || i >= (int)E->prof.recs.size()) return set_error(BNN_ERR_ARG, "record %d out of range", i);
    const auto& r = E->prof.recs[i];
    if (label) *label = r.label.c_str();
    if (optype) *optype = r.optype.c_str();
    if (work) *work = r.work;
    if (ms) *ms = r.ms;
    if (calls) *calls = r.calls;
    return BNN_OK;
}

BNN_API int bnn_react_set_conv_kernel(int kind) {
    if (kind != 0 && kind != 1) return set_error(BNN_ERR_ARG, "ReAct conv kernel kind %d (0 = TMA, 1 = plain)", kind);
    g_conv3_kind = kind;
    return BNN_OK;
}

BNN_API int bnn_react_device_error(int device, unsigned int* wait_timeouts) {
    if (!wait_timeouts) return set_error(BNN_ERR_ARG, "NULL argument");
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return set_error(BNN_ERR_ARG, "cannot select device %d", device);
    }
    cudaError_t e = cudaMemcpyFromSymbol(wait_timeouts, react::g_react_wait_timeouts, sizeof(unsigned int));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(BNN_ERR_CUDA, "read wait counter: %s", cudaGetErrorString(e));
    return BNN_OK;
}

BNN_API int bnn_react_forward_launches(const ModelR* m, int N, int H, int W) {
    if (!m || N <= 0 || H < 16 || W < 16) return 0;
    // every block: proj, conv1 (enc1: the real conv), epi1, conv2, one
    // closing epilogue (encoder: skip + pooled down in one pass); head
    return 9 * 5 + 1;
}
