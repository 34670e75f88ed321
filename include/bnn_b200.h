/* bnn_b200.h - extensions of the B200 binary-UNet engine beyond the
 * reference's three-call API (bnn_model.h). Plain C ABI: pointers, sizes and
 * int status codes only; `stream` arguments are cudaStream_t passed as
 * void* (NULL = the legacy default stream).
 *
 * Bit-packed activation layout used by every device-pointer call:
 *   uint32 [N][H][W][ceil(C/32)], channel c -> bit (c & 31) of word (c >> 5),
 *   bit 1 = +1, bit 0 = -1, unused high bits of the last word are 0.
 *
 * Each entry point notes the reference interface it replaces or extends
 * (paths within Sboyle132/BNNs_to_C).
 */
#ifndef BNN_B200_H
#define BNN_B200_H
#include <stddef.h>
#include <stdint.h>
#include "bnn_model.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    BNN_OK = 0,
    BNN_ERR_IO = 1,          /* file cannot be opened / read */
    BNN_ERR_FORMAT = 2,      /* blob violates the v1 layout (reference bnn_model.c:66-96) */
    BNN_ERR_UNSUPPORTED = 3, /* valid blob, but a topology bnn_forward cannot run */
    BNN_ERR_ARG = 4,         /* bad argument (size, pointer, device) */
    BNN_ERR_CUDA = 5,        /* CUDA runtime error (message names the call) */
    BNN_ERR_OOM = 6          /* host or device allocation failed */
};

/* Message of the last failing call on this host thread ("" if none). */
const char *bnn_last_error(void);

/* Status-returning forms of bnn_load (reference csrc/bnn_model.c:66-96):
 * identical parsing and the same error conditions, but no exit(). The
 * in-memory form parses `n` bytes at `data`. */
int bnn_load_ex(const char *path, Model **out);
int bnn_load_mem(const void *data, size_t n, Model **out);

/* Batched forward with host pointers: input [N][n_bands][H][W] float32 ->
 * logits [N][n_classes][H][W] float32; each patch's result equals
 * bnn_forward on that patch (reference csrc/bnn_model.c:150-253). Patches
 * are sharded by index in contiguous slices over the Model's devices
 * (bnn_set_devices), one host thread per device; on each device copies in,
 * compute and copies out overlap chunk by chunk. Page-locked host buffers
 * (cudaHostAlloc / cudaHostRegister) give full copy bandwidth. Blocks until
 * the logits are in host memory. */
int bnn_forward_batch(const Model *m, const float *input, int N, int H, int W,
                      float *logits);

/* Batched forward on device memory of `device`: enqueued on `stream`,
 * returns without synchronising. d_input and d_logits must stay valid until
 * the stream reaches this work. Repeated calls with the same (N, H, W) on
 * the same stream replay one captured CUDA graph. */
int bnn_forward_device(const Model *m, int device, const float *d_input, int N,
                       int H, int W, float *d_logits, void *stream);

/* Patch-wise forward of a whole scene: the reference's tiler
 * (bnn_forward_react_patched, csrc/bnn_model_react.c:454-476, same
 * signature) applied to the v1 network. The [n_bands][H][W] cube is cut into
 * non-overlapping PxP tiles, zero-padded past the right and bottom edges,
 * each tile runs through the full network as a standalone PxP image, and the
 * in-scene part of its logits is stitched into [n_classes][H][W]. Tile rows
 * are split over the Model's devices (bnn_set_devices). Host pointers;
 * blocks until the logits are in host memory. P >= 16. */
int bnn_forward_patched(const Model *m, const float *input, int H, int W,
                        float *logits, int P);

/* The same on device memory of `device`, enqueued on `stream` (tiles are
 * gathered and stitched on the GPU, in chunks of 4096 tiles). */
int bnn_forward_patched_device(const Model *m, int device, const float *d_cube,
                               int H, int W, int P, float *d_logits,
                               void *stream);

/* Process-wide choice of the binary-conv kernel, for measurement and A/B
 * parity tests: 0 = tcgen05 (default): int8 MMAs, and e2m1 MMAs
 * (kind::mxf4: +-1 exact in 4 bits, 64 channels per instruction, fp32
 * accumulators holding exact integers) for the non-pooled 64- and
 * 128-channel layers with at least 4 input words and the 256-channel ones
 * with at least 16, where they measured faster; mma.sync int8 where the
 * staging does not fit; 1 = XOR + POPC on
 * the integer pipe; 2 = mma.sync int8 for every layer; 3 = as 4, but layers
 * of at most 32 channels without a pool take the kernel with a kernel row's
 * three column taps stacked in N (measured slower); 4 = tcgen05 int8 MMAs
 * for every layer; 5 = e2m1 MMAs for every non-pooled layer. All compute
 * the reference's P exactly; set it before the forwards to compare
 * (captured graphs keep the kernels they captured). */
int bnn_set_bconv_kernel(int kind);

/* Process-wide choice of the first conv's tensor-core kernel (A/B testing):
 * 0 = tcgen05, nine shifted taps (default; shapes it cannot stage fall back
 * to 1), 1 = mma.sync, 2 = tcgen05 with the three column taps of a kernel
 * row stacked in the MMA's N where the width divides 32 (kind 0 for other
 * widths), 3 = tcgen05 with the weights in the MMA's M (kernel-row taps x
 * channels) and the staged positions in N (kind 0 where it cannot stage).
 * All decide every output by the same error bound and fix up the rest in
 * the reference's fp32 order, so all give the reference's bits. For a v2
 * model's stem: 0 = the measured-faster of its two exact-order kernels for
 * the stem's width (register-streamed up to 16 channels, input streamed by
 * bulk copies through a shared-memory ring above), 1 = the other one. */
int bnn_set_first_conv_kernel(int kind);

/* Debug fill of the activation arenas (the v1 / v2 engine's and the ReAct
 * engine's), the device-side form of csrc/bnn_react_arena.c:30-32: with a
 * byte set, every forward first writes that byte over its whole arena (bit
 * planes, int32 planes, the undecided-output list), so a kernel that reads
 * what no earlier launch of the same forward wrote changes the logits. The
 * byte comes from BNN_ARENA_POISON (its integer value & 255) the first
 * time it is needed, unless bnn_set_arena_poison set it: -1 = off (the
 * default), 0..255 = the byte. bnn_arena_poison returns the byte in force
 * (-1 = off). One cudaMemsetAsync per forward when on, nothing when off. */
int bnn_set_arena_poison(int byte);
int bnn_arena_poison(void);

/* Number of bounded device-side waits (mbarriers of the TMA / tcgen05
 * pipelines) that gave up on `device` since the library was loaded; a
 * non-zero count means some output of those launches is not to be trusted.
 * Expected to stay 0. */
int bnn_device_error(int device, unsigned int *wait_timeouts);

/* Synchronous calls (bnn_forward, bnn_forward_batch, bnn_forward_patched,
 * bnn_gpu_bconv_dispatch and its allocation-free twin) compare that count
 * before and after their own launches and return BNN_ERR_CUDA (bnn_forward:
 * print + exit(1)) when it went up. The asynchronous device-pointer calls
 * leave it to the caller to poll bnn_device_error. */

/* Self-test of the bounded device wait (no reference counterpart): one
 * thread waits on an mbarrier phase that nothing completes, for `rounds`
 * try_wait rounds (1 .. 2^22; the pipelines use 2^22, seconds in total),
 * gives up and records it exactly as a pipeline CTA does. *gave_up = 1 when
 * the wait returned "not completed" and set its abort flag; *timeouts gets
 * the device counter afterwards. The context stays usable. */
int bnn_wait_probe(int device, int rounds, int *gave_up, unsigned int *timeouts);

/* Host-side fault injection for tests of the failure paths (no reference
 * counterpart; nothing faults or stalls a GPU):
 *   BNN_FAULT_ALLOC: the arg-th next device allocation made by the engine
 *     (weights, activation arena, staging) fails as an out-of-memory
 *     cudaMalloc would (BNN_ERR_OOM);
 *   BNN_FAULT_WAIT: the next synchronous call queues, after its own
 *     launches, one bounded wait that gives up (bnn_wait_probe's kernel with
 *     a short limit), so the call must report BNN_ERR_CUDA;
 *   BNN_FAULT_SHARD: host thread `arg` of the next multi-device
 *     bnn_forward_batch fails before it launches anything; the others run,
 *     and the error is returned after every thread has been joined.
 * kind 0 clears every pending injection. Each injection fires once. */
#define BNN_FAULT_ALLOC 1
#define BNN_FAULT_WAIT 2
#define BNN_FAULT_SHARD 3
int bnn_debug_inject_fault(int kind, int arg);

/* Name and template parameters of the last binary-conv kernel the calling
 * thread launched (bnn_bconv_layer_run, a forward, the dispatch shims),
 * e.g. "bconv_ws_kernel<64,4,i8,8> (tcgen05 kind::i8)"; "" before any. */
const char *bnn_bconv_last_kernel(void);

/* Devices used by bnn_forward_batch, in shard order. n = 0 restores the
 * default: the calling thread's current device. */
int bnn_set_devices(Model *m, const int *devices, int n);
int bnn_get_devices(const Model *m, int *devices, int cap);

/* Patches per pipelined chunk in bnn_forward_batch (default 256). */
int bnn_set_chunk(Model *m, int patches);

/* Debug / parity: one patch on the current device, every intermediate
 * copied back and reported in bnn_forward's order with the names
 * "<block>.conv<k>.P" (int32 [C][H][W]), "<block>.<act>" (int8 +-1
 * [C][H][W]), "enc1.conv1.out" (float32, the real conv output),
 * "<block>.pool.P", "<dec>.cat" (int8; 0 where the upsample does not
 * reach, as in the reference's up_cat) and "logits". kind: 0 int8, 1 int32,
 * 2 float32. The stages are the reference forward's intermediates
 * (csrc/bnn_model.c:150-253), which its own forward frees unseen. */
typedef void (*bnn_stage_cb)(void *ctx, const char *name, int kind, int C,
                             int H, int W, const void *data);
int bnn_forward_stages(const Model *m, const float *input, int H, int W,
                       float *logits, bnn_stage_cb cb, void *ctx);

/* Per-op profiler: the reference's PROF/prof_report (csrc/bnn_prof.h:13-32,
 * csrc/bnn_prof.c:42-77) done with CUDA events around each kernel launch.
 * While enabled, forwards launch eagerly (no graph) and accumulate
 * per-label device time. Work units as the reference: out_elems * taps. */
int bnn_profile_enable(Model *m, int on);
void bnn_profile_reset(Model *m);
int bnn_profile_count(const Model *m);
int bnn_profile_get(const Model *m, int i, const char **label,
                    const char **optype, double *work, double *ms, int *calls);
void bnn_profile_report(const Model *m, void *file /* FILE* */);

/* GPU-backed host-pointer form of the reference's bconv_dispatch
 * (csrc/bnn_conv.c:216-223, same signature and result): int8 +-1 input
 * [Cin][H][W] (values <= 0 count as -1, as in the reference), kidx-packed
 * weights, int32 P [Cout][Ho][Wo]. kh = kw = 3, stride 1, pad 0 or 1. */
int bnn_gpu_bconv_dispatch(const int8_t *a, const uint64_t *packed_w, int32_t *P,
                           int Cin, int H, int W, int Cout, int kh, int kw,
                           int pad, int stride);

/* Allocation-free twin of bnn_gpu_bconv_dispatch: same arguments, same
 * result, but it never calls cudaMalloc or cudaFree (nor any allocating
 * library routine). It has no counterpart in the reference: it is for
 * callers that cannot let this library allocate device memory - processes
 * whose GPU memory is fixed up front by their own allocator or budget, and
 * latency-bound loops that cannot take the device-wide synchronisation of
 * cudaFree. Its staging buffers live in one static device array of
 * BNN_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
 * the process exits; a call whose buffers do not fit returns BNN_ERR_ARG
 * before touching the GPU (it needs about 1.2*Cin*H*W + 8*Cout*H*W +
 * 11.3*CoutP*Cin bytes with CoutP = Cout rounded up to 128, each buffer
 * rounded up to 256). The weights it stages are those of the mma.sync
 * kernel (bconv_mma_kernel), so this path always runs that kernel (or the
 * XOR/POPC one under bnn_set_bconv_kernel(1)), never the tcgen05 kernels
 * of the allocating twin: same result bit for bit, lower throughput.
 * Every call looks up that array's device address with the device current;
 * the first call on a device also sets the kernels' shared-memory
 * attributes, so make that first call before any stream capture. All calls
 * share the one array and it keeps the last call's
 * contents: calls that overlap on the GPU (from several host threads on one
 * device) race, so serialise them. Runs on the current device and returns
 * when P is in host memory. */
#define BNN_NOALLOC_SCRATCH_BYTES (32u << 20)
int bnn_gpu_bconv_dispatch_noalloc(const int8_t *a, const uint64_t *packed_w,
                                   int32_t *P, int Cin, int H, int W, int Cout,
                                   int kh, int kw, int pad, int stride);

/* GPU-backed host-pointer form of conv_realin_naive for the 3x3 pad-1
 * stride-1 first conv (csrc/bnn_conv_realin.c:66-116,165-172): bit-identical
 * float32 output, same operation order. */
int bnn_gpu_conv_realin(const float *x, const int8_t *wsign, const float *alpha,
                        float *out, int Cin, int H, int W, int Cout, int kh,
                        int kw, int pad, int stride);

/* One fused binary 3x3 conv layer on device buffers (the isolated-kernel
 * benchmark): P (reference bconv_dispatch, csrc/bnn_conv.c:216-223) ->
 * per-channel integer fold (apply_fold_int, csrc/bnn_fold.c:37-60) -> bit
 * pack; optionally also 2x2 max-pool of P (maxpool_P, csrc/bnn_maxpool.c:
 * 28-48) -> second fold -> bit pack. The accumulator never leaves the chip
 * unless d_P / d_Ppool are given (debug). Weights: kidx-packed uint64
 * [Cout][ceil(9*Cin/64)] as in the blob; fold arrays: [Cout] each; the
 * pooled fold arrays may be NULL (no pooled output). */
typedef struct bnn_bconv_layer bnn_bconv_layer;
int bnn_bconv_layer_create(int device, int Cin, int Cout,
                           const uint64_t *packed_kidx, const int32_t *type,
                           const int32_t *t, const int32_t *lo, const int32_t *hi,
                           const int32_t *pool_type, const int32_t *pool_t,
                           const int32_t *pool_lo, const int32_t *pool_hi,
                           bnn_bconv_layer **out);
int bnn_bconv_layer_run(const bnn_bconv_layer *L, const uint32_t *d_in, int N,
                        int H, int W, uint32_t *d_out, uint32_t *d_out_pool,
                        int32_t *d_P, int32_t *d_Ppool, void *stream);
void bnn_bconv_layer_destroy(bnn_bconv_layer *L);

/* Seeded synthetic patches (bnn_synth.h) written on `device`:
 * [N][bands][H][W] float32 for patch indices first..first+N-1. */
int bnn_synth_device(int device, uint32_t seed, uint32_t first_patch, int N,
                     int bands, int H, int W, float *d_out, void *stream);

/* int8 +-1 [N][C][H][W] <-> bit-packed [N][H][W][ceil(C/32)] on device
 * (values > 0 -> bit 1). */
int bnn_pack_act_device(const int8_t *d_a, int N, int C, int H, int W,
                        uint32_t *d_bits, void *stream);
int bnn_unpack_act_device(const uint32_t *d_bits, int N, int C, int H, int W,
                          int8_t *d_a, void *stream);

/* The first conv + real fold alone (enc1.conv1 -> enc1.act1 bit plane,
 * reference csrc/bnn_model.c:156-167) on device memory: d_input [N][bands]
 * [H][W] float32 -> d_bits [N][H][W][ceil(C/32)]. exact = 0 runs the
 * production path (int8 tensor cores decided by an error bound, undecided
 * outputs recomputed in the reference's fp32 order); exact = 1 runs the
 * all-fp32 exact-order kernel. Both give the reference's bits. If
 * `undecided` is not NULL the call synchronises and stores how many outputs
 * the production path sent to the exact fix-up (0xffffffff: the list
 * overflowed and the whole batch was recomputed exactly). On the engine
 * handle of a v2 model (bnn_stem_as_model) it runs the stem + stem fold
 * instead (csrc/bnn_model_stem.c:172-187), whose kernel is exact-order by
 * construction: `exact` is ignored and `undecided` gets 0. */
int bnn_first_conv_device(const Model *m, int device, const float *d_input,
                          int N, int H, int W, uint32_t *d_bits, int exact,
                          unsigned int *undecided, void *stream);

/* Number of this library's kernel launches one forward of (N, H, W)
 * issues (for launch accounting in benchmarks). */
int bnn_forward_launches(const Model *m, int N, int H, int W);

#ifdef __cplusplus
}
#endif
#endif
