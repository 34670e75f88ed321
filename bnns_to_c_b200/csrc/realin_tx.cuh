// realin_tx.cuh - the first conv on tcgen05 with the weights as the A
// operand and the staged positions in N (included by engine.cu after
// kernels.cuh).
//
// Numerics are those of realin_ws_kernel: the input as three int8 planes of
// q = rint(x * 2^18), exact plane sums from the MMAs, the same per-position
// error bound and fold thresholds, undecided outputs listed for
// realin_fixup_kernel. What changes is the shape of the MMAs.
//
// realin_ws_kernel puts 128 positions in M and the 32 channels in N: every
// MMA reads a 4 KB A tile for a 1 KB B tile, and each tap reads the plane
// again (27 A tiles per 32-band chunk and tile), so shared-memory operand
// bandwidth bounds it. Here A = the weights of one kernel row dy, rows
// dx*32 + co (96 rows; the descriptor's last 32 rows read the next block,
// whose results land in TMEM lanes nobody reads), and B = the staged plane
// from position dy*Wp, N = 144 positions. TMEM lane dx*32 + co, column n of
// plane accumulator pl then holds sum_dy w[co][dy][dx] . x[n + dy*Wp], and
// the output at staged position Wp + 1 + j is
//     Q0[j] + Q1[j + 1] + Q2[j + 2]    (Qdx = the dx lane quarter)
// with Q = S_0 << 16 + S_1 << 8 + S_2 over the three planes. Per 32-band
// chunk an item takes 9 MMAs (3 planes x 3 kernel rows) reading 3 B tiles
// of 4.5 KB per plane, against 54 MMAs and 270 KB in realin_ws_kernel.
//
// An item is R rows of one image (R*Wp <= 142 outputs), staged as in
// realin_ws_kernel: rows y0-1 .. y0+R, W pixels plus one zero column,
// flattened (position = row*Wp + col). TMEM: the three plane accumulators,
// 144 columns each, one item at a time; the epilogue drains them into
// registers at once so the next item's MMAs can start.
//
// Warps (16): 0-2 and 4-6 epilogue (warp w reads TMEM lanes 32*(w%4)..,
// columns 72*(w/4)..; lane quarter 3 holds only the unused rows, so warps
// 3 and 7 are producers), 3, 7, 8-13 producers (the first also drives the
// TMA ring), 14-15 MMA issue (issuer 0: planes 0 and 2, issuer 1: plane 1;
// warp 15 allocates TMEM). The lane quarters 0 and 2 hand their sums to
// quarter 1 through shared memory (mbarriers xfull / xempty); quarter 1
// writes the output sums back (sfull), and every epilogue thread decides
// one output position for all 32 channels (thresholds by constant index,
// rows padded to 33 words: no bank conflicts either way).
// Every wait is bounded; a CTA that gives up raises ctl[1] (the fix-up then
// recomputes the whole batch).
// ---------------------------------------------------------------------
#pragma once

namespace bnn {

constexpr int TX_N = 144;           // D columns per plane (N of every MMA)
constexpr int TX_TO = TX_N - 2;     // outputs per item at most
constexpr int TX_NPROD = 256;       // warps 3, 7, 8-13
constexpr int TX_NQ = 2;            // staged positions per producer thread, at most
constexpr int TX_MAX_SP = TX_NPROD * TX_NQ;
constexpr int TX_NT = 512;
constexpr int TX_NEPI = 192;        // warps 0-2, 4-6
constexpr int TX_NQ1 = 64;          // warps 1 and 5: lane quarter 1
// quarter 0 (then the sums) [column][33] and quarter 2 [column][32], int32
constexpr size_t TX_XBYTES = (size_t)TX_N * (33 + 32) * 4;
constexpr size_t TX_MAX_SMEM = (size_t)224 * 1024;

__host__ __device__ inline size_t tx_box_bytes(int W, int R) { return (size_t)W * (R + 2) * 32 * 4; }
__host__ __device__ inline size_t tx_stage_bytes(int SP) { return (size_t)3 * 2 * SP * 16; }
// weights (+ one box ring) first: the last weight block's overhanging 32
// descriptor rows read the start of the boxes
__host__ __device__ inline size_t tx_fixed_bytes(int W, int R, int SP) {
    return RX_WBYTES + RW_NB * tx_box_bytes(W, R) + TX_XBYTES + (size_t)2 * SP * 4;
}

// 8 consecutive TMEM columns of this thread's lane (no wait)
__device__ __forceinline__ void tc_ld8_nw(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
// wait for every outstanding tcgen05.ld, tied to 24 registers (three x8 loads)
__device__ __forceinline__ void tc_wait_ld24(uint32_t* a, uint32_t* b, uint32_t* c) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]), "+r"(c[4]), "+r"(c[5]), "+r"(c[6]), "+r"(c[7])
                 :
                 : "memory");
}

__global__ void __launch_bounds__(TX_NT, 1) realin_tx_kernel(const __grid_constant__ CUtensorMap tmap,
                                                            const RealinWsParams p) {
    extern __shared__ __align__(1024) unsigned char tx_smem[];
    __shared__ __align__(8) unsigned long long boxf_b[RW_NB], boxe_b[RW_NB], full_b[4], empty_b[4], accf_b, acce_b,
        xfull_b, xempty_b, sfull_b, bpxf_b[2], bpxe_b[2], wrdy_b;
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s;
    volatile int* abort_v = &abort_s;

    const int SP = p.SP, Wp = p.Wp, R = p.R, NS = p.NS, KC = p.KC;
    const size_t box_bytes = tx_box_bytes(p.W, R), stage_bytes = tx_stage_bytes(SP);
    unsigned char* boxes = tx_smem + RX_WBYTES;                          // [RW_NB][32][R+2][W] f32
    unsigned char* stages = boxes + RW_NB * box_bytes;                   // [NS][3 planes][2 halves][SP][16]
    int* xq = reinterpret_cast<int*>(stages + NS * stage_bytes);         // quarters 0 and 2 (TX_XBYTES)
    float* bpx = reinterpret_cast<float*>(xq + TX_N * (33 + 32));         // [2][SP] error bound per position
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int my_items = (int)blockIdx.x < p.n_items ? (p.n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (warp == 15) {
        tc_alloc(smem_u32(&tmem_s), 512);
        tc_relinquish();
    }
    if (tid == 0) {
        abort_s = 0;
        for (int b = 0; b < RW_NB; ++b) {
            mbar_init(smem_u32(&boxf_b[b]), 1);
            mbar_init(smem_u32(&boxe_b[b]), TX_NPROD);
        }
        for (int s = 0; s < NS; ++s) {
            mbar_init(smem_u32(&full_b[s]), TX_NPROD);
            mbar_init(smem_u32(&empty_b[s]), 2);
        }
        mbar_init(smem_u32(&accf_b), 2);
        mbar_init(smem_u32(&acce_b), TX_NEPI);
        mbar_init(smem_u32(&xfull_b), TX_NEPI - TX_NQ1);
        mbar_init(smem_u32(&xempty_b), TX_NEPI);
        mbar_init(smem_u32(&sfull_b), TX_NQ1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&bpxf_b[b]), TX_NPROD);
            mbar_init(smem_u32(&bpxe_b[b]), TX_NEPI);
        }
        mbar_init(smem_u32(&wrdy_b), 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    const uint32_t sm0 = smem_u32(tx_smem);
    const bool producer = warp == 3 || warp == 7 || (warp >= 8 && warp < 14);

    if (producer) {
        // ------------------------------------------------------------ producers
        const int pt = (warp == 3 ? 0 : warp == 7 ? 1 : warp - 6) * 32 + lane;
        const int nseq = my_items * KC;
        auto issue_box = [&](int seq) {  // TMA of chunk kc of item seq/KC into buffer seq % RW_NB
            const int item = (int)blockIdx.x + (seq / KC) * (int)gridDim.x, kc = seq % KC;
            const int n = item / p.ipi, y0 = (item - n * p.ipi) * R;
            const uint32_t bar = smem_u32(&boxf_b[seq % RW_NB]);
            mbar_expect_tx(bar, (uint32_t)box_bytes);
            tma_load_4d(sm0 + (uint32_t)(RX_WBYTES + (seq % RW_NB) * box_bytes), &tmap, 0, y0 - 1, kc * 32, n, bar);
        };
        if (pt == 0) {
            // the weights once per CTA, then the first boxes
            mbar_expect_tx(smem_u32(&wrdy_b), (uint32_t)RX_WBYTES);
            bulk_g2s(sm0, p.wu, (uint32_t)RX_WBYTES, smem_u32(&wrdy_b));
            for (int s = 0; s < RW_NB && s < nseq; ++s) issue_box(s);
        }
        int stage = 0, seq = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int it = 0; it < my_items && ok && !*abort_v; ++it) {
            // per staged position: sum |x| and sum (Cin - band) |x| (both rounded up)
            float tsum[TX_NQ], wsum[TX_NQ], amax[TX_NQ];
#pragma unroll
            for (int j = 0; j < TX_NQ; ++j) { tsum[j] = 0.0f; wsum[j] = 0.0f; amax[j] = 0.0f; }
            for (int kc = 0; kc < KC; ++kc, ++seq) {
                const int bb = seq % RW_NB;
                if (pt == 0 && seq >= 1 && seq + RW_NB - 1 < nseq) {
                    // refill the buffer of chunk seq-1 with chunk seq+RW_NB-1 once
                    // every producer is done with it
                    if (!mbar_wait_ab(smem_u32(&boxe_b[(seq - 1) % RW_NB]), (uint32_t)((seq - 1) / RW_NB) & 1u,
                                      abort_v)) { ok = false; break; }
                    issue_box(seq + RW_NB - 1);
                }
                if (!mbar_wait_ab(smem_u32(&boxf_b[bb]), (uint32_t)(seq / RW_NB) & 1u, abort_v)) { ok = false; break; }
                if (!mbar_wait_ab(smem_u32(&empty_b[stage]), phase ^ 1u, abort_v)) { ok = false; break; }
                const float* bx = reinterpret_cast<const float*>(boxes + bb * box_bytes);
                unsigned char* st = stages + stage * stage_bytes;
                const size_t bstride = (size_t)(R + 2) * p.W;  // floats between bands in the box
#pragma unroll
                for (int j = 0; j < TX_NQ; ++j) {
                    const int q = pt + TX_NPROD * j;
                    if (q < SP) {
                        const int row = q / Wp, col = q - row * Wp;
                        // plane 0 = byte 2 (signed), plane 1 = byte 1, plane 2 = byte 0; word k = bands 4k..4k+3
                        uint32_t w[3][8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) w[0][k] = w[1][k] = w[2][k] = 0u;
                        if (col >= 1 && row < R + 2) {
                            const float* src = bx + (size_t)row * p.W + (col - 1);
#pragma unroll
                            for (int g2 = 0; g2 < 4; g2 += 2) {  // 16 bands loaded at once
                                float xv[16];
#pragma unroll
                                for (int i = 0; i < 16; ++i) xv[i] = src[(size_t)(g2 * 8 + i) * bstride];
                                // the error-bound sums exactly as realin_ws_kernel forms them
                                float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                                for (int i = 0; i < 16; i += 2) {
                                    s0 = __fadd_ru(s0, fabsf(xv[i]));
                                    s1 = __fadd_ru(s1, fabsf(xv[i + 1]));
                                    amax[j] = fmaxf(amax[j], fmaxf(fabsf(xv[i]), fabsf(xv[i + 1])));
                                }
                                const float s01 = __fadd_ru(s0, s1);
                                tsum[j] = __fadd_ru(tsum[j], s01);
                                wsum[j] = __fmaf_ru(fmaxf((float)(p.Cin - kc * 32 - g2 * 8), 0.0f), s01, wsum[j]);
#pragma unroll
                                for (int g = g2; g < g2 + 2; ++g) {
                                    uint32_t qv[8];
#pragma unroll
                                    for (int i = 0; i < 8; ++i)
                                        qv[i] = (uint32_t)(__float_as_int(__fmaf_rn(xv[(g - g2) * 8 + i],
                                                                                    (float)(1 << RM_FIX), 12582912.0f)) -
                                                           0x4B400000);
#pragma unroll
                                    for (int h = 0; h < 2; ++h) {
                                        const uint32_t lo0 = __byte_perm(qv[h * 4 + 0], qv[h * 4 + 1], 0x5140);
                                        const uint32_t hi0 = __byte_perm(qv[h * 4 + 2], qv[h * 4 + 3], 0x5140);
                                        w[2][g * 2 + h] = __byte_perm(lo0, hi0, 0x5410);  // bytes 0
                                        w[1][g * 2 + h] = __byte_perm(lo0, hi0, 0x7632);  // bytes 1
                                        w[0][g * 2 + h] = __byte_perm(__byte_perm(qv[h * 4 + 0], qv[h * 4 + 1], 0x6262),
                                                                      __byte_perm(qv[h * 4 + 2], qv[h * 4 + 3], 0x6262),
                                                                      0x5410);  // bytes 2
                                    }
                                }
                            }
                        }
#pragma unroll
                        for (int pl = 0; pl < 3; ++pl) {
                            *reinterpret_cast<uint4*>(st + ((size_t)(pl * 2) * SP + q) * 16) =
                                make_uint4(w[pl][0], w[pl][1], w[pl][2], w[pl][3]);
                            *reinterpret_cast<uint4*>(st + ((size_t)(pl * 2 + 1) * SP + q) * 16) =
                                make_uint4(w[pl][4], w[pl][5], w[pl][6], w[pl][7]);
                        }
                    }
                }
                fence_async_smem();
                mbar_arrive(smem_u32(&full_b[stage]));
                mbar_arrive(smem_u32(&boxe_b[bb]));
                if (++stage == NS) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            // error bounds of this item's staged positions, once the deciders
            // are done with the item that used this table two items ago
            const int buf = it & 1;
            if (!mbar_wait_ab(smem_u32(&bpxe_b[buf]), (uint32_t)((it >> 1) & 1) ^ 1u, abort_v)) break;
            float* bt = bpx + buf * SP;
            const float rnd = __fmul_ru((float)p.Cin, 1.0f / (float)(1 << (RM_FIX + 1)));
#pragma unroll
            for (int j = 0; j < TX_NQ; ++j) {
                const int q = pt + TX_NPROD * j;
                if (q < SP) {
                    const int row = q / Wp, col = q - row * Wp;
                    float e = 0.0f;  // zero columns and positions past the box are exact zeros
                    if (col >= 1 && row < R + 2)
                        e = amax[j] < 16.0f ? __fmaf_ru(p.ca, wsum[j], __fmaf_ru(p.cb, tsum[j], rnd))
                                            : __int_as_float(0x7f800000);
                    bt[q] = e;  // NaN inputs: the sums are NaN, and so is e
                }
            }
            mbar_arrive(smem_u32(&bpxf_b[buf]));
        }
    } else if (warp >= 14) {
        // ------------------------------------------------------------ MMA issuers
        const int u = warp - 14;
        if (lane == 0 && mbar_wait_ab(smem_u32(&wrdy_b), 0u, abort_v)) {
            // A = weights (signed); B = a plane: plane 0 signed, planes 1-2 unsigned; D s32; M = 128, N = TX_N
            const uint32_t id_s =
                (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TX_N >> 3) << 17) | ((128u >> 4) << 24);
            const uint32_t id_u = (2u << 4) | (1u << 7) | ((uint32_t)(TX_N >> 3) << 17) | ((128u >> 4) << 24);
            const uint32_t st0 = sm0 + (uint32_t)(RX_WBYTES + RW_NB * box_bytes);
            int stage = 0;
            uint32_t phase = 0;
            for (int it = 0; it < my_items && !*abort_v; ++it) {
                // the epilogue has drained the previous item's accumulators
                if (!mbar_wait_ab(smem_u32(&acce_b), (uint32_t)(it & 1) ^ 1u, abort_v)) break;
                tc_fence_after();
                bool ok = true;
                for (int kc = 0; kc < KC; ++kc) {
                    if (!mbar_wait_ab(smem_u32(&full_b[stage]), phase, abort_v)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t st_s = st0 + (uint32_t)(stage * stage_bytes);
#pragma unroll 1
                    for (int pl = u; pl < 3; pl += 2) {  // issuer 0: planes 0 and 2, issuer 1: plane 1
                        const uint32_t id = pl == 0 ? id_s : id_u;
#pragma unroll
                        for (int dy = 0; dy < 3; ++dy) {
                            // weights [chunk][kernel row][16-band half][dx*32 + co][16 bands]
                            const uint64_t ad = tc_desc(sm0 + (uint32_t)((kc * 3 + dy) * 2 * 96 * 16), 96 * 16);
                            const uint64_t bd =
                                tc_desc(st_s + (uint32_t)(((pl * 2) * SP + dy * Wp) * 16), (uint32_t)SP * 16);
                            // an item's first MMA into each plane accumulator overwrites it
                            tc_mma_i8(tmem + (uint32_t)(pl * TX_N), ad, bd, id, (kc | dy) ? 1u : 0u);
                        }
                    }
                    tc_commit(smem_u32(&empty_b[stage]));
                    if (++stage == NS) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(smem_u32(&accf_b));
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue (warps 0-2, 4-6)
        const int quad = warp & 3, half = warp >> 2, c0 = half * 72;
        const int et = (warp < 4 ? warp : warp - 1) * 32 + lane;  // 0..191
        const uint32_t tq = tmem + ((uint32_t)(quad * 32) << 16);
        int* xs = xq;                                   // quarter 0, then the sums: [TX_N][33]
        int* x2 = xq + TX_N * 33;                       // quarter 2: [TX_N][32]
        for (int it = 0; it < my_items && !*abort_v; ++it) {
            const int item = (int)blockIdx.x + it * (int)gridDim.x;
            const int n = item / p.ipi, y0 = (item - n * p.ipi) * R;
            if (!mbar_wait_ab(smem_u32(&accf_b), (uint32_t)(it & 1), abort_v)) break;
            tc_fence_after();
            // drain: Q = S_0 << 16 + S_1 << 8 + S_2 for this lane's 72 columns
            // (|S_0| <= 3*128*64 and S_1, S_2 <= 3*128*255: Q fits in 31 bits)
            int Q[72];
#pragma unroll
            for (int ch = 0; ch < 9; ++ch) {
                uint32_t a[8], b[8], c[8];
                tc_ld8_nw(tq + (uint32_t)(c0 + ch * 8), a);
                tc_ld8_nw(tq + (uint32_t)(TX_N + c0 + ch * 8), b);
                tc_ld8_nw(tq + (uint32_t)(2 * TX_N + c0 + ch * 8), c);
                tc_wait_ld24(a, b, c);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    Q[ch * 8 + i] = (int)(((uint32_t)a[i] << 16) + ((uint32_t)b[i] << 8) + (uint32_t)c[i]);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&acce_b));
            if (quad != 1) {
                // lane quarters 0 and 2 hand their sums to quarter 1, once every
                // decider is done with the previous item's
                if (!mbar_wait_ab(smem_u32(&xempty_b), (uint32_t)(it & 1) ^ 1u, abort_v)) break;
                if (quad == 0) {
#pragma unroll
                    for (int i = 0; i < 72; ++i) xs[(c0 + i) * 33 + lane] = Q[i];
                } else {
#pragma unroll
                    for (int i = 0; i < 72; ++i) x2[(c0 + i) * 32 + lane] = Q[i];
                }
                mbar_arrive(smem_u32(&xfull_b));
            } else {
                // quarter 1: the sum of output j = 71*half + jj (staged position
                // Wp + 1 + j) is Q0[j] + Q1[j + 1] + Q2[j + 2], written over Q0[j]
                if (!mbar_wait_ab(smem_u32(&xfull_b), (uint32_t)(it & 1), abort_v)) break;
                const int j0 = 71 * half;
#pragma unroll
                for (int jj = 0; jj < 71; ++jj) {
                    const int j = j0 + jj;
                    // Q1[j + 1] is this lane's Q[jj + 1] (half 0) or Q[jj] (half 1): indices stay compile-time
                    const int q1 = half == 0 ? Q[jj + 1] : Q[jj];
                    xs[j * 33 + lane] += q1 + x2[(j + 2) * 32 + lane];
                }
                mbar_arrive(smem_u32(&sfull_b));
            }
            // every epilogue thread decides one output position for all channels
            if (!mbar_wait_ab(smem_u32(&sfull_b), (uint32_t)(it & 1), abort_v)) break;
            const int buf = it & 1;
            if (!mbar_wait_ab(smem_u32(&bpxf_b[buf]), (uint32_t)((it >> 1) & 1), abort_v)) break;
            if (et < TX_TO) {
                const float* bt = bpx + buf * SP;
                const int ol = Wp + 1 + et;
                const int orow = ol / Wp, ocol = ol - orow * Wp;
                const int yl = y0 + orow - 1;
                if (orow <= R && ocol >= 1 && yl < p.H) {
                    float ef = 0.0f;
#pragma unroll
                    for (int t = 0; t < 9; ++t) ef = __fadd_ru(ef, bt[ol + (t / 3 - 1) * Wp + (t % 3 - 1)]);
                    // E = ceil(e * 2^18) (exact scaling); e past 2^40, inf or NaN: nothing is decided
                    const bool fin = ef <= 1.0995116e12f;
                    const long long E = fin ? __float2ll_ru(ef * 262144.0f) : 0ll;
                    const int* srow = xs + et * 33;
                    uint32_t bits = 0u, und = 0u;
#pragma unroll
                    for (int co = 0; co < 32; ++co) {
                        if (co < p.Cout) {
                            const long long Q = (long long)srow[co];
                            const long long Qs = (p.thr_neg >> co) & 1u ? -Q : Q;
                            const long long C = p.thrC[co];
                            const bool ok = fin && !((p.thr_exact >> co) & 1u);
                            if (ok && Qs - E >= C) bits |= 1u << co;
                            else if (!(ok && Qs + E < C)) und |= 1u << co;
                        }
                    }
                    const size_t pix = ((size_t)n * p.H + yl) * p.W + (ocol - 1);
                    p.out[pix * p.cwo] = bits;
                    if (und) realin_list(p.list, p.ctl, p.cap, pix, 0, und);
                }
            }
            mbar_arrive(smem_u32(&xempty_b));
            mbar_arrive(smem_u32(&bpxe_b[buf]));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (abort_s) {
        // let any MMA or copy still in flight land before TMEM and shared
        // memory are released; the fix-up then recomputes the batch exactly
        for (int i = 0; i < (1 << 16); ++i) __nanosleep(1000);
        if (tid == 0) {
            atomicExch(p.ctl + 1, 1u);
            atomicAdd(&g_bnn_wait_timeouts, 1u);
        }
    }
    if (warp == 15) {
        tc_fence_after();
        tc_dealloc(tmem, 512);
    }
}

}  // namespace bnn
