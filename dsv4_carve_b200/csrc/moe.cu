// moe.cu -- routed-expert MoE decode layer for sm_100a, one launch per layer.
//
// Replaces the lna2 ticket kernel (recipe-lna/lna2/lna_moe_ticket.cu:240-429)
// with the same numerics contract (lna_moe_ticket.cu:5-12):
//   x -> fp16; gate/up accumulate fp32; output Hadamard + svh fp32;
//   silu(min(g, L)) * clamp(u, -L, L) fp32 -> fp16; down-input suh + Hadamard
//   -> fp16; down accumulate fp32; output Hadamard + svh fp32; weighted sum
//   over top-k slots in slot order, fp32; one cast to the output dtype.
//
// Structure (B200 design, not the reference's): every CTA builds the same
// route plan in shared memory (groups = experts in ascending id, pairs =
// unique (expert, row)).  Work is a flat ticket space of units:
//   phase A  (group, 128-col block j of inter, gate|up, k-chunk s of hidden)
//   phase B  (group, 128-col block c of hidden, k-chunk s of inter)
// all phase-A tickets before all phase-B tickets.  Partials go to scratch;
// the last unit of (group, j) finishes gate+up block j and writes the
// down-input block (SwiGLU + suh + Hadamard) -- the last unit of (group, c)
// finishes down block c -- the last group to finish block c does the
// fixed-order gather of that block.  Phase-B units wait (bounded) on a
// per-(group, chunk) counter.  Every ticket comes from one global counter, so
// when a CTA holds a phase-B ticket every phase-A ticket has already been
// claimed by a running CTA; a CTA works its tickets in claim order and
// phase-A units never wait, so each wait is on work that is in progress and
// progress needs no co-residency and no grid barrier.
#include <mutex>

#include "engine.cuh"
#include "host.hpp"

namespace exl3 {

constexpr int kMoeMaxRows = 32;      // row bitmask is one 32-bit word
constexpr int kMoeMaxSlots = 256;    // m * topk
constexpr int kMoeMaxExperts = 1024;
constexpr int kMoeMaxTopk = 16;
constexpr int kMoeKmax = 4;          // ring slot sized for K <= 4
constexpr int kMoeMaxHidden = 8192;
constexpr int kMoeMaxInter = 4096;
// Counter strides (per group) inside the control region.
constexpr int kStrideA = kMoeMaxInter / 128;    // cntA[g][j]
constexpr int kStrideR = kMoeMaxInter / 128;    // readyB[g][s]
constexpr int kStrideB = kMoeMaxHidden / 128;   // cntB[g][c]
constexpr int kCtrlWords = 16;
constexpr int64_t kMoeCtrlNeeded =
    4LL * (kCtrlWords + (int64_t) kMoeMaxSlots * (kStrideA + kStrideR + kStrideB) + kStrideB);
static_assert(kMoeCtrlNeeded <= EXL3_MOE_CTRL_BYTES, "control region too small");

struct MoeParams {
    const void* x;
    void* out;
    const int64_t* tab[9];      // gate t/su/sv, up t/su/sv, down t/su/sv
    const int32_t* ktab;        // per-expert K, or null (then kuni)
    const int32_t* ids;
    const float* weights;
    int x_dtype, out_dtype;
    int m, H, I, topk, E, kuni;
    float limit;
    int kca, nka;               // gate/up k-chunk over H
    int kcb, nkb;               // down k-chunk over I
    uint32_t* ctrl;             // [0] ticket [1] retire [2] status
    uint32_t* cntA;
    uint32_t* readyB;
    uint32_t* cntB;
    uint32_t* cntG;
    float* partA;               // [pairs][2][nka][I]
    __half* act;                // [pairs][I]
    float* partB;               // [pairs][nkb][H]
    float* downc;               // [pairs][H]
};

struct MoeCfg {
    static constexpr int SK = stage_slices(kMoeKmax);
    static constexpr int STAGE = SK * 8 * TileFmt<kMoeKmax>::BYTES;
    static constexpr int NS = 49152 / STAGE;
};

struct MoePlan {
    uint32_t emask[kMoeMaxExperts];   // row bitmask per expert
    int epair[kMoeMaxExperts];        // first pair of the expert
    int wsum[2][kConsumerWarps];      // scan scratch
    short gexp[kMoeMaxSlots];         // group -> expert
    short gpair[kMoeMaxSlots];        // group -> first pair
    uint32_t gmask[kMoeMaxSlots];     // group -> row bitmask
    short slotpair[kMoeMaxSlots];     // slot -> pair (-1 if skipped)
    int G, P;
};

struct alignas(128) MoeSmem {
    uint8_t ring[MoeCfg::NS][MoeCfg::STAGE];
    uint4 bfrag[kActBytes / 16];
    float cbuf[kMaxRows * kCols];
    MoePlan plan;
    uint64_t full[MoeCfg::NS];
    uint64_t empty[MoeCfg::NS];
    uint64_t dqf[kDQ];
    uint64_t dqe[kDQ];
    int desc[kDQ][6];                 // kind, g, mat, blk, s, K
    int rows[kMaxRows];
    int flag;
};

// Route plan, identical in every CTA (recipe-lna/lna2/lna_moe_ticket.cu:167-214
// restated): per-expert row mask, exclusive scans over experts -> group id and
// first pair, slot -> pair via popcount.  Uses the 256 consumer threads.
__device__ void build_plan(MoePlan& P, const MoeParams& p, int tid) {
    const bool worker = tid < kConsumerThreads;
    for (int e = tid; e < p.E; e += kThreads) P.emask[e] = 0u;
    __syncthreads();
    const int nslots = p.m * p.topk;
    for (int s = tid; s < nslots; s += kThreads) {
        const int id = p.ids[s];
        if (id >= 0 && id < p.E) atomicOr(&P.emask[id], 1u << (s / p.topk));
    }
    __syncthreads();
    // Each worker thread owns experts [4t, 4t+4) (E <= 1024).
    const int warp = tid >> 5, lane = tid & 31;
    int has[4] = {0, 0, 0, 0}, pop[4] = {0, 0, 0, 0};
    int lh = 0, lp = 0;
    if (worker) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int e = tid * 4 + q;
            const uint32_t mk = e < p.E ? P.emask[e] : 0u;
            has[q] = mk != 0u;
            pop[q] = __popc(mk);
            lh += has[q];
            lp += pop[q];
        }
    }
    int ih = lh, ip = lp;   // inclusive warp scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, ih, o);
        const int b = __shfl_up_sync(0xffffffffu, ip, o);
        if (lane >= o) { ih += a; ip += b; }
    }
    if (worker && lane == 31) { P.wsum[0][warp] = ih; P.wsum[1][warp] = ip; }
    __syncthreads();
    if (worker) {
        int bh = 0, bp = 0;
        for (int w = 0; w < warp; ++w) { bh += P.wsum[0][w]; bp += P.wsum[1][w]; }
        int gh = bh + ih - lh, gp = bp + ip - lp;   // exclusive prefix of this thread
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int e = tid * 4 + q;
            if (e < p.E) {
                P.epair[e] = gp;
                if (has[q]) {
                    P.gexp[gh] = (short) e;
                    P.gpair[gh] = (short) gp;
                    P.gmask[gh] = P.emask[e];
                }
            }
            gh += has[q];
            gp += pop[q];
        }
        if (tid == kConsumerThreads - 1) { P.G = gh; P.P = gp; }
    }
    __syncthreads();
    for (int s = tid; s < nslots; s += kThreads) {
        const int id = p.ids[s];
        short sp = -1;
        if (id >= 0 && id < p.E) {
            const int row = s / p.topk;
            sp = (short) (P.epair[id] + __popc(P.emask[id] & ((1u << row) - 1u)));
        }
        P.slotpair[s] = sp;
    }
    __syncthreads();
}

// Consume one unit's stages for a runtime K / row-block count.
template <int CB, bool PRECISE, int K>
__device__ __forceinline__ bool moe_consume_k(MoeSmem& S, uint32_t& it, int nst, int RB, float (&acc)[4][4],
                                              int cwarp, int lane, uint32_t* status) {
    const LaneGeom<K> geom = lane_geom<K>(lane);
    // The ring slot is sized for kMoeKmax; a K-bit stage uses its first bytes.
    auto ring = S.ring;
    switch (RB) {
        case 1: return consume_stages<K, CB, 1, MoeCfg::NS, MoeCfg::STAGE, MoeCfg::SK, PRECISE>(ring, S.full, S.empty, it, nst, 0, S.bfrag, acc, geom, cwarp, lane, status);
        case 2: return consume_stages<K, CB, 2, MoeCfg::NS, MoeCfg::STAGE, MoeCfg::SK, PRECISE>(ring, S.full, S.empty, it, nst, 0, S.bfrag, acc, geom, cwarp, lane, status);
        case 3: return consume_stages<K, CB, 3, MoeCfg::NS, MoeCfg::STAGE, MoeCfg::SK, PRECISE>(ring, S.full, S.empty, it, nst, 0, S.bfrag, acc, geom, cwarp, lane, status);
        default: return consume_stages<K, CB, 4, MoeCfg::NS, MoeCfg::STAGE, MoeCfg::SK, PRECISE>(ring, S.full, S.empty, it, nst, 0, S.bfrag, acc, geom, cwarp, lane, status);
    }
}

template <int CB, bool PRECISE>
__device__ __forceinline__ bool moe_consume(MoeSmem& S, uint32_t& it, int nst, int K, int RB, float (&acc)[4][4],
                                            int cwarp, int lane, uint32_t* status) {
    switch (K) {
        case 1: return moe_consume_k<CB, PRECISE, 1>(S, it, nst, RB, acc, cwarp, lane, status);
        case 2: return moe_consume_k<CB, PRECISE, 2>(S, it, nst, RB, acc, cwarp, lane, status);
        case 3: return moe_consume_k<CB, PRECISE, 3>(S, it, nst, RB, acc, cwarp, lane, status);
        default: return moe_consume_k<CB, PRECISE, 4>(S, it, nst, RB, acc, cwarp, lane, status);
    }
}

__device__ __forceinline__ int unit_count_A(const MoeParams& p, int G) { return G * (p.I / kCols) * 2 * p.nka; }
__device__ __forceinline__ int unit_count_B(const MoeParams& p, int G) { return G * (p.H / kCols) * p.nkb; }

template <int CB, bool PRECISE>
__global__ void __launch_bounds__(kThreads, 2) moe_kernel(MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    MoeSmem& S = *reinterpret_cast<MoeSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* status = p.ctrl + 2;

    if (tid == 0) {
        for (int s = 0; s < MoeCfg::NS; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], kConsumerWarps); }
        for (int s = 0; s < kDQ; ++s) { mbar_init(&S.dqf[s], 1); mbar_init(&S.dqe[s], 1); }
        fence_barrier_init();
    }
    build_plan(S.plan, p, tid);
    const MoePlan& P = S.plan;
    const int G = P.G;
    const int NBI = p.I / kCols, NBH = p.H / kCols;
    const int UA = unit_count_A(p, G);
    const int total = UA + unit_count_B(p, G);

    if (G == 0 && blockIdx.x == 0) {
        // No valid route: the layer output is zero.
        for (int i = tid; i < p.m * p.H; i += kThreads) store_out(p.out, p.out_dtype, i, 0.f);
    }

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------- producer
        int ticket = claim_ticket(&p.ctrl[0], lane);
        uint32_t it = 0, du = 0;
        bool ok = true;
        while (ok) {
            int d[6] = {-1, 0, 0, 0, 0, 0};
            const uint8_t* src = nullptr;
            int64_t rowstride = 0;
            int nst = 0, K = 0;
            if (ticket < total) {
                int g, mat = 0, blk, s, kind;
                if (ticket < UA) {
                    kind = 0;
                    const int per = NBI * 2 * p.nka;
                    g = ticket / per;
                    int r = ticket % per;
                    blk = r / (2 * p.nka);
                    r %= 2 * p.nka;
                    mat = r / p.nka;
                    s = r % p.nka;
                } else {
                    kind = 1;
                    const int t2 = ticket - UA;
                    const int per = NBH * p.nkb;
                    g = t2 / per;
                    const int r = t2 % per;
                    blk = r / p.nkb;
                    s = r % p.nkb;
                }
                const int e = P.gexp[g];
                K = p.ktab ? p.ktab[e] : p.kuni;
                d[0] = kind; d[1] = g; d[2] = mat; d[3] = blk; d[4] = s; d[5] = K;
                if (K >= 1 && K <= kMoeKmax) {
                    const int tb = 32 * K;
                    if (kind == 0) {
                        src = reinterpret_cast<const uint8_t*>(p.tab[mat ? 3 : 0][e]);
                        rowstride = (int64_t) (p.I / 16) * tb;
                        src += (int64_t) s * (p.kca / 16) * rowstride + (int64_t) blk * 8 * tb;
                        nst = p.kca / (16 * MoeCfg::SK);
                    } else {
                        src = reinterpret_cast<const uint8_t*>(p.tab[6][e]);
                        rowstride = (int64_t) (p.H / 16) * tb;
                        src += (int64_t) s * (p.kcb / 16) * rowstride + (int64_t) blk * 8 * tb;
                        nst = p.kcb / (16 * MoeCfg::SK);
                    }
                } else {
                    d[5] = 0;   // consumers skip the unit (error recorded)
                }
            }
            if (lane == 0) {
                const int slot = du % kDQ;
                ok = mbar_wait(&S.dqe[slot], ((du / kDQ) + 1u) & 1u, status);
                if (ok) {
#pragma unroll
                    for (int q = 0; q < 6; ++q) S.desc[slot][q] = d[q];
                    mbar_arrive(&S.dqf[slot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            ++du;
            if (d[0] < 0 || !ok) break;
            if (d[5] == 0) {
                if (lane == 0) set_error(status, ERR_BAD_K);
            } else {
                const int rowbytes = 8 * 32 * K;
                const bool valid = aligned16_dev(src) && (rowstride & 15) == 0;
                if (!valid && lane == 0) set_error(status, ERR_MISALIGNED);
                for (int st = 0; st < nst && ok; ++st)
                    ok = produce_stage<MoeCfg::NS, MoeCfg::STAGE>(S.ring, S.full, S.empty, it,
                                                                  src + (int64_t) st * MoeCfg::SK * rowstride,
                                                                  rowstride, rowbytes, MoeCfg::SK, valid, lane,
                                                                  status);
            }
            ticket = claim_ticket(&p.ctrl[0], lane);
        }
        drain_ring<MoeCfg::NS>(S.full, it, lane, status);
    } else {
        // ---------------------------------------------------------- consumers
        const int ctid = tid;
        uint32_t it = 0, du = 0;
        while (true) {
            const int slot = du % kDQ;
            if (!consumers_all(mbar_wait_warp(&S.dqf[slot], (du / kDQ) & 1u, status, lane))) break;
            int d[6];
#pragma unroll
            for (int q = 0; q < 6; ++q) d[q] = S.desc[slot][q];
            consumers_sync();
            if (ctid == 0) mbar_arrive(&S.dqe[slot]);
            ++du;
            if (d[0] < 0) break;
            const int kind = d[0], g = d[1], mat = d[2], blk = d[3], s = d[4], K = d[5];
            if (K == 0) continue;
            const int e = P.gexp[g];
            const uint32_t gm = P.gmask[g];
            const int nrows = __popc(gm);
            const int pair0 = P.gpair[g];
            const int RB = row_blocks(nrows);
            if (ctid < kMaxRows) {
                int r = -1;
                if (ctid < nrows) {
                    if (kind == 0) {
                        // ctid-th set bit of the row mask
                        uint32_t mk = gm;
                        for (int q = 0; q < ctid; ++q) mk &= mk - 1u;
                        r = __ffs((int) mk) - 1;
                    } else {
                        r = pair0 + ctid;
                    }
                }
                S.rows[ctid] = r;
            }
            if (kind == 1 && ctid == 0) {
                // down input chunk s of this group must be complete
                wait_counter(&p.readyB[g * kStrideR + s], (uint32_t) (p.kcb / kCols), status);
            }
            consumers_sync();

            const int kc = kind == 0 ? p.kca : p.kcb;
            const int kslices = kc / 16;
            const int sub0 = (act_slices(RB) / 16) * 16;
            const int sub = sub0 < kslices ? sub0 : kslices;
            float acc[4][4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
            bool ok = true;
            for (int ks0 = 0; ks0 < kslices && ok; ks0 += sub) {
                const int nks = min(sub, kslices - ks0);
                if (ks0 > 0) consumers_sync();
                if (kind == 0) {
                    const __half* suh = reinterpret_cast<const __half*>(p.tab[mat ? 4 : 1][e]);
                    build_bfrag<PRECISE>(S.bfrag, RB, nrows, S.rows, p.x, p.x_dtype, p.H, s * kslices + ks0, nks,
                                         suh, warp, lane);
                } else {
                    build_bfrag<PRECISE>(S.bfrag, RB, nrows, S.rows, p.act, 0, p.I, s * kslices + ks0, nks, nullptr,
                                         warp, lane);
                }
                consumers_sync();
                ok = consumers_all(moe_consume<CB, PRECISE>(S, it, nks / MoeCfg::SK, K, RB, acc, warp, lane, status));
            }
            if (!consumers_all(ok)) break;
            acc_to_cbuf(S.cbuf, acc, RB, warp, lane);
            consumers_sync();

            if (kind == 0) {
                // ---- phase A: partial, then maybe finish gate+up block blk
                for (int idx = ctid; idx < nrows * kCols; idx += kConsumerThreads) {
                    const int r = idx / kCols, c = idx % kCols;
                    p.partA[(((int64_t) (pair0 + r) * 2 + mat) * p.nka + s) * p.I + blk * kCols + c] = S.cbuf[idx];
                }
                consumers_sync();
                if (ctid == 0) {
                    __threadfence();   // release: covers every consumer's writes (ordered by the barrier)
                    const uint32_t old = atomicAdd(&p.cntA[g * kStrideA + blk], 1u);
                    const int last = old == (uint32_t) (2 * p.nka - 1);
                    if (last) {
                        atomicExch(&p.cntA[g * kStrideA + blk], 0u);
                        __threadfence();   // acquire: the other units' partials
                    }
                    S.flag = last;
                }
                consumers_sync();
                if (S.flag) {
                    const __half* gsv = reinterpret_cast<const __half*>(p.tab[2][e]) + blk * kCols;
                    const __half* usv = reinterpret_cast<const __half*>(p.tab[5][e]) + blk * kCols;
                    const __half* dsu = reinterpret_cast<const __half*>(p.tab[7][e]) + blk * kCols;
                    for (int r = warp; r < nrows; r += kConsumerWarps) {
                        const int64_t pr = pair0 + r;
                        float gv[4], uv[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            float a = 0.f, b = 0.f;
                            for (int c2 = 0; c2 < p.nka; ++c2) {
                                a += __ldcg(&p.partA[((pr * 2 + 0) * p.nka + c2) * p.I + blk * kCols + lane * 4 + q]);
                                b += __ldcg(&p.partA[((pr * 2 + 1) * p.nka + c2) * p.I + blk * kCols + lane * 4 + q]);
                            }
                            gv[q] = a;
                            uv[q] = b;
                        }
                        out_transform(gv, gsv, lane);
                        out_transform(uv, usv, lane);
                        float dv[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            float gg = gv[q], uu = uv[q];
                            if (gg > p.limit) gg = p.limit;
                            if (uu < -p.limit) uu = -p.limit;
                            if (uu > p.limit) uu = p.limit;
                            const __half a = __float2half_rn((gg / (1.0f + __expf(-gg))) * uu);
                            dv[q] = __half2float(__hmul(a, dsu[lane * 4 + q]));
                        }
                        wht128_warp(dv, lane);
                        __half* dst = p.act + pr * p.I + blk * kCols + lane * 4;
#pragma unroll
                        for (int q = 0; q < 4; ++q) dst[q] = __float2half_rn(dv[q] * kHadNorm);
                    }
                    consumers_sync();
                    if (ctid == 0) {
                        __threadfence();   // release the down-input block
                        atomicAdd(&p.readyB[g * kStrideR + (blk * kCols) / p.kcb], 1u);
                    }
                }
            } else {
                // ---- phase B: partial, then maybe finish down block blk
                bool fin = true;
                if (p.nkb > 1) {
                    for (int idx = ctid; idx < nrows * kCols; idx += kConsumerThreads) {
                        const int r = idx / kCols, c = idx % kCols;
                        p.partB[((int64_t) (pair0 + r) * p.nkb + s) * p.H + blk * kCols + c] = S.cbuf[idx];
                    }
                    consumers_sync();
                    if (ctid == 0) {
                        __threadfence();
                        const uint32_t old = atomicAdd(&p.cntB[g * kStrideB + blk], 1u);
                        const int last = old == (uint32_t) (p.nkb - 1);
                        if (last) {
                            atomicExch(&p.cntB[g * kStrideB + blk], 0u);
                            __threadfence();
                        }
                        S.flag = last;
                    }
                    consumers_sync();
                    fin = S.flag != 0;
                    if (fin) {
                        for (int idx = ctid; idx < nrows * kCols; idx += kConsumerThreads) {
                            const int r = idx / kCols, c = idx % kCols;
                            float v = 0.f;
                            for (int c2 = 0; c2 < p.nkb; ++c2)
                                v += __ldcg(&p.partB[((int64_t) (pair0 + r) * p.nkb + c2) * p.H + blk * kCols + c]);
                            S.cbuf[idx] = v;
                        }
                        consumers_sync();
                    }
                }
                if (fin) {
                    const __half* dsv = reinterpret_cast<const __half*>(p.tab[8][e]) + blk * kCols;
                    for (int r = warp; r < nrows; r += kConsumerWarps) {
                        float v[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) v[q] = S.cbuf[r * kCols + lane * 4 + q];
                        out_transform(v, dsv, lane);
                        float4 o = make_float4(v[0], v[1], v[2], v[3]);
                        __stcg(reinterpret_cast<float4*>(p.downc + (int64_t) (pair0 + r) * p.H + blk * kCols + lane * 4), o);
                    }
                    consumers_sync();
                    if (ctid == 0) {
                        __threadfence();
                        const uint32_t old = atomicAdd(&p.cntG[blk], 1u);
                        const int last = old == (uint32_t) (G - 1);
                        if (last) {
                            atomicExch(&p.cntG[blk], 0u);
                            __threadfence();
                        }
                        S.flag = last;
                    }
                    consumers_sync();
                    if (S.flag) {
                        // fixed-order gather of column block blk for every row
                        for (int idx = ctid; idx < p.m * kCols; idx += kConsumerThreads) {
                            const int r = idx / kCols, c = idx % kCols;
                            float sum = 0.f;
                            for (int k = 0; k < p.topk; ++k) {
                                const int pr = P.slotpair[r * p.topk + k];
                                if (pr >= 0)
                                    sum += p.weights[r * p.topk + k] *
                                           __ldcg(&p.downc[(int64_t) pr * p.H + blk * kCols + c]);
                            }
                            store_out(p.out, p.out_dtype, (int64_t) r * p.H + blk * kCols + c, sum);
                        }
                    }
                }
            }
            consumers_sync();
        }
    }

    // Retire: the last CTA out restores the control region for the next launch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&p.ctrl[1], 1u);
        S.flag = old == gridDim.x - 1;
    }
    __syncthreads();
    if (S.flag) {
        __threadfence();
        for (int i = tid; i < G * kStrideR; i += kThreads) p.readyB[i] = 0u;
        if (tid == 0) {
            atomicExch(&p.ctrl[0], 0u);
            atomicExch(&p.ctrl[1], 0u);
        }
    }
}

// ------------------------------------------------------------------ host side
namespace {

struct MoeGeom {
    int kca, nka, kcb, nkb;
    int64_t pairs;
    int64_t off_partA, off_act, off_partB, off_downc, total;
};

MoeGeom moe_geom(int64_t m, int64_t topk, int64_t H, int64_t I) {
    MoeGeom g{};
    g.kca = H >= 1024 && H % 1024 == 0 ? 1024 : (H % 512 == 0 ? 512 : (H % 256 == 0 ? 256 : 128));
    g.nka = (int) (H / g.kca);
    g.kcb = I >= 1024 && I % 1024 == 0 ? 1024 : (I % 512 == 0 ? 512 : (I % 256 == 0 ? 256 : 128));
    if (g.kcb > I) g.kcb = (int) I;
    g.nkb = (int) (I / g.kcb);
    g.pairs = m * topk;
    int64_t off = EXL3_MOE_CTRL_BYTES;
    g.off_partA = off;
    off = align_up(off + g.pairs * 2 * g.nka * I * 4, 256);
    g.off_act = off;
    off = align_up(off + g.pairs * I * 2, 256);
    g.off_partB = off;
    off = align_up(off + (g.nkb > 1 ? g.pairs * g.nkb * H * 4 : 0), 256);
    g.off_downc = off;
    off = align_up(off + g.pairs * H * 4, 256);
    g.total = off;
    return g;
}

struct MoePrepared {
    bool ready = false;
    int sms = 0, resident = 0, grid = 0;
};

std::mutex g_moe_mu;
MoePrepared g_moe_prep[64][3][2];

template <int CB, bool PRECISE>
int moe_prepare_cb(int dev, MoePrepared* out) {
    std::lock_guard<std::mutex> lock(g_moe_mu);
    MoePrepared& pr = g_moe_prep[dev & 63][CB][PRECISE ? 1 : 0];
    if (!pr.ready) {
        DeviceInfo di;
        if (int rc = device_info(dev, &di)) return rc;
        const int smem = (int) sizeof(MoeSmem);
        auto kern = moe_kernel<CB, PRECISE>;
        EXL3_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        int res = 0;
        EXL3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, kern, kThreads, smem));
        EXL3_REQUIRE(res > 0, EXL3_ERR_UNSUPPORTED, "moe kernel has no resident CTA");
        pr.sms = di.sms;
        pr.resident = res;
        pr.grid = di.sms * res;
        pr.ready = true;
    }
    *out = pr;
    return EXL3_OK;
}

int moe_prepare_any(int cb, bool precise, MoePrepared* out) {
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    EXL3_REQUIRE(dev < 64, EXL3_ERR_UNSUPPORTED, "device index >= 64");
    if (precise) {
        switch (cb) {
            case 0: return moe_prepare_cb<0, true>(dev, out);
            case 1: return moe_prepare_cb<1, true>(dev, out);
            default: return moe_prepare_cb<2, true>(dev, out);
        }
    }
    switch (cb) {
        case 0: return moe_prepare_cb<0, false>(dev, out);
        case 1: return moe_prepare_cb<1, false>(dev, out);
        default: return moe_prepare_cb<2, false>(dev, out);
    }
}

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" int64_t exl3_moe_scratch_bytes(int64_t m, int64_t topk, int64_t hidden, int64_t inter) {
    if (m < 1 || topk < 1 || hidden < 128 || inter < 128) return -1;
    return moe_geom(m, topk, hidden, inter).total;
}

extern "C" int64_t exl3_moe_max_rows(void) { return kMoeMaxRows; }

extern "C" int exl3_moe_prepare(int kmax) {
    EXL3_REQUIRE(kmax >= 1 && kmax <= kMoeKmax, EXL3_ERR_UNSUPPORTED, "moe: K must be in 1..%d", kMoeKmax);
    MoePrepared pr;
    for (int cb = 0; cb < 3; ++cb)
        for (int precise = 0; precise < 2; ++precise)
            if (int rc = moe_prepare_any(cb, precise != 0, &pr)) return rc;
    return EXL3_OK;
}

extern "C" int exl3_moe_info(int kmax, int64_t* info) {
    EXL3_REQUIRE(info, EXL3_ERR_ARG, "exl3_moe_info: null output");
    if (int rc = exl3_moe_prepare(kmax)) return rc;
    MoePrepared pr;
    if (int rc = moe_prepare_any(1, false, &pr)) return rc;
    const int64_t v[14] = {pr.sms, pr.resident, kConsumerWarps + 1, pr.grid, kThreads, 3, MoeCfg::NS,
                           kMoeMaxRows, (int64_t) sizeof(MoeSmem), EXL3_MOE_CTRL_BYTES,
                           exl3_moe_scratch_bytes(kMoeMaxRows, 8, 4096, 2048), kMoeMaxRows, kMoeMaxSlots, 1};
    for (int i = 0; i < 14; ++i) info[i] = v[i];
    return EXL3_OK;
}

extern "C" int exl3_moe_decode(const void* x, int x_dtype, void* out, int out_dtype, int64_t m, int64_t hidden,
                               int64_t inter, const int64_t* gate_trellis, const int64_t* gate_suh,
                               const int64_t* gate_svh, const int64_t* up_trellis, const int64_t* up_suh,
                               const int64_t* up_svh, const int64_t* down_trellis, const int64_t* down_suh,
                               const int64_t* down_svh, int64_t n_experts, const int32_t* k_table, int K, int kmax,
                               int cb, const int32_t* ids, const float* weights, int64_t topk, float swiglu_limit,
                               void* scratch, int64_t scratch_bytes, int precise, void* stream) {
    EXL3_REQUIRE(x && out && ids && weights && scratch, EXL3_ERR_ARG, "moe: null pointer argument");
    const int64_t* tabs[9] = {gate_trellis, gate_suh, gate_svh, up_trellis, up_suh,
                              up_svh,       down_trellis, down_suh, down_svh};
    for (int i = 0; i < 9; ++i) EXL3_REQUIRE(tabs[i], EXL3_ERR_ARG, "moe: null pointer table %d", i);
    EXL3_REQUIRE(m >= 1 && m <= kMoeMaxRows, EXL3_ERR_ARG, "moe: row count out of range (1 <= m <= %d)", kMoeMaxRows);
    EXL3_REQUIRE(topk >= 1 && topk <= kMoeMaxTopk && m * topk <= kMoeMaxSlots, EXL3_ERR_ARG,
                 "moe: topk out of range (1 <= topk <= %d, m*topk <= %d)", kMoeMaxTopk, kMoeMaxSlots);
    EXL3_REQUIRE(n_experts >= 1 && n_experts <= kMoeMaxExperts, EXL3_ERR_ARG, "moe: pointer table has invalid expert count");
    EXL3_REQUIRE(hidden % 128 == 0 && hidden >= 128 && hidden <= kMoeMaxHidden, EXL3_ERR_ARG,
                 "moe: hidden must be a multiple of 128 in [128, %d]", kMoeMaxHidden);
    EXL3_REQUIRE(inter % 128 == 0 && inter >= 128 && inter <= kMoeMaxInter, EXL3_ERR_ARG,
                 "moe: intermediate must be a multiple of 128 in [128, %d]", kMoeMaxInter);
    EXL3_REQUIRE(x_dtype >= 0 && x_dtype <= 2 && out_dtype >= 0 && out_dtype <= 2, EXL3_ERR_ARG, "moe: bad dtype code");
    EXL3_REQUIRE(cb >= 0 && cb <= 2, EXL3_ERR_ARG, "moe: codebook must be 0, 1 or 2");
    if (!k_table) {
        EXL3_REQUIRE(K >= 1 && K <= kMoeKmax, EXL3_ERR_UNSUPPORTED, "moe: K must be in 1..%d (got %d)", kMoeKmax, K);
    } else {
        EXL3_REQUIRE(kmax >= 1 && kmax <= kMoeKmax, EXL3_ERR_UNSUPPORTED, "moe: kmax must be in 1..%d", kMoeKmax);
    }
    EXL3_REQUIRE(swiglu_limit > 0.0f && swiglu_limit < 3.0e38f, EXL3_ERR_ARG,
                 "moe: requires a finite positive SwiGLU limit");
    EXL3_REQUIRE(aligned16(scratch), EXL3_ERR_ARG, "moe: scratch must be 16-byte aligned");
    const MoeGeom g = moe_geom(m, topk, hidden, inter);
    EXL3_REQUIRE(scratch_bytes >= g.total, EXL3_ERR_ARG, "moe: scratch too small (%lld < %lld bytes)",
                 (long long) scratch_bytes, (long long) g.total);
    EXL3_REQUIRE(g.kca % (MoeCfg::SK * 16) == 0 && g.kcb % (MoeCfg::SK * 16) == 0, EXL3_ERR_UNSUPPORTED,
                 "moe: internal k-chunks (%d, %d) do not tile the ring stages", g.kca, g.kcb);
    MoePrepared pr;
    if (int rc = moe_prepare_any(cb, precise != 0, &pr)) return rc;

    MoeParams p{};
    p.x = x;
    p.out = out;
    for (int i = 0; i < 9; ++i) p.tab[i] = tabs[i];
    p.ktab = k_table;
    p.kuni = K;
    p.ids = ids;
    p.weights = weights;
    p.x_dtype = x_dtype;
    p.out_dtype = out_dtype;
    p.m = (int) m;
    p.H = (int) hidden;
    p.I = (int) inter;
    p.topk = (int) topk;
    p.E = (int) n_experts;
    p.limit = swiglu_limit;
    p.kca = g.kca;
    p.nka = g.nka;
    p.kcb = g.kcb;
    p.nkb = g.nkb;
    uint8_t* sb = static_cast<uint8_t*>(scratch);
    uint32_t* c32 = reinterpret_cast<uint32_t*>(sb);
    p.ctrl = c32;
    p.cntA = c32 + kCtrlWords;
    p.readyB = p.cntA + kMoeMaxSlots * kStrideA;
    p.cntB = p.readyB + kMoeMaxSlots * kStrideR;
    p.cntG = p.cntB + kMoeMaxSlots * kStrideB;
    p.partA = reinterpret_cast<float*>(sb + g.off_partA);
    p.act = reinterpret_cast<__half*>(sb + g.off_act);
    p.partB = reinterpret_cast<float*>(sb + g.off_partB);
    p.downc = reinterpret_cast<float*>(sb + g.off_downc);

    const int smem = (int) sizeof(MoeSmem);
    auto s = static_cast<cudaStream_t>(stream);
    if (precise) {
        switch (cb) {
            case 0: moe_kernel<0, true><<<pr.grid, kThreads, smem, s>>>(p); break;
            case 1: moe_kernel<1, true><<<pr.grid, kThreads, smem, s>>>(p); break;
            default: moe_kernel<2, true><<<pr.grid, kThreads, smem, s>>>(p); break;
        }
    } else {
        switch (cb) {
            case 0: moe_kernel<0, false><<<pr.grid, kThreads, smem, s>>>(p); break;
            case 1: moe_kernel<1, false><<<pr.grid, kThreads, smem, s>>>(p); break;
            default: moe_kernel<2, false><<<pr.grid, kThreads, smem, s>>>(p); break;
        }
    }
    EXL3_CUDA(cudaGetLastError());
    return EXL3_OK;
}

// ------------------------------------------------------------------ allocation-free variant
// exl3_moe_decode_noalloc: the same layer as exl3_moe_decode for callers that
// may not allocate device memory at all -- code running while a CUDA graph is
// being captured (an allocation there is either illegal or baked into the
// graph), hosts whose memory is owned by another allocator and who therefore
// cannot hand out a scratch buffer, and latency-critical callers that cannot
// afford cudaMalloc's implicit synchronization.  Its scratch is the array
// below, compiled into the library: EXL3_MOE_STATIC_SCRATCH_BYTES (4 MiB) of
// device memory that every GPU which loads the library holds until the
// process exits.  Geometries whose scratch (exl3_moe_scratch_bytes) exceeds it
// are rejected.
namespace exl3 {
namespace {

static __device__ __align__(256) uint8_t g_moe_static_scratch[EXL3_MOE_STATIC_SCRATCH_BYTES];

// Device address of g_moe_static_scratch, looked up once per device with that
// device current (in host code the array's name is only a host-side stand-in).
std::mutex g_static_mu;
void* g_static_ptr[64] = {};

int static_scratch_ptr(int dev, void** out) {
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_ptr[dev] == nullptr) {
        void* p = nullptr;
        EXL3_CUDA(cudaGetSymbolAddress(&p, g_moe_static_scratch));
        EXL3_REQUIRE(p != nullptr && aligned16(p), EXL3_ERR_CUDA, "moe noalloc: static scratch has no device address");
        g_static_ptr[dev] = p;
    }
    *out = g_static_ptr[dev];
    return EXL3_OK;
}

}  // namespace
}  // namespace exl3

extern "C" int exl3_moe_decode_noalloc(const void* x, int x_dtype, void* out, int out_dtype, int64_t m,
                                       int64_t hidden, int64_t inter, const int64_t* gate_trellis,
                                       const int64_t* gate_suh, const int64_t* gate_svh, const int64_t* up_trellis,
                                       const int64_t* up_suh, const int64_t* up_svh, const int64_t* down_trellis,
                                       const int64_t* down_suh, const int64_t* down_svh, int64_t n_experts,
                                       const int32_t* k_table, int K, int kmax, int cb, const int32_t* ids,
                                       const float* weights, int64_t topk, float swiglu_limit, int precise,
                                       void* stream) {
    EXL3_REQUIRE(m >= 1 && topk >= 1 && hidden >= 128 && inter >= 128, EXL3_ERR_ARG,
                 "moe noalloc: row count, topk, hidden and intermediate must be positive");
    const int64_t need = exl3_moe_scratch_bytes(m, topk, hidden, inter);
    EXL3_REQUIRE(need > 0 && need <= EXL3_MOE_STATIC_SCRATCH_BYTES, EXL3_ERR_ARG,
                 "moe noalloc: this geometry needs %lld scratch bytes, more than the static maximum of %d "
                 "(use exl3_moe_decode with a caller-provided scratch)",
                 (long long) need, (int) EXL3_MOE_STATIC_SCRATCH_BYTES);
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    EXL3_REQUIRE(dev >= 0 && dev < 64, EXL3_ERR_UNSUPPORTED, "moe noalloc: device index >= 64");
    void* scratch = nullptr;
    if (int rc = exl3::static_scratch_ptr(dev, &scratch)) return rc;
    // The array keeps the previous call's contents; the control region (ticket
    // and retire counters, status word, completion counters) must be zero.
    auto s = static_cast<cudaStream_t>(stream);
    EXL3_CUDA(cudaMemsetAsync(scratch, 0, EXL3_MOE_CTRL_BYTES, s));
    return exl3_moe_decode(x, x_dtype, out, out_dtype, m, hidden, inter, gate_trellis, gate_suh, gate_svh,
                           up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh, n_experts, k_table, K,
                           kmax, cb, ids, weights, topk, swiglu_limit, scratch, EXL3_MOE_STATIC_SCRATCH_BYTES,
                           precise, stream);
}
