// moe.cu -- routed-expert MoE decode layer for sm_100a, one launch per layer.
//
// Replaces the lna2 ticket kernel (recipe-lna/lna2/lna_moe_ticket.cu:240-429)
// with the same numerics contract (lna_moe_ticket.cu:5-12):
//   x -> fp16; gate/up accumulate fp32; output Hadamard + svh fp32;
//   silu(min(g, L)) * clamp(u, -L, L) fp32 -> fp16; down-input suh + Hadamard
//   -> fp16; down accumulate fp32; output Hadamard + svh fp32; weighted sum
//   over top-k slots in slot order, fp32; one cast to the output dtype.
//
// Structure (B200 design, not the reference's).  Every CTA builds the same
// route plan in shared memory (groups = experts in ascending id, pairs =
// unique (expert, row), a group's pairs contiguous).  Then:
//   P  (consumer warps, at start; items claimed per warp from a counter):
//      (group, gate|up, 128-block of hidden): x -> fp16, * suh, Hadamard ->
//      fp16, written to scratch already in MMA B-fragment order;
//   A  units (group, 128-col block of I, gate|up, k-chunk of hidden);
//   B  units (group, 128-col block of hidden, k-chunk of I);
// A and B units come from one global ticket counter, all A before all B.
// CTA roles: warp 8 (producer) claims a unit, publishes its descriptor, points
// a tensor map at the expert's matrix, waits (bounded) until the unit's input
// fragments are ready and streams every stage -- SK k-slices of the unit's 8
// weight tiles (one 3-D TMA box) plus the matching B fragments (one bulk copy)
// -- into a shared-memory ring.  Warps 0-7 (consumers) decode n-tile w of
// each k-slice in registers and run the MMAs, then drop their fp32 partial
// into a shared-memory tile.  Warp 9 (epilogue) stores the tile, bumps the
// block's completion counter and, when it completes a block, runs the block
// epilogue (A: sum the partials, out-Hadamard * svh for gate and up, SwiGLU,
// down suh + Hadamard -> down-input fragments; B: sum, out-H * svh; the last
// group to finish a hidden block gathers it in slot order).  The consumers
// never meet a CTA-wide barrier or a global fence.
// Waits only point backwards (A on P, B on A), every P item and every unit
// is claimed by a running warp or CTA and P / A work never waits on later
// work, so progress needs no co-residency and no grid barrier.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "host.hpp"
#include "stage.cuh"
#include "tcgen05.cuh"

namespace exl3 {

constexpr int kMoeMaxRows = 32;      // row bitmask is one 32-bit word
constexpr int kMoeMaxSlots = 256;    // m * topk
constexpr int kMoeMaxExperts = 1024;
constexpr int kMoeMaxTopk = 16;
constexpr int kMoeKmax = 4;          // weight part of a ring stage sized for K <= 4
constexpr int kMoeMaxHidden = 8192;
constexpr int kMoeMaxInter = 4096;
constexpr int kMoeSK = kStageSK;                          // k-slices per ring stage
constexpr int kMoeWBytes = kMoeSK * 8 * 32 * kMoeKmax;    // largest weight part of a stage (8 KB)
constexpr int kMoeMaxStages = 12;                         // ring depth cap
constexpr int kMoeRingBytes = 98304;                      // ring + partial tiles per CTA
constexpr int kMoeDQ = 4;                                 // descriptor queue depth
constexpr int kMoeMaxNka = 8;                             // hidden k-chunks
constexpr int kMoeMaxNkb = 4;                             // intermediate k-chunks
constexpr int kNBImax = kMoeMaxInter / 128;
constexpr int kNBHmax = kMoeMaxHidden / 128;
// CTA roles: warps 0-7 consume (decode + MMA), warp 8 produces (tickets,
// stage copies), warp 9 stores partials and runs the block epilogues.
// Ring stages still queued when the producer claims its next unit: at most
// this, and at most the shorter unit kind's stage count (TP8 shard: 2-stage
// down units, where claiming later leaves the last units to idle CTAs:
// 42.4 -> 41.5 us; config 2's 16-stage units want the deeper run-ahead).
constexpr int kMoeClaimAhead = 4;
constexpr int kMoeConsumerWarps = 8;
constexpr int kMoeProducerWarp = 8;
constexpr int kMoeEpilogueWarp = 9;
constexpr int kMoeThreads = 320;
static_assert(kMoeMaxSlots <= kMoeThreads, "the route plan gives every slot its own thread");
// Control region (uint32 words).  ctrl[0] unit ticket, [1] retired CTAs,
// [2] status word, [3] unused.  Then the per-group counters.
constexpr int kCtrlWords = 16;
constexpr int kOffCntA = kCtrlWords;                                  // [group][I block]
constexpr int kOffReadyP = kOffCntA + kMoeMaxSlots * kNBImax;          // [group][2][hidden chunk]
constexpr int kOffReadyB = kOffReadyP + kMoeMaxSlots * 2 * kMoeMaxNka; // [group][I chunk]
constexpr int kOffCntB = kOffReadyB + kMoeMaxSlots * kMoeMaxNkb;       // [group][hidden block]
constexpr int kOffCntG = kOffCntB + kMoeMaxSlots * kNBHmax;            // [hidden block]
constexpr int kCtrlEnd = kOffCntG + kNBHmax;
static_assert(4 * kCtrlEnd <= EXL3_MOE_CTRL_BYTES, "control region too small");

// ------------------------------------------------------------------ phase clock
// Compile-gated phase timers (-DEXL3_PHASE_CLOCK; the B200 counterpart of the
// reference's LNA2_PHASE_CLOCK, recipe-lna/lna2/lna_moe_ticket.cu:62-64,280-290).
// Each warp accumulates clock64 cycles per phase in registers and lane 0 adds
// them into g_phase when the warp retires; exl3_phase_clock_read copies them
// out.  Release builds compile all of it away.
#ifdef EXL3_PHASE_CLOCK
enum {
    PH_P = 0,          // consumer: input-transform items
    PH_DESC,           // consumer: waiting for a unit descriptor
    PH_DATA,           // consumer: waiting for stage data (inside the unit loop)
    PH_UNIT,           // consumer: unit loop incl. data waits
    PH_PARTIAL,        // consumer: partial tile write
    PH_FIN_A,          // epilogue: phase-A block epilogue
    PH_FIN_B,          // epilogue: phase-B block epilogue + gather
    PH_PROD_DESC,      // producer: ticket + descriptor publish
    PH_PROD_DEP,       // producer: waiting for input fragments
    PH_PROD_SLOT,      // producer: waiting for ring slots
    PH_PROD_ISSUE,     // producer: issuing copies
    PH_EPI_DESC,       // epilogue: waiting for a descriptor
    PH_EPI_WAIT,       // epilogue: waiting for a partial tile
    PH_EPI_STORE,      // epilogue: partial store + completion counter
    PH_UNITS,          // count of units consumed (per warp)
    PH_FINS_A,         // count of phase-A epilogues
    PH_FINS_B,         // count of phase-B epilogues
    PH_TOTAL,          // cycles from kernel start to warp exit
    PH_PROD_TMAP,      // producer: pointing the unit's tensor map at its matrix
    PH_N
};
static __device__ unsigned long long g_phase[PH_N];
#define PHASE_DECL unsigned long long ph_[PH_N] = {}; unsigned long long ph_t_ = clock64(); const unsigned long long ph_start_ = ph_t_;
#define PHASE_MARK(c) do { const unsigned long long n_ = clock64(); ph_[c] += n_ - ph_t_; ph_t_ = n_; } while (0)
#define PHASE_COUNT(c) (ph_[c] += 1)
#define PHASE_FLUSH(lane) do { ph_[PH_TOTAL] = clock64() - ph_start_; if ((lane) == 0) for (int i_ = 0; i_ < PH_N; ++i_) atomicAdd(&g_phase[i_], ph_[i_]); } while (0)
#define PH_ARG , ph_[PH_DATA]
#else
#define PHASE_DECL
#define PHASE_MARK(c)
#define PHASE_COUNT(c)
#define PHASE_FLUSH(lane)
#define PH_ARG
#endif

// Per-CTA timeline (%globaltimer ns; -DEXL3_TIMELINE, or with the phase
// clocks): entry, plan built, consumer warp 0 done with its input items,
// consumer warp 0 / producer / epilogue leave their loops, retire barrier
// passed, exit.  Eight stores per CTA, so the timing it shows is the plain
// build's.  Read with exl3_timeline_read.
#if defined(EXL3_PHASE_CLOCK) && !defined(EXL3_TIMELINE)
#define EXL3_TIMELINE
#endif
#ifdef EXL3_TIMELINE
static __device__ unsigned long long g_tl[320][8];
#define TL_MARK(i) do { if ((threadIdx.x & 31) == 0) g_tl[blockIdx.x][i] = globaltimer_ns(); } while (0)
// Per-unit marks, by ticket t: [0] descriptor published, [1] tensor map
// ready, [2] input dependency met, [3] last stage issued, [4] consumer warp 0
// starts the unit, [5] it ends the unit, [6] epilogue done with the unit,
// [7] the CTA.  Read with exl3_unit_trace_read.
constexpr int kUtMax = 8192;
static __device__ unsigned long long g_ut[kUtMax][8];
#define UT_MARK(t, i) do { if ((threadIdx.x & 31) == 0 && (t) >= 0 && (t) < kUtMax) g_ut[t][i] = globaltimer_ns(); } while (0)
#define UT_CTA(t) do { if ((threadIdx.x & 31) == 0 && (t) >= 0 && (t) < kUtMax) g_ut[t][7] = blockIdx.x; } while (0)
#else
#define TL_MARK(i)
#define UT_MARK(t, i)
#define UT_CTA(t)
#endif

// Tensor maps: one 3-D map per (projection kind, K) describes an expert
// matrix as [k/16 slices][n/16 tiles][16K u16 words]; a box is one ring
// stage (SK slices x 8 tiles).  The host encodes them once per (hidden,
// intermediate) with a placeholder address; each unit's producer copies the
// template to shared memory, replaces the address with its expert's matrix
// and publishes it to a per-CTA global slot.  A slot is rewritten only after
// every copy issued through it has landed: slots are used round robin and
// kMoeTmapSlots exceeds the ring depth (<= 12 stages, >= 1 stage per unit).
constexpr int kMoeTmapSlots = 13;
constexpr int kMoeMaxGrid = 320;   // 2 CTAs per SM on up to 160 SMs

struct MoeParams {
    CUtensorMap tmpl[8];        // [kind (0 gate/up, 1 down)][K - 1]
    CUtensorMap* tmaps;         // [grid][kMoeTmapSlots] per-CTA working maps
    const void* x;
    void* out;
    const int64_t* tab[9];      // gate t/su/sv, up t/su/sv, down t/su/sv
    const int32_t* ktab;        // per-expert K, or null (then kuni)
    RouteIn route;              // expert ids / routing weights (dtype, optional expert map)
    int x_dtype, out_dtype;
    int m, H, I, topk, E, kuni;
    float limit;
    int kca, nka;               // gate/up k-chunk over H
    int kcb, nkb;               // down k-chunk over I
    int claim_ahead;            // see kMoeClaimAhead
    RingGeom ring;              // ns stages of slot_bytes (weights: wpart bytes, then B fragments)
    uint32_t* ctrl;
    float* partA;               // [pairs][2][nka][I]
    uint32_t* xg;               // input fragments: per pair 2 * (H/16) row-slices of 16*FW bytes
    uint32_t* ag;               // down-input fragments: per pair (I/16) row-slices
    float* partB;               // [pairs][nkb][H] (== downc when nkb == 1)
    float* downc;               // [pairs][H]
    // Fused tensor-parallel sum (exl3_moe_decode_tp; tp_world == 0: none).
    // Every rank holds an exchange buffer (tp_buffer_* below); the CTA that
    // gathers a hidden block pushes its partial rows into slot [rank] of
    // every rank's buffer, raises its flag there, waits for all ranks' flags
    // in its own buffer and writes the rank-ordered fp32 sum.
    const int64_t* tp_bufs;     // [world] device addresses of the ranks' exchange buffers
    int tp_rank, tp_world, tp_mcap;
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

// Route plan, identical in every CTA (recipe-lna/lna2/lna_moe_ticket.cu:167-214
// restated): per-expert row mask, exclusive scans over experts -> group id and
// first pair, slot -> pair via popcount.  Uses the 256 consumer threads.
__device__ void build_plan(MoePlan& P, const MoeParams& p, int tid) {
    const bool worker = tid < kConsumerThreads;      // 256 threads own 4 experts each
    const int nthr = (int) blockDim.x;
    // thread s owns slot s (m * topk <= kMoeMaxSlots <= the block): its id is
    // loaded once, ahead of the mask clearing, and reused for slot -> pair
    const int nslots = p.m * p.topk;
    const int my_id = tid < nslots ? route_local_id(p.route, tid, p.E) : -1;
    for (int e = tid; e < p.E; e += nthr) P.emask[e] = 0u;
    __syncthreads();
    if (my_id >= 0) atomicOr(&P.emask[my_id], 1u << (tid / p.topk));
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
    if (tid < nslots) {
        short sp = -1;
        if (my_id >= 0) {
            const int row = tid / p.topk;
            sp = (short) (P.epair[my_id] + __popc(P.emask[my_id] & ((1u << row) - 1u)));
        }
        P.slotpair[tid] = sp;
    }
    __syncthreads();
}

struct alignas(128) MoeHead {
    MoePlan plan;
    uint64_t full[kMoeMaxStages];
    uint64_t empty[kMoeMaxStages];
    uint64_t dqf[kMoeDQ];
    uint64_t dqe[kMoeDQ];
    uint64_t pfull[2];          // partial tile written by the consumer warps
    uint64_t pempty[2];         // partial tile stored by the epilogue warp
    int desc[kMoeDQ][8];        // kind, group, mat, block, chunk, K, ticket
    int last_cta;
    int retire_rank;            // order in which this CTA retired
    uint32_t tp_epoch;          // this launch's exchange epoch (fused TP sum)
    alignas(128) CUtensorMap tmap;   // the producer's tensor map under construction
};
constexpr int kMoeHeadBytes = (int) ((sizeof(MoeHead) + 127) / 128 * 128);

// Phase P: one warp transforms hidden block kb of every row of group g for
// projection mat (0 gate, 1 up): fp16(x) * suh in fp16, 128-point Hadamard in
// fp32, * 1/sqrt(128) -> fp16 (recipe-lna/lna2/lna_moe_ticket.cu:119-144),
// written as B fragments.
// The suh values are loaded once and the activations of four rows at a time
// are in flight together, so the item costs about one load latency per four
// rows rather than one per row (it is on the path to the layer's first units).
template <bool PRECISE>
__device__ void moe_input_item(const MoeParams& p, const MoePlan& P, int g, int mat, int kb, int lane) {
    constexpr int FW = Frag<PRECISE>::FW;
    constexpr int kRowBatch = 4;
    const int e = P.gexp[g];
    uint32_t gm = P.gmask[g];
    const int nrows = __popc(gm), pair0 = P.gpair[g];
    const int HS = p.H / 16;
    const __half* suh = reinterpret_cast<const __half*>(p.tab[mat ? 4 : 1][e]);
    uint32_t* gbase = p.xg + (size_t) pair0 * 2 * HS * 4 * FW;
    const int k0 = kb * 128 + lane * 4;
    __half su[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) su[q] = suh[k0 + q];
    for (int r0 = 0; r0 < nrows; r0 += kRowBatch) {
        __half xa[kRowBatch][4];
#pragma unroll
        for (int j = 0; j < kRowBatch; ++j) {
            if (r0 + j < nrows) {
                const int row = __ffs((int) gm) - 1;
                gm &= gm - 1u;
#pragma unroll
                for (int q = 0; q < 4; ++q) xa[j][q] = load_act_half(p.x, p.x_dtype, (int64_t) row * p.H + k0 + q);
            }
        }
#pragma unroll
        for (int j = 0; j < kRowBatch; ++j) {
            if (r0 + j >= nrows) break;   // warp-uniform
            const int ri = r0 + j;
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = __half2float(__hmul(xa[j][q], su[q]));
            wht128_warp(v, lane);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int kl = lane * 4 + q;
                const int ks = kb * 8 + (kl >> 4);
                uint32_t* rs = gbase + ((size_t) (mat * HS + ks) * nrows + ri) * 4 * FW;
                store_frag<PRECISE>(rs, kl & 15, __float2half_rn(v[q] * kHadNorm));
            }
        }
    }
}

// Phase-A epilogue of (group g, I block blk), by one warp: sum the gate and up
// partials in fixed order, output transform, SwiGLU (clamp, then SiLU), down
// suh + Hadamard -> fp16 down-input fragments (lna_moe_ticket.cu:329-359).
template <bool PRECISE>
__device__ void moe_finish_a(const MoeParams& p, const MoePlan& P, int g, int blk, int lane) {
    constexpr int FW = Frag<PRECISE>::FW;
    const int e = P.gexp[g];
    const int nrows = __popc(P.gmask[g]), pair0 = P.gpair[g];
    const int IS = p.I / 16;
    const __half* gsv = reinterpret_cast<const __half*>(p.tab[2][e]) + blk * kCols;
    const __half* usv = reinterpret_cast<const __half*>(p.tab[5][e]) + blk * kCols;
    const __half* dsu = reinterpret_cast<const __half*>(p.tab[7][e]) + blk * kCols;
    uint32_t* abase = p.ag + (size_t) pair0 * IS * 4 * FW;
    // the block's svh (gate, up) and down suh, loaded once for all rows
    float gs[4], us[4];
    __half ds[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        gs[q] = __half2float(gsv[lane * 4 + q]);
        us[q] = __half2float(usv[lane * 4 + q]);
        ds[q] = dsu[lane * 4 + q];
    }
    for (int ri = 0; ri < nrows; ++ri) {
        const int64_t pr = pair0 + ri;
        float gv[4] = {0.f, 0.f, 0.f, 0.f}, uv[4] = {0.f, 0.f, 0.f, 0.f};
        // four chunks of gate and of up at a time (eight loads in flight:
        // one round for up to 4 chunks), summed in chunk order
        for (int c0 = 0; c0 < p.nka; c0 += 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + j < p.nka) {
                    a[j] = __ldcg(reinterpret_cast<const float4*>(
                        p.partA + ((pr * 2 + 0) * p.nka + c0 + j) * p.I + blk * kCols + lane * 4));
                    b[j] = __ldcg(reinterpret_cast<const float4*>(
                        p.partA + ((pr * 2 + 1) * p.nka + c0 + j) * p.I + blk * kCols + lane * 4));
                }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + j < p.nka) {
                    gv[0] += a[j].x; gv[1] += a[j].y; gv[2] += a[j].z; gv[3] += a[j].w;
                    uv[0] += b[j].x; uv[1] += b[j].y; uv[2] += b[j].z; uv[3] += b[j].w;
                }
        }
        // output transform: H128, / sqrt(128), * svh (same float order as out_transform)
        wht128_warp(gv, lane);
        wht128_warp(uv, lane);
        float dv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float gg = gv[q] * kHadNorm * gs[q], uu = uv[q] * kHadNorm * us[q];
            if (gg > p.limit) gg = p.limit;
            if (uu < -p.limit) uu = -p.limit;
            if (uu > p.limit) uu = p.limit;
            const __half a = __float2half_rn((gg / (1.0f + __expf(-gg))) * uu);
            dv[q] = __half2float(__hmul(a, ds[q]));
        }
        wht128_warp(dv, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int kl = lane * 4 + q;
            const int ks = blk * 8 + (kl >> 4);
            uint32_t* rs = abase + ((size_t) ks * nrows + ri) * 4 * FW;
            store_frag<PRECISE>(rs, kl & 15, __float2half_rn(dv[q] * kHadNorm));
        }
    }
}

// ------------------------------------------------------------------ fused TP sum
// Exchange buffer of one rank: [0, 256) header (word 0: epoch counter), then
// partial rows [2 parities][world][mcap][H] of 8-byte words, each one fp32
// value in the low half and the epoch that wrote it in the high half, stored
// and loaded as single 8-byte accesses: a reader that sees the epoch sees the
// value, so no flags and no fences are needed (the low-latency format NCCL
// uses for small messages).  Parity = epoch & 1: a rank reaches epoch e + 2
// only after every rank has pushed e + 1, which each does only after its own
// epoch-e launch has finished reading, so one parity is never written while
// it is read.
constexpr int kTpHeader = 256;
__host__ __device__ inline int64_t tp_buffer_bytes_for(int world, int64_t mcap, int64_t H) {
    return kTpHeader + (int64_t) 2 * world * mcap * H * 8;
}

__device__ __forceinline__ void st_relaxed_sys_v2(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" :: "l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Row r of this rank's partial of hidden block blk (4 values per lane) into
// slot [rank] of every rank's exchange buffer.
__device__ __forceinline__ void tp_push_row(const MoeParams& p, uint32_t epoch, int blk, int lane, int r,
                                            const float (&v)[4]) {
    const int W = p.tp_world, par = (int) (epoch & 1u);
    const uint64_t tag = (uint64_t) epoch << 32;
    const uint64_t w0 = tag | __float_as_uint(v[0]), w1 = tag | __float_as_uint(v[1]);
    const uint64_t w2 = tag | __float_as_uint(v[2]), w3 = tag | __float_as_uint(v[3]);
    for (int j = 0; j < W; ++j) {
        uint64_t* dst = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(p.tp_bufs[j]) + kTpHeader) +
                        (((int64_t) par * W + p.tp_rank) * p.tp_mcap + r) * p.H + blk * kCols + lane * 4;
        st_relaxed_sys_v2(dst, w0, w1);
        st_relaxed_sys_v2(dst + 2, w2, w3);
    }
}

__device__ __forceinline__ void ld_relaxed_sys_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p));
}

// Wait (bounded) until word *e carries `epoch`; returns it.
__device__ __noinline__ uint64_t tp_wait_word(const uint64_t* e, uint32_t epoch, bool& ok) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kSpinCap; ++i) {
        __nanosleep(32);
        const uint64_t v = ld_relaxed_sys(e);
        if ((uint32_t) (v >> 32) == epoch) return v;
        if ((i & 63u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    ok = false;
    return 0;
}

// Row r of block blk of the output, by one warp (4 values per lane): the sum
// over ranks, in rank order, of their partials in this rank's buffer.  Two
// ranks' words are loaded before any is tested, so their latencies overlap;
// a word that does not carry this launch's epoch yet is waited for (bounded).
__device__ void tp_finish_row(const MoeParams& p, uint32_t epoch, int blk, int r, int lane, bool& ok) {
    const int W = p.tp_world, par = (int) (epoch & 1u);
    const uint64_t* src = reinterpret_cast<const uint64_t*>(reinterpret_cast<const uint8_t*>(p.tp_bufs[p.tp_rank]) +
                                                            kTpHeader) +
                          ((int64_t) par * W * p.tp_mcap + r) * p.H + blk * kCols + lane * 4;
    const int64_t rs = (int64_t) p.tp_mcap * p.H;   // words between ranks' slots
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < W; j += 2) {
        uint64_t v[2][4];
        const int nj = j + 1 < W ? 2 : 1;
        for (int jj = 0; jj < nj; ++jj) {
            ld_relaxed_sys_v2(src + (j + jj) * rs, v[jj][0], v[jj][1]);
            ld_relaxed_sys_v2(src + (j + jj) * rs + 2, v[jj][2], v[jj][3]);
        }
        for (int jj = 0; jj < nj; ++jj)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint64_t w = v[jj][q];
                if ((uint32_t) (w >> 32) != epoch) w = ok ? tp_wait_word(src + (j + jj) * rs + q, epoch, ok) : 0;
                s[q] += __uint_as_float((uint32_t) w);
            }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) store_out(p.out, p.out_dtype, (int64_t) r * p.H + blk * kCols + lane * 4 + q, s[q]);
}

// Phase-B block epilogue, part 1 (lna_moe_ticket.cu:368-378): the block's
// down output of every row of group g -- the k-chunk partials summed in chunk
// order (or, with a single chunk, the unit's tile straight from shared
// memory), out-H128 * svh -- into downc.  `sv` holds this lane's four svh
// values when the caller loaded them ahead (else null).
__device__ void moe_finish_b_rows(const MoeParams& p, const MoePlan& P, int g, int blk, int lane,
                                  const float* tile, const uint2* sv) {
    const int e = P.gexp[g];
    const int nrows = __popc(P.gmask[g]), pair0 = P.gpair[g];
    uint2 s4;
    if (sv != nullptr) s4 = *sv;
    else s4 = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.tab[8][e]) + blk * kCols + lane * 4));
    const __half2 s01 = *reinterpret_cast<const __half2*>(&s4.x), s23 = *reinterpret_cast<const __half2*>(&s4.y);
    const float sc[4] = {__low2float(s01), __high2float(s01), __low2float(s23), __high2float(s23)};
    for (int ri = 0; ri < nrows; ++ri) {
        const int64_t pr = pair0 + ri;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (tile != nullptr) {
            const float4 a = *reinterpret_cast<const float4*>(tile + ri * kCols + lane * 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        } else {
            for (int c2 = 0; c2 < p.nkb; ++c2) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(
                    p.partB + (pr * p.nkb + c2) * p.H + blk * kCols + lane * 4));
                v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
            }
        }
        wht128_warp(v, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = v[q] * kHadNorm * sc[q];
        __stcg(reinterpret_cast<float4*>(p.downc + pr * p.H + blk * kCols + lane * 4),
               make_float4(v[0], v[1], v[2], v[3]));
    }
}

// Row r of hidden block blk of the layer output, by one warp (4 values per
// lane), once every group has finished the block: the top-k slots summed in
// slot order in fp32 (recipe-lna/lna2/lna_moe_ticket.cu:409-428); with the
// fused TP sum the rank's partial row goes to the exchange instead.  The
// slots' rows are loaded eight at a time before any is summed, so their L2
// latencies overlap.
__device__ void moe_gather_row(const MoeParams& p, const MoePlan& P, int blk, int r, int lane, uint32_t epoch) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < p.topk; k0 += 8) {
        float4 d[8];
        float wv[8];
        bool ok[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = k0 + j;
            const int pr = k < p.topk ? (int) P.slotpair[r * p.topk + k] : -1;
            ok[j] = pr >= 0;
            wv[j] = ok[j] ? route_weight(p.route, r * p.topk + k) : 0.f;
            d[j] = __ldcg(reinterpret_cast<const float4*>(p.downc + (int64_t) (ok[j] ? pr : 0) * p.H +
                                                           blk * kCols + lane * 4));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (ok[j]) {
                s[0] += wv[j] * d[j].x; s[1] += wv[j] * d[j].y; s[2] += wv[j] * d[j].z; s[3] += wv[j] * d[j].w;
            }
        }
    }
    if (p.tp_world > 0) {
        tp_push_row(p, epoch, blk, lane, r, s);
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
            store_out(p.out, p.out_dtype, (int64_t) r * p.H + blk * kCols + lane * 4 + q, s[q]);
    }
}

// Phase-B block epilogue, part 2: count the group's block as done (release:
// the warp's downc stores first).  The gather waits for the count at retire.
__device__ __forceinline__ void moe_finish_b_count(int blk, int lane, uint32_t* cntG) {
    __syncwarp();
    if (lane == 0) red_add_release_gpu(&cntG[blk], 1u);
}

template <int CB, bool PRECISE>
__global__ void __launch_bounds__(kMoeThreads, 2) moe_kernel(const __grid_constant__ MoeParams p) {
    constexpr int FW = Frag<PRECISE>::FW;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    MoeHead& S = *reinterpret_cast<MoeHead*>(smem_raw);
    uint8_t* ring = smem_raw + kMoeHeadBytes;
    float* ptile = reinterpret_cast<float*>(ring + (size_t) p.ring.ns * p.ring.slot_bytes);   // [2][m][128]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* status = p.ctrl + 2;
    uint32_t* cntA = p.ctrl + kOffCntA;
    uint32_t* readyP = p.ctrl + kOffReadyP;
    uint32_t* readyB = p.ctrl + kOffReadyB;
    uint32_t* cntB = p.ctrl + kOffCntB;
    uint32_t* cntG = p.ctrl + kOffCntG;

    if (tid == 0) TL_MARK(0);
    // Programmatic dependent launch: the next layer's launch may take SMs as
    // this grid's CTAs retire.  Up to griddepcontrol.wait this CTA touches only
    // shared memory and its own inputs (ids), never the scratch, the exchange
    // buffers or the output that the previous launch in the stream may still use.
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < p.ring.ns; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], kMoeConsumerWarps); }
        for (int s = 0; s < kMoeDQ; ++s) { mbar_init(&S.dqf[s], 1); mbar_init(&S.dqe[s], kMoeConsumerWarps + 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&S.pfull[s], kMoeConsumerWarps); mbar_init(&S.pempty[s], 1); }
        fence_barrier_init();
    }
    build_plan(S.plan, p, tid);     // ends with __syncthreads (also publishes the barrier init)
    pdl_wait();
    if (tid == 0)
        S.tp_epoch = p.tp_world > 0 ? __ldcg(reinterpret_cast<const uint32_t*>(p.tp_bufs[p.tp_rank])) + 1u : 0u;
    __syncthreads();
    if (tid == 0) TL_MARK(1);
    const MoePlan& P = S.plan;
    const int G = P.G;
    const int NBI = p.I / kCols, NBH = p.H / kCols;
    const int UA = G * NBI * 2 * p.nka;
    const int total = UA + G * NBH * p.nkb;

    if (G == 0 && blockIdx.x == 0) {
        // No valid route: the layer output is zero.
        for (int i = tid; i < p.m * p.H; i += kMoeThreads) store_out(p.out, p.out_dtype, i, 0.f);
    }

    if (warp == kMoeProducerWarp) {
        // ------------------------------------------------------------ producer
        PHASE_DECL
        int ticket = claim_ticket(&p.ctrl[0], lane);
        uint32_t it = 0, du = 0, units = 0;
        bool ok = true;
        while (ok) {
            int d[6] = {-1, 0, 0, 0, 0, 0};
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
                int K = p.ktab ? p.ktab[P.gexp[g]] : p.kuni;
                if (K < 1 || 256 * K * kMoeSK > p.ring.wpart) K = 0;   // above the launch's kmax: stage too small
                d[0] = kind; d[1] = g; d[2] = mat; d[3] = blk; d[4] = s; d[5] = K;
            }
            if (lane == 0) {
                const int slot = du % kMoeDQ;
                ok = mbar_wait(&S.dqe[slot], ((du / kMoeDQ) + 1u) & 1u, status);
                if (ok) {
#pragma unroll
                    for (int q = 0; q < 6; ++q) S.desc[slot][q] = d[q];
#ifdef EXL3_TIMELINE
                    S.desc[slot][6] = ticket;
#endif
                    mbar_arrive(&S.dqf[slot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            ++du;
            UT_MARK(ticket, 0);
            UT_CTA(ticket);
            PHASE_MARK(PH_PROD_DESC);
            if (d[0] < 0 || !ok) break;
            if (d[5] == 0) {
                if (lane == 0) set_error(status, ERR_BAD_K);
                ticket = claim_ticket(&p.ctrl[0], lane);
                continue;
            }
            const int kind = d[0], g = d[1], mat = d[2], blk = d[3], s = d[4], K = d[5];
            const int e = P.gexp[g];
            const int nrows = __popc(P.gmask[g]), pair0 = P.gpair[g];
            const int tb = 32 * K;                  // bytes per tile
            const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.tab[kind == 0 ? (mat ? 3 : 0) : 6][e]);
            const uint8_t* bsrc;
            int ks0, nst;
            const int64_t rsb = (int64_t) nrows * 16 * FW;   // B-fragment bytes per k-slice
            if (kind == 0) {
                ks0 = s * (p.kca / 16);
                bsrc = reinterpret_cast<const uint8_t*>(p.xg) + (int64_t) pair0 * 2 * p.H * FW +
                       ((int64_t) mat * (p.H / 16) + ks0) * rsb;
                nst = p.kca / (16 * kMoeSK);
            } else {
                ks0 = s * (p.kcb / 16);
                bsrc = reinterpret_cast<const uint8_t*>(p.ag) + (int64_t) pair0 * p.I * FW + (int64_t) ks0 * rsb;
                nst = p.kcb / (16 * kMoeSK);
            }
            const bool valid = aligned16_dev(wbase);
            if (!valid && lane == 0) set_error(status, ERR_MISALIGNED);
            // Point this unit's tensor map at the expert's matrix.
            CUtensorMap* gtm = p.tmaps + (size_t) blockIdx.x * kMoeTmapSlots + (int) (units % kMoeTmapSlots);
            ++units;
            if (valid) {
                const uint4* tsrc = reinterpret_cast<const uint4*>(&p.tmpl[kind * 4 + K - 1]);
                if (lane < 8) reinterpret_cast<uint4*>(&S.tmap)[lane] = tsrc[lane];
                __syncwarp();
                if (lane == 0) tmap_replace_address(&S.tmap, wbase);
                __syncwarp();
                tmap_publish(gtm, &S.tmap);
                if (lane == 0) tmap_acquire(gtm);
            }
            PHASE_MARK(PH_PROD_TMAP);
            UT_MARK(ticket, 1);
            // The unit's input fragments must be complete before they are copied.
            if (lane == 0) {
                if (kind == 0) wait_counter(&readyP[(g * 2 + mat) * kMoeMaxNka + s], (uint32_t) (p.kca / kCols), status);
                else wait_counter(&readyB[g * kMoeMaxNkb + s], (uint32_t) (p.kcb / kCols), status);
                fence_proxy_async_global();
            }
            __syncwarp();
            UT_MARK(ticket, 2);
            PHASE_MARK(PH_PROD_DEP);
            const uint32_t wbytes = (uint32_t) (kMoeSK * 8 * tb);
            const int bbytes = (int) (kMoeSK * rsb);
            for (int st = 0; st < nst && ok; ++st) {
                const int slot = (int) (it % (uint32_t) p.ring.ns);
                if (lane == 0) {
                    ok = mbar_wait(&S.empty[slot], ((it / (uint32_t) p.ring.ns) + 1u) & 1u, status);
                    PHASE_MARK(PH_PROD_SLOT);
                    if (ok) {
                        uint8_t* dst = ring + (size_t) slot * p.ring.slot_bytes;
                        if (valid) {
                            mbar_arrive_expect_tx(&S.full[slot], wbytes + (uint32_t) bbytes);
                            tma_load_3d(dst, gtm, 0, blk * 8, ks0 + st * kMoeSK, &S.full[slot]);
                            bulk_g2s(dst + p.ring.wpart, bsrc + (int64_t) st * bbytes, (uint32_t) bbytes, &S.full[slot]);
                        } else {
                            mbar_arrive(&S.full[slot]);
                        }
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
                ++it;
                PHASE_MARK(PH_PROD_ISSUE);
            }
            UT_MARK(ticket, 3);
            // Claim the next unit only once at most `ahead` stages of this CTA's
            // ring are unconsumed: a CTA with a long backlog leaves the last
            // tickets to idle CTAs instead of ending the layer late.  (Stage j is
            // consumed when empty[j % ns] completes phase j / ns; ahead <= ns - 2
            // keeps that phase the barrier's latest.)
            int next_raw = total;
            if (lane == 0 && ok) {
                const uint32_t ns = (uint32_t) p.ring.ns;
                const uint32_t ahead = min((uint32_t) p.claim_ahead, ns - 2u);
                if (it > ahead) {
                    const uint32_t j = it - ahead - 1u;
                    ok = mbar_wait(&S.empty[j % ns], (j / ns) & 1u, status);
                }
                if (ok) next_raw = (int) atomicAdd(&p.ctrl[0], 1u);
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            ticket = __shfl_sync(0xffffffffu, next_raw, 0);
            if (!ok) break;
        }
        // no bulk copy may still be writing shared memory when the CTA retires
        if (lane == 0) {
            const uint32_t first = it > (uint32_t) p.ring.ns ? it - (uint32_t) p.ring.ns : 0u;
            for (uint32_t i = first; i < it; ++i)
                if (!mbar_wait(&S.full[i % p.ring.ns], (i / p.ring.ns) & 1u, status)) break;
        }
        TL_MARK(4);
        PHASE_FLUSH(lane);
    } else if (warp == kMoeEpilogueWarp) {
        // ------------------------------------------------------------ epilogue
        // Stores each unit's partial tile, counts completions per block and runs
        // the block epilogues, off the consumers' critical path.
        PHASE_DECL
        uint32_t du = 0, uu = 0;
        while (true) {
            const int slot = du % kMoeDQ;
            if (!mbar_wait_lanes(&S.dqf[slot], (du / kMoeDQ) & 1u, status)) break;
            int d[6];
#pragma unroll
            for (int q = 0; q < 6; ++q) d[q] = S.desc[slot][q];
#ifdef EXL3_TIMELINE
            const int tk_ = S.desc[slot][6];
#endif
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.dqe[slot]);
            ++du;
            PHASE_MARK(PH_EPI_DESC);
            if (d[0] < 0) break;
            const int kind = d[0], g = d[1], mat = d[2], blk = d[3], s = d[4], K = d[5];
            if (K == 0) continue;
            const bool single = kind == 1 && p.nkb == 1;
            uint2 sv4 = make_uint2(0u, 0u);   // the block's svh, loaded while the tile is computed
            if (single)
                sv4 = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.tab[8][P.gexp[g]]) +
                                                           blk * kCols + lane * 4));
            const int ps = (int) (uu & 1u);
            if (!mbar_wait_lanes(&S.pfull[ps], (uu >> 1) & 1u, status)) break;
            PHASE_MARK(PH_EPI_WAIT);
            const int nrows = __popc(P.gmask[g]), pair0 = P.gpair[g];
            const float* tile = ptile + (size_t) ps * p.m * kCols;
            if (single) {
                // A single k-chunk over I: the tile is the block's whole sum, so it
                // is finished here without a partial store or a completion count.
                PHASE_COUNT(PH_FINS_B);
                moe_finish_b_rows(p, P, g, blk, lane, tile, &sv4);
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&S.pempty[ps]);
                    red_add_release_gpu(&cntG[blk], 1u);
                }
                ++uu;
                PHASE_MARK(PH_FIN_B);
                UT_MARK(tk_, 6);
                continue;
            }
            for (int r = 0; r < nrows; ++r) {
                const float4 v = *reinterpret_cast<const float4*>(tile + r * kCols + lane * 4);
                float* dst = kind == 0
                    ? p.partA + (((int64_t) (pair0 + r) * 2 + mat) * p.nka + s) * p.I + blk * kCols
                    : p.partB + ((int64_t) (pair0 + r) * p.nkb + s) * p.H + blk * kCols;
                __stcg(reinterpret_cast<float4*>(dst + lane * 4), v);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.pempty[ps]);
            ++uu;
            int last = 0;
            if (lane == 0) {
                uint32_t* cnt = kind == 0 ? &cntA[g * kNBImax + blk] : &cntB[g * kNBHmax + blk];
                const uint32_t target = kind == 0 ? (uint32_t) (2 * p.nka) : (uint32_t) p.nkb;
                // release this unit's partial (the whole warp's stores, ordered by
                // the __syncwarp above)
                // release this unit's partial; the last unit also acquires the others'
                const uint32_t old = atom_add_acq_rel_gpu(cnt, 1u);
                last = old == target - 1u;
                if (last) atomicExch(cnt, 0u);
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            PHASE_MARK(PH_EPI_STORE);
            UT_MARK(tk_, 6);
            if (!last) continue;
            if (kind == 0) {
                PHASE_COUNT(PH_FINS_A);
                moe_finish_a<PRECISE>(p, P, g, blk, lane);
                __syncwarp();
                if (lane == 0) {
                    fence_proxy_async_global();   // release the down-input fragments
                    red_add_release_gpu(&readyB[g * kMoeMaxNkb + (blk * kCols) / p.kcb], 1u);
                }
                PHASE_MARK(PH_FIN_A);
            } else {
                PHASE_COUNT(PH_FINS_B);
                moe_finish_b_rows(p, P, g, blk, lane, nullptr, nullptr);
                moe_finish_b_count(blk, lane, cntG);
                PHASE_MARK(PH_FIN_B);
            }
        }
        TL_MARK(5);
        PHASE_FLUSH(lane);
    } else {
        // ------------------------------------------------------------ consumers
        // Phase P: input transforms, item i to consumer warp i of the grid
        // (strided).  Every CTA reaches this point right after its dependency
        // wait, so a fixed share needs no claim: a shared claim counter cost
        // thousands of same-address atomics at the start of every layer.
        PHASE_DECL
        const int NKB = p.H / kCols;
        const int PI = G * 2 * NKB;
        const int nw = (int) gridDim.x * kMoeConsumerWarps;
        for (int item = (int) blockIdx.x * kMoeConsumerWarps + warp; item < PI; item += nw) {
            const int g = item / (2 * NKB);
            const int r = item % (2 * NKB);
            const int mat = r / NKB, kb = r % NKB;
            moe_input_item<PRECISE>(p, P, g, mat, kb, lane);
            __syncwarp();
            if (lane == 0) {
                fence_proxy_async_global();
                red_add_release_gpu(&readyP[(g * 2 + mat) * kMoeMaxNka + kb / (p.kca / kCols)], 1u);
            }
        }
        PHASE_MARK(PH_P);
        if (warp == 0) TL_MARK(2);

        uint32_t it = 0, du = 0, uu = 0;
        const int t4 = lane & 3, gr = lane >> 2;
        while (true) {
            const int slot = du % kMoeDQ;
            if (!mbar_wait_lanes(&S.dqf[slot], (du / kMoeDQ) & 1u, status)) break;
            PHASE_MARK(PH_DESC);
            int d[6];
#pragma unroll
            for (int q = 0; q < 6; ++q) d[q] = S.desc[slot][q];
#ifdef EXL3_TIMELINE
            const int tk_ = S.desc[slot][6];
            if (warp == 0) UT_MARK(tk_, 4);
#endif
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.dqe[slot]);
            ++du;
            if (d[0] < 0) break;
            const int kind = d[0], g = d[1], K = d[5];
            if (K == 0) continue;
            const int nrows = __popc(P.gmask[g]);
            const int nst = (kind == 0 ? p.kca : p.kcb) / (16 * kMoeSK);
            float acc[4][4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
            const bool ok = ring_consume_any<CB, PRECISE>(K, row_blocks(nrows), p.ring, ring, S.full, S.empty, it, nst,
                                                         nrows, acc, warp, lane, status PH_ARG);
            PHASE_MARK(PH_UNIT);
            PHASE_COUNT(PH_UNITS);
            if (!ok) break;
#ifdef EXL3_TIMELINE
            if (warp == 0) UT_MARK(tk_, 5);
#endif
            // this warp's 16 columns into the partial tile: D fragment (ch gr, row 2t),
            // (gr, 2t+1), (gr+8, 2t), (gr+8, 2t+1)
            const int ps = (int) (uu & 1u);
            if (!mbar_wait_lanes(&S.pempty[ps], ((uu >> 1) + 1u) & 1u, status)) break;
            float* tile = ptile + (size_t) ps * p.m * kCols;
            const int col = warp * 16 + gr;
#pragma unroll
            for (int rb = 0; rb < 4; ++rb) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = rb * 8 + 2 * t4 + h;
                    if (r < nrows) {
                        tile[r * kCols + col] = acc[rb][h];
                        tile[r * kCols + col + 8] = acc[rb][2 + h];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.pfull[ps]);
            ++uu;
            PHASE_MARK(PH_PARTIAL);
        }
        if (warp == 0) TL_MARK(3);
        PHASE_FLUSH(lane);
    }

    // Retire: the last CTA out restores the control region for the next launch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&p.ctrl[1], 1u);
        S.last_cta = old == gridDim.x - 1;
        TL_MARK(6);
        S.retire_rank = (int) old;
    }
    __syncthreads();
    if (G > 0) {
        // Gather (and with TP the sum over ranks): the k-th CTA to retire --
        // its units are done and no ticket is left, so its waits hold up
        // nothing -- takes output blocks k, k + grid, ...: once every group
        // has counted the block, all ten warps gather one row each, so the
        // rows' L2 round trips overlap instead of running one after another.
        bool ok = true;
        for (int blk = S.retire_rank; blk < NBH; blk += (int) gridDim.x) {
            int done = 1;
            if (tid == 0) {
                done = wait_counter(&cntG[blk], (uint32_t) G, status) ? 1 : 0;
                atomicExch(&cntG[blk], 0u);   // every group has counted: restore for the next launch
                fence_acq_rel_gpu();          // acquire every group's down output of the block
            }
            if (!__syncthreads_and(done)) break;
            for (int r = warp; r < p.m; r += kMoeThreads / 32) moe_gather_row(p, P, blk, r, lane, S.tp_epoch);
            if (p.tp_world > 0)
                for (int r = warp; r < p.m; r += kMoeThreads / 32) tp_finish_row(p, S.tp_epoch, blk, r, lane, ok);
        }
        ok = __all_sync(0xffffffffu, ok);
        if (!ok && lane == 0) set_error(status, ERR_DEP_TIMEOUT);
    }
    if (tid == 0) TL_MARK(7);
    if (S.last_cta) {
        __threadfence();
        for (int i = tid; i < G * 2 * kMoeMaxNka; i += kMoeThreads) readyP[i] = 0u;
        for (int i = tid; i < G * kMoeMaxNkb; i += kMoeThreads) readyB[i] = 0u;
        if (tid == 0) {
            atomicExch(&p.ctrl[0], 0u);
            atomicExch(&p.ctrl[1], 0u);
            // the next launch exchanges under the next epoch
            if (p.tp_world > 0) atomicExch(reinterpret_cast<uint32_t*>(p.tp_bufs[p.tp_rank]), S.tp_epoch);
        }
    }
}

// ------------------------------------------------------------------ host side
namespace {

// Number of k-chunks of a dimension of `n` elements: the smallest count
// >= ceil(n / kchunk) that splits it into whole 128-element blocks, at most
// `cap` (the largest such divisor otherwise).
int chunks_for(int64_t n, int cap, int kchunk) {
    const int64_t blocks = n / 128;
    const int lo = (int) ((n + kchunk - 1) / kchunk);
    for (int c = lo; c <= cap; ++c)
        if (blocks % c == 0) return c;
    for (int c = cap; c >= 1; --c)
        if (blocks % c == 0) return c;
    return 1;
}

struct MoeGeom {
    int kca, nka, kcb, nkb;
    int64_t pairs;
    int64_t off_tmaps, off_partA, off_xg, off_ag, off_partB, off_downc, total;
};

// Target k-chunk of the units: 2048 when the gate/up units at that size alone
// still give every CTA four or more -- long units pay their per-unit costs
// (claim, tensor-map update, dependency check, partial hand-off) less often,
// and with a single down chunk the down partials are finished from shared
// memory (config 2: 200 -> 192 us per layer) -- else 1024: the TP shards,
// whose few long units would leave CTAs idle (TP8: 44 -> 48 us at 2048).
// `grid` 0 gives 1024, the choice that needs the most scratch.
int moe_kchunk(int64_t m, int64_t topk, int64_t E, int64_t H, int64_t I, int grid) {
    if (grid <= 0) return 1024;
    const int64_t gmax = std::min<int64_t>(E, m * topk);
    const int64_t units = gmax * (I / 128) * 2 * chunks_for(H, kMoeMaxNka, 2048);
    return units >= 4 * (int64_t) grid ? 2048 : 1024;
}

// Scratch geometry (fragments sized for the fast path's 4 words per lane,
// which the precise path's 2 words also fit).  Fewer chunks never need more
// scratch, so the 1024 geometry bounds every choice.
MoeGeom moe_geom(int64_t m, int64_t topk, int64_t H, int64_t I, int kchunk = 1024) {
    MoeGeom g{};
    g.nka = chunks_for(H, kMoeMaxNka, kchunk);
    g.kca = (int) (H / g.nka);
    g.nkb = chunks_for(I, kMoeMaxNkb, kchunk);
    g.kcb = (int) (I / g.nkb);
    g.pairs = m * topk;
    int64_t off = EXL3_MOE_CTRL_BYTES;
    g.off_tmaps = off;                               // per-CTA tensor-map slots
    off = align_up(off + (int64_t) kMoeMaxGrid * kMoeTmapSlots * (int64_t) sizeof(CUtensorMap), 256);
    g.off_partA = off;
    off = align_up(off + g.pairs * 2 * g.nka * I * 4, 256);
    g.off_xg = off;                                  // per pair: 2 projections x H x FW bytes
    off = align_up(off + g.pairs * 2 * H * 4, 256);
    g.off_ag = off;                                  // per pair: I x FW bytes
    off = align_up(off + g.pairs * I * 4, 256);
    g.off_partB = off;                               // with one I chunk the partials alias downc
    off = align_up(off + (g.nkb > 1 ? g.pairs * g.nkb * H * 4 : 0), 256);
    g.off_downc = off;
    off = align_up(off + g.pairs * H * 4, 256);
    g.total = off;
    return g;
}

// Ring stage: the weight part (SK k-slices x 8 tiles at the launch's largest
// K) and the B fragments of SK k-slices of up to m rows; as many stages as fit
// the budget left after the two partial tiles (2 x m x 128 floats), 2 to 12.
void ring_geom(int64_t m, int kmax, bool precise, int* wpart, int* slot_bytes, int* ns) {
    const int fw = precise ? 2 : 4;
    *wpart = kMoeSK * 8 * 32 * kmax;
    *slot_bytes = *wpart + kMoeSK * (int) m * 16 * fw;
    const int budget = kMoeRingBytes - 2 * (int) m * kCols * 4;
    int n = budget / *slot_bytes;
    *ns = n < 2 ? 2 : (n > kMoeMaxStages ? kMoeMaxStages : n);
}

// The largest case (32 rows, 4-word fragments): 2 stages of 24 KB + 32 KB of
// partial tiles fit the budget.
static_assert(2 * (kMoeWBytes + kMoeSK * kMoeMaxRows * 64) + 2 * kMoeMaxRows * kCols * 4 <= kMoeRingBytes,
              "ring budget below 2 stages");
int moe_smem_max() { return kMoeHeadBytes + kMoeRingBytes; }

// Tensor-map templates per (hidden, intermediate): kind 0 = gate/up
// [H/16][I/16][16K], kind 1 = down [I/16][H/16][16K]; box = [16K, 8, SK].
// Encoded once on the host (cuTensorMapEncodeTiled through the runtime's
// driver entry point) with a placeholder address that every unit replaces.
struct MoeTemplates {
    CUtensorMap t[8];
};

int encode_templates(int64_t H, int64_t I, void* placeholder, MoeTemplates* out) {
    static std::mutex mu;
    static std::map<std::pair<int64_t, int64_t>, MoeTemplates> cache;
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({H, I});
    if (it != cache.end()) {
        *out = it->second;
        return EXL3_OK;
    }
    if (encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        EXL3_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        EXL3_REQUIRE(fn != nullptr && q == cudaDriverEntryPointSuccess, EXL3_ERR_CUDA,
                     "moe: cuTensorMapEncodeTiled is not available from the driver");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    MoeTemplates T{};
    for (int kind = 0; kind < 2; ++kind)
        for (int K = 1; K <= kMoeKmax; ++K) {
            const cuuint64_t ncols = (cuuint64_t) ((kind == 0 ? I : H) / 16);
            const cuuint64_t nks = (cuuint64_t) ((kind == 0 ? H : I) / 16);
            const cuuint64_t dims[3] = {(cuuint64_t) (16 * K), ncols, nks};
            const cuuint64_t strides[2] = {(cuuint64_t) (32 * K), ncols * (cuuint64_t) (32 * K)};
            const cuuint32_t box[3] = {(cuuint32_t) (16 * K), 8u, (cuuint32_t) kMoeSK};
            const cuuint32_t estr[3] = {1u, 1u, 1u};
            const CUresult r = encode(&T.t[kind * 4 + K - 1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, placeholder, dims,
                                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "moe: cuTensorMapEncodeTiled failed (%d) for K=%d",
                         (int) r, K);
        }
    cache[{H, I}] = T;
    *out = T;
    return EXL3_OK;
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
        const int smem = moe_smem_max();
        auto kern = moe_kernel<CB, PRECISE>;
        EXL3_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        int res = 0;
        EXL3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, kern, kMoeThreads, smem));
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
    int slot = 0, ns = 0;
    int wpart = 0;
    ring_geom(4, kmax, false, &wpart, &slot, &ns);
    const int64_t v[14] = {pr.sms, pr.resident, kMoeThreads / 32, pr.grid, kMoeThreads, 3, ns,
                           kMoeMaxRows, (int64_t) moe_smem_max(), EXL3_MOE_CTRL_BYTES,
                           exl3_moe_scratch_bytes(kMoeMaxRows, 8, 4096, 2048), kMoeMaxRows, kMoeMaxSlots, 1};
    for (int i = 0; i < 14; ++i) info[i] = v[i];
    return EXL3_OK;
}

#ifdef EXL3_PHASE_CLOCK
// Phase-clock readout of the instrumented build (not part of the release
// ABI): copies the accumulated per-phase cycle sums, optionally zeroing them.
extern "C" int exl3_phase_clock_read(unsigned long long* out, int n, int reset) {
    EXL3_REQUIRE(out && n >= 1 && n <= exl3::PH_N, EXL3_ERR_ARG, "phase clock: bad output");
    EXL3_CUDA(cudaDeviceSynchronize());
    EXL3_CUDA(cudaMemcpyFromSymbol(out, exl3::g_phase, sizeof(unsigned long long) * n));
    if (reset) {
        unsigned long long z[exl3::PH_N] = {};
        EXL3_CUDA(cudaMemcpyToSymbol(exl3::g_phase, z, sizeof(z)));
    }
    return EXL3_OK;
}

#endif

#ifdef EXL3_TIMELINE
extern "C" int exl3_timeline_read(unsigned long long* out, int n) {
    EXL3_REQUIRE(out && n >= 1 && n <= 320 * 8, EXL3_ERR_ARG, "timeline: bad output");
    EXL3_CUDA(cudaDeviceSynchronize());
    EXL3_CUDA(cudaMemcpyFromSymbol(out, exl3::g_tl, sizeof(unsigned long long) * n));
    return EXL3_OK;
}

// Per-unit marks of the timeline build ([ticket][8], see UT_MARK); every
// launch rewrites the marks of its tickets.
extern "C" int exl3_unit_trace_read(unsigned long long* out, int n) {
    EXL3_REQUIRE(out && n >= 1 && n <= exl3::kUtMax * 8, EXL3_ERR_ARG, "unit trace: bad output");
    EXL3_CUDA(cudaDeviceSynchronize());
    EXL3_CUDA(cudaMemcpyFromSymbol(out, exl3::g_ut, sizeof(unsigned long long) * n));
    return EXL3_OK;
}
#endif

namespace exl3 {
namespace {

struct TpArgs {
    const int64_t* bufs = nullptr;   // device [world] exchange-buffer addresses
    int rank = 0, world = 0;
    int64_t mcap = 0;
};

int moe_decode_impl(const void* x, int x_dtype, void* out, int out_dtype, int64_t m, int64_t hidden, int64_t inter,
                    const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                    const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                    const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh, int64_t n_experts,
                    const int32_t* k_table, int K, int kmax, int cb, const RouteIn& route, int64_t topk,
                    float swiglu_limit, void* scratch, int64_t scratch_bytes, int precise, const TpArgs& tp,
                    void* stream) {
    EXL3_REQUIRE(x && out && route.ids && route.weights && scratch, EXL3_ERR_ARG, "moe: null pointer argument");
    EXL3_REQUIRE(route.ids64 == 0 || route.ids64 == 1, EXL3_ERR_ARG, "moe: ids dtype must be 0 (int32) or 1 (int64)");
    EXL3_REQUIRE(route.w_dtype >= 0 && route.w_dtype <= 2, EXL3_ERR_ARG, "moe: routing weight dtype code out of range");
    EXL3_REQUIRE(route.emap == nullptr || (route.n_global >= 1 && route.n_global <= (int64_t) 1 << 31), EXL3_ERR_ARG,
                 "moe: expert map must have 1..2^31 entries");
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
    // the scratch is checked against exl3_moe_scratch_bytes (the most any k-chunk choice needs)
    const int64_t need = moe_geom(m, topk, hidden, inter).total;
    EXL3_REQUIRE(scratch_bytes >= need, EXL3_ERR_ARG, "moe: scratch too small (%lld < %lld bytes)",
                 (long long) scratch_bytes, (long long) need);
    MoePrepared pr;
    if (int rc = moe_prepare_any(cb, precise != 0, &pr)) return rc;
    const MoeGeom g = moe_geom(m, topk, hidden, inter, moe_kchunk(m, topk, n_experts, hidden, inter, pr.grid));
    EXL3_REQUIRE(g.kca % (kMoeSK * 16) == 0 && g.kcb % (kMoeSK * 16) == 0 && g.nka <= kMoeMaxNka &&
                     g.nkb <= kMoeMaxNkb, EXL3_ERR_UNSUPPORTED,
                 "moe: internal k-chunks (%d, %d) do not tile the ring stages", g.kca, g.kcb);

    MoeParams p{};
    p.x = x;
    p.out = out;
    for (int i = 0; i < 9; ++i) p.tab[i] = tabs[i];
    p.ktab = k_table;
    p.kuni = K;
    p.route = route;
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
    p.claim_ahead = std::max(1, std::min({kMoeClaimAhead, g.kca / (16 * kMoeSK), g.kcb / (16 * kMoeSK)}));
    uint8_t* sb = static_cast<uint8_t*>(scratch);
    EXL3_REQUIRE(pr.grid <= kMoeMaxGrid, EXL3_ERR_UNSUPPORTED, "moe: grid %d above %d", pr.grid, kMoeMaxGrid);
    MoeTemplates tmpl;
    if (int rc = encode_templates(hidden, inter, sb + g.off_tmaps, &tmpl)) return rc;
    for (int i = 0; i < 8; ++i) p.tmpl[i] = tmpl.t[i];
    p.tmaps = reinterpret_cast<CUtensorMap*>(sb + g.off_tmaps);
    p.ctrl = reinterpret_cast<uint32_t*>(sb);
    p.partA = reinterpret_cast<float*>(sb + g.off_partA);
    p.xg = reinterpret_cast<uint32_t*>(sb + g.off_xg);
    p.ag = reinterpret_cast<uint32_t*>(sb + g.off_ag);
    p.downc = reinterpret_cast<float*>(sb + g.off_downc);
    // With a single k-chunk over I a block's partial is its full sum: the
    // epilogue reads it and writes the transformed value in place.
    p.partB = g.nkb > 1 ? reinterpret_cast<float*>(sb + g.off_partB) : p.downc;
    p.tp_bufs = tp.bufs;
    p.tp_rank = tp.rank;
    p.tp_world = tp.world;
    p.tp_mcap = (int) tp.mcap;
    ring_geom(m, k_table ? kmax : K, precise != 0, &p.ring.wpart, &p.ring.slot_bytes, &p.ring.ns);
    shift_table_init(p.ring.st);

    const int smem = kMoeHeadBytes + p.ring.ns * p.ring.slot_bytes + 2 * (int) m * kCols * 4;
    auto s = static_cast<cudaStream_t>(stream);
    void (*kern)(MoeParams) = nullptr;
    if (precise) kern = cb == 0 ? moe_kernel<0, true> : (cb == 1 ? moe_kernel<1, true> : moe_kernel<2, true>);
    else kern = cb == 0 ? moe_kernel<0, false> : (cb == 1 ? moe_kernel<1, false> : moe_kernel<2, false>);
    // programmatic stream serialization: see the kernel's prologue
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned) pr.grid);
    cfg.blockDim = dim3((unsigned) kMoeThreads);
    cfg.dynamicSmemBytes = (size_t) smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    EXL3_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
    return EXL3_OK;
}

}  // namespace
}  // namespace exl3

extern "C" int exl3_moe_decode(const void* x, int x_dtype, void* out, int out_dtype, int64_t m, int64_t hidden,
                               int64_t inter, const int64_t* gate_trellis, const int64_t* gate_suh,
                               const int64_t* gate_svh, const int64_t* up_trellis, const int64_t* up_suh,
                               const int64_t* up_svh, const int64_t* down_trellis, const int64_t* down_suh,
                               const int64_t* down_svh, int64_t n_experts, const int32_t* k_table, int K, int kmax,
                               int cb, const int32_t* ids, const float* weights, int64_t topk, float swiglu_limit,
                               void* scratch, int64_t scratch_bytes, int precise, void* stream) {
    const exl3::RouteIn route{ids, weights, nullptr, 0, 0, 2};
    return exl3::moe_decode_impl(x, x_dtype, out, out_dtype, m, hidden, inter, gate_trellis, gate_suh, gate_svh,
                                 up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh, n_experts, k_table, K,
                                 kmax, cb, route, topk, swiglu_limit, scratch, scratch_bytes, precise,
                                 exl3::TpArgs{}, stream);
}

namespace exl3 {
// The C-ABI route descriptor as the kernels' RouteIn (an error code when it is invalid).
int route_from_abi(const exl3_moe_route* r, RouteIn* out) {
    EXL3_REQUIRE(r != nullptr, EXL3_ERR_ARG, "moe: null route descriptor");
    EXL3_REQUIRE(r->ids_dtype == 0 || r->ids_dtype == 1, EXL3_ERR_ARG,
                 "moe: route ids_dtype must be 0 (int32) or 1 (int64)");
    EXL3_REQUIRE(r->weights_dtype >= EXL3_DTYPE_F16 && r->weights_dtype <= EXL3_DTYPE_F32, EXL3_ERR_ARG,
                 "moe: route weights_dtype must be fp16, bf16 or fp32");
    EXL3_REQUIRE(r->expert_map == nullptr || r->n_global >= 1, EXL3_ERR_ARG,
                 "moe: route expert_map given with n_global < 1");
    *out = RouteIn{r->ids, r->weights, r->expert_map, r->expert_map ? r->n_global : 0, r->ids_dtype,
                   r->weights_dtype};
    return EXL3_OK;
}
}  // namespace exl3

extern "C" int exl3_moe_decode_routed(const void* x, int x_dtype, void* out, int out_dtype, int64_t m,
                                      int64_t hidden, int64_t inter, const int64_t* gate_trellis,
                                      const int64_t* gate_suh, const int64_t* gate_svh, const int64_t* up_trellis,
                                      const int64_t* up_suh, const int64_t* up_svh, const int64_t* down_trellis,
                                      const int64_t* down_suh, const int64_t* down_svh, int64_t n_experts,
                                      const int32_t* k_table, int K, int kmax, int cb, const exl3_moe_route* route,
                                      int64_t topk, float swiglu_limit, void* scratch, int64_t scratch_bytes,
                                      int precise, const int64_t* tp_bufs, int tp_rank, int tp_world,
                                      int64_t tp_max_rows, void* stream) {
    exl3::RouteIn r;
    if (int rc = exl3::route_from_abi(route, &r)) return rc;
    exl3::TpArgs tp;
    if (tp_bufs != nullptr) {
        EXL3_REQUIRE(tp_world >= 1 && tp_world <= 32 && tp_rank >= 0 && tp_rank < tp_world, EXL3_ERR_ARG,
                     "moe tp: rank %d of world %d out of range (world 1..32)", tp_rank, tp_world);
        EXL3_REQUIRE(m <= tp_max_rows && tp_max_rows <= exl3::kMoeMaxRows, EXL3_ERR_ARG,
                     "moe tp: m = %lld above the exchange buffers' row capacity %lld", (long long) m,
                     (long long) tp_max_rows);
        tp.bufs = tp_bufs;
        tp.rank = tp_rank;
        tp.world = tp_world;
        tp.mcap = tp_max_rows;
    }
    return exl3::moe_decode_impl(x, x_dtype, out, out_dtype, m, hidden, inter, gate_trellis, gate_suh, gate_svh,
                                 up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh, n_experts, k_table, K,
                                 kmax, cb, r, topk, swiglu_limit, scratch, scratch_bytes, precise, tp, stream);
}

// ------------------------------------------------------------------ fused tensor-parallel sum
extern "C" int64_t exl3_tp_buffer_bytes(int world, int64_t max_rows, int64_t hidden) {
    if (world < 1 || world > 32 || max_rows < 1 || max_rows > exl3::kMoeMaxRows || hidden < 128 ||
        hidden > exl3::kMoeMaxHidden || hidden % 128)
        return -1;
    return exl3::tp_buffer_bytes_for(world, max_rows, hidden);
}

extern "C" int exl3_tp_buffer_alloc(int world, int64_t max_rows, int64_t hidden, void** out) {
    EXL3_REQUIRE(out, EXL3_ERR_ARG, "tp buffer: null output pointer");
    const int64_t bytes = exl3_tp_buffer_bytes(world, max_rows, hidden);
    EXL3_REQUIRE(bytes > 0, EXL3_ERR_ARG, "tp buffer: world 1..32, rows 1..%d, hidden a multiple of 128 <= %d",
                 exl3::kMoeMaxRows, exl3::kMoeMaxHidden);
    void* p = nullptr;
    EXL3_CUDA(cudaMalloc(&p, (size_t) bytes));
    const cudaError_t e = cudaMemset(p, 0, (size_t) bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        EXL3_CUDA(e);
    }
    *out = p;
    return EXL3_OK;
}

extern "C" int exl3_tp_buffer_free(void* p) {
    if (p) EXL3_CUDA(cudaFree(p));
    return EXL3_OK;
}

extern "C" int exl3_tp_ipc_handle(void* p, void* handle) {
    EXL3_REQUIRE(p && handle, EXL3_ERR_ARG, "tp ipc: null pointer");
    cudaIpcMemHandle_t h;
    EXL3_CUDA(cudaIpcGetMemHandle(&h, p));
    memcpy(handle, &h, sizeof(h));
    return EXL3_OK;
}

extern "C" int exl3_tp_ipc_open(const void* handle, void** out) {
    EXL3_REQUIRE(handle && out, EXL3_ERR_ARG, "tp ipc: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    EXL3_CUDA(cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
    return EXL3_OK;
}

extern "C" int exl3_tp_ipc_close(void* p) {
    if (p) EXL3_CUDA(cudaIpcCloseMemHandle(p));
    return EXL3_OK;
}

extern "C" int exl3_moe_decode_tp(const void* x, int x_dtype, void* out, int out_dtype, int64_t m, int64_t hidden,
                                  int64_t inter, const int64_t* gate_trellis, const int64_t* gate_suh,
                                  const int64_t* gate_svh, const int64_t* up_trellis, const int64_t* up_suh,
                                  const int64_t* up_svh, const int64_t* down_trellis, const int64_t* down_suh,
                                  const int64_t* down_svh, int64_t n_experts, const int32_t* k_table, int K, int kmax,
                                  int cb, const int32_t* ids, const float* weights, int64_t topk,
                                  float swiglu_limit, void* scratch, int64_t scratch_bytes, int precise,
                                  const int64_t* tp_bufs, int tp_rank, int tp_world, int64_t tp_max_rows,
                                  void* stream) {
    EXL3_REQUIRE(tp_bufs, EXL3_ERR_ARG, "moe tp: null exchange-buffer table");
    EXL3_REQUIRE(tp_world >= 1 && tp_world <= 32 && tp_rank >= 0 && tp_rank < tp_world, EXL3_ERR_ARG,
                 "moe tp: rank %d of world %d out of range (world 1..32)", tp_rank, tp_world);
    EXL3_REQUIRE(m <= tp_max_rows && tp_max_rows <= exl3::kMoeMaxRows, EXL3_ERR_ARG,
                 "moe tp: m = %lld above the exchange buffers' row capacity %lld", (long long) m,
                 (long long) tp_max_rows);
    exl3::TpArgs tp;
    tp.bufs = tp_bufs;
    tp.rank = tp_rank;
    tp.world = tp_world;
    tp.mcap = tp_max_rows;
    const exl3::RouteIn route{ids, weights, nullptr, 0, 0, 2};
    return exl3::moe_decode_impl(x, x_dtype, out, out_dtype, m, hidden, inter, gate_trellis, gate_suh, gate_svh,
                                 up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh, n_experts, k_table, K,
                                 kmax, cb, route, topk, swiglu_limit, scratch, scratch_bytes, precise, tp, stream);
}

// ------------------------------------------------------------------ allocation-free variant
// exl3_moe_decode_noalloc: the same layer as exl3_moe_decode for callers that
// cannot allocate device memory at all -- a plugin inside a serving process
// whose device memory is owned by the host's caching allocator (no cudaMalloc
// of its own, and no buffer handed to it), and latency-critical callers that
// cannot afford cudaMalloc's implicit synchronization.  Its scratch is the
// array below, compiled into the library: EXL3_MOE_STATIC_SCRATCH_BYTES
// (8 MiB) of device memory that every GPU which loads the library holds until
// the process exits.  Geometries whose scratch (exl3_moe_scratch_bytes)
// exceeds it are rejected.
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
