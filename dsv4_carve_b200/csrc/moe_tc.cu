// moe_tc.cu -- routed-expert MoE layer for prefill chunks (many rows per
// expert) on the tcgen05 tensor cores.
//
// Replaces the fused prefill launch exl3_moe (orders/F1-ref/exl3_moe.cu:99-301,
// orders/F1-ref/exl3_moe_kernel.cuh:17-283) together with the torch glue the
// plugin runs around it (argsort / scatter_add counts / TEMP_ROWS_FUSED
// slicing, recipe-lna/vllm_exl3_exl3.py.lna:1597-1704): the route plan is
// built on the device.  Numerics are those of the decode layer
// (recipe-lna/lna2/lna_moe_ticket.cu:5-12; semantic reference
// recipe-lna/vllm_exl3_exl3.py.lna:988-1027): gate / up accumulate fp32 over
// the fp16-rounded decoded weights, output Hadamard * svh in fp32,
// silu(min(g, L)) * clamp(u, -L, L) -> fp16, * down suh, Hadamard -> fp16,
// down fp32, output Hadamard * svh, per-token slot-order fp32 sum, one cast.
//
// Four launches per chunk of <= 2048 tokens, chained with programmatic
// dependent launch:
//  1. pf_plan_kernel (one CTA): per-expert token bitmasks -> counts -> pairs
//     (expert, token) sorted by expert then token; slot -> pair; per-expert
//     offsets of pairs, 128-row passes and work units; clears the counters.
//  2. pf_input_kernel: every (pair, gate|up, 128-block of hidden): x -> fp16,
//     * suh, Hadamard -> fp16 rows of xg / xu [pairs][hidden].
//  3. pf_gemm_kernel (persistent, one CTA per SM): units from one ticket
//     counter, all gate/up units (expert, 128-column strip of I, 128-row pass)
//     before all down units (expert, 128-column strip of hidden, 128-row
//     pass).  A down unit waits (bounded) until the 128-column strips of its
//     pass are all written; those come only from gate/up units, claimed
//     earlier and never waiting, so no co-residency is assumed.
//       warp 16 (producer)  claims tickets, publishes unit descriptors, streams
//                           per 64-k step the packed weights (bulk copies of
//                           whole k-slice rows of 8 tiles) and the pass's
//                           activation rows (2-D TMA, 128-byte swizzle);
//       warps 0-15          decode the weight tiles, round to fp16 and write
//                           them K-major / swizzled as the MMA's A operand;
//       warp 17             owns 512 TMEM columns (two accumulator sets) and
//                           issues tcgen05.mma: D[column][row] over the rows
//                           of the pass (N = rows rounded to 16);
//       warps 18-21         epilogue, overlapping the next unit's mainloop:
//                           TMEM -> shared -> per row: gate/up: out-H * svh,
//                           SwiGLU, * down suh, Hadamard -> fp16 down input;
//                           down: out-H * svh -> fp32 down output rows.
//  4. pf_gather_kernel: out[t] = sum over slots, in slot order, of
//     weight * down output row of the slot's pair; one cast.
// Every wait is bounded (2 s); a wait that runs out sets a status bit and the
// roles wind down; TMEM is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <type_traits>
#include <utility>

#include "host.hpp"
#include "tcgen05.cuh"

namespace exl3 {

constexpr int kPfDecWarps = 16;
constexpr int kPfProducerWarp = 16;             // tickets, weight tensor maps, weight stages
constexpr int kPfMmaWarp = 17;
constexpr int kPfEpiWarp0 = 18;                 // warps 18..21: TMEM lane groups 2, 3, 0, 1
constexpr int kPfEpiWarps = 4;
constexpr int kPfXWarp = 22;                    // activation stages (and the down units' dependency waits)
constexpr int kPfThreads = (kPfXWarp + 1) * 32;
constexpr int kPfRows = 64;                     // rows per pass (MMA N <= 64)
constexpr int kPfKStep = 64;                    // k per step (4 k-slices)
constexpr int kPfKmax = 4;                      // largest bit width
constexpr int kPfBoxRows = 16;                 // rows per activation TMA box
constexpr int kPfBoxBytes = kPfBoxRows * 128;   // [16 rows][64 k] fp16
constexpr int kPfXBox = kPfRows * 128;          // one matrix's activation tile [128 rows][64 k] fp16
constexpr int kPfXStage = 2 * kPfXBox;          // gate + up tiles
constexpr int kPfXStages = 3;
constexpr int kPfAStage = 2 * 128 * 128;        // gate + up decoded tiles [128 cols][64 k] fp16
constexpr int kPfAStages = 3;
static_assert(kPfAStages == 3 && kPfXStages == 3, "one commit frees a step's decoded weights and activations together");
constexpr int kPfWStage = 2 * 4 * 8 * 32 * kPfKmax;   // 2 matrices x 4 k-slices x 8 tiles at K = 4
constexpr int kPfWStages = 6;
constexpr int kPfChunkRows = 32;                // epilogue staging rows
constexpr int kPfStageBytes = 2 * kPfChunkRows * 128 * 4;
constexpr int kPfDQ = 4;                        // unit descriptor queue depth
constexpr int kPfMaxTokens = 2048;              // tokens per plan (TEMP_ROWS_FUSED)
constexpr int kPfMaskWords = 16384;             // experts x token words of the plan's bitmasks
constexpr int kPfMaxExperts = 1024;
constexpr int kPfMaxTopk = 16;
constexpr int kPfCtrlWords = 16;                // [0] ticket [2] status [4] gate/up units [5] down units [6] pairs
constexpr int kPfCtrlBytes = 65536;             // control words + per-pass counters
constexpr int kPfMaxPasses = kPfCtrlBytes / 4 - kPfCtrlWords;
constexpr int kPfMapSlots = 8;                  // weight tensor maps per matrix per CTA, used in turn by units
static_assert(kPfMapSlots > kPfWStages, "a map slot is reused only after its copies have landed");
constexpr int kPfMaxGrid = 256;                 // CTAs the map slots are sized for
constexpr int kPfHeadBytes = 1024;

struct PfUnit {
    int mode;        // 0 gate/up, 1 down, -1 end
    int e;
    int K;
    int strip;
    int row0;        // first pair of the pass
    int rows;        // rows in the pass (1..128)
    int gp;          // global pass index
    int ksteps;
};

struct PfHead {
    CUtensorMap tmap[2];                        // staging of this unit's weight maps (128-byte aligned)
    uint64_t wfull[kPfWStages], wempty[kPfWStages];
    uint64_t aready[kPfAStages];
    uint64_t xfull[kPfXStages];
    uint64_t sfree[kPfAStages];                 // step buffers (decoded weights + activations) consumed by the MMAs
    uint64_t accfull[2], accfree[2];
    uint64_t dfull[kPfDQ], dempty[kPfDQ];
    PfUnit desc[kPfDQ];
    uint32_t tmem;
};
constexpr int kPfSmem = 1024 + kPfXStages * kPfXStage + kPfAStages * kPfAStage + kPfWStages * kPfWStage +
                        kPfStageBytes + kPfHeadBytes;
static_assert(sizeof(PfHead) <= kPfHeadBytes, "head must fit its slot");

struct PfPlan {
    int* e_off;      // [E + 1] first pair of each expert
    int* pass_off;   // [E + 1] first global pass of each expert
    int* gu_off;     // [E + 1] first gate/up unit of each expert
    int* dn_off;     // [E + 1] first down unit of each expert
    int* pair_tok;   // [cap] token of each pair
    int* pair_exp;   // [cap] expert of each pair
    int* slot_pair;  // [T * topk] pair of each slot, -1 if skipped
    int4* units;     // [unit cap] {expert, strip, first pair, rows | global pass << 8}: gate/up units, then down
    int unit_cap;
};

struct PfParams {
    CUtensorMap xg_map, xu_map, xd_map;   // [cap][H] / [cap][H] / [cap][I] fp16, box [64, 16], 128-byte swizzle
    CUtensorMap tmpl[8];                  // weight map templates [gate/up, down][K - 1], box [16K, 8, 4]
    CUtensorMap* maps;                    // [grid][kPfMapSlots][2] global slots the producer points at experts
    const int64_t* tab[9];
    const int32_t* ktab;
    int Kscalar;
    int E, H, I;
    float limit;
    uint32_t* ctrl;
    ShiftTable st;                        // IMAD shift multipliers of the window extraction
    PfPlan plan;
    __half* xd;
    float* dn;
};

// Compile-gated phase clocks (-DEXL3_PHASE_CLOCK): each role adds the
// cycles it spends in its waits into g_pf_phase; exl3_pf_phase_read copies
// them out.  Release builds compile all of it away.
#ifdef EXL3_PHASE_CLOCK
enum {
    PF_DEC_DESC, PF_DEC_W, PF_DEC_AFREE, PF_DEC_TOTAL,
    PF_MMA_DESC, PF_MMA_ACCFREE, PF_MMA_X, PF_MMA_A, PF_MMA_TOTAL,
    PF_PR_TICKET, PF_PR_DEMPTY, PF_PR_DEP, PF_PR_WEMPTY, PF_PR_XFREE, PF_PR_TOTAL,
    PF_EP_DESC, PF_EP_ACC, PF_EP_TOTAL, PF_UNITS, PF_XP_TOTAL, PF_N
};
__device__ unsigned long long g_pf_phase[PF_N];
struct PfClock {
    unsigned long long v[PF_N];
    unsigned long long t;
};
#define PFC_PARAM , PfClock& pfc
#define PFC_FWD , pfc
#define PFC_DECL PfClock pfc{}; pfc.t = clock64(); const unsigned long long pfc_start = pfc.t;
#define PFC_RESET() (pfc.t = clock64())
#define PFC_MARK(c) do { const unsigned long long n_ = clock64(); pfc.v[c] += n_ - pfc.t; pfc.t = n_; } while (0)
#define PFC_COUNT(c) (pfc.v[c] += 1)
#define PFC_FLUSH(total, lane) do { pfc.v[total] = clock64() - pfc_start; \
    if ((lane) == 0) for (int i_ = 0; i_ < PF_N; ++i_) if (pfc.v[i_]) atomicAdd(&g_pf_phase[i_], pfc.v[i_]); } while (0)
#else
#define PFC_PARAM
#define PFC_FWD
#define PFC_DECL
#define PFC_RESET()
#define PFC_MARK(c)
#define PFC_COUNT(c)
#define PFC_FLUSH(total, lane)
#endif

__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// Largest i in [0, n] with off[i] <= u (off ascending, off[0] = 0).
__device__ __forceinline__ int upper_slot(const int* off, int n, int u) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldcg(off + mid) <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ------------------------------------------------------------------ 1. plan
// Exclusive block scan of one value per thread (1024 threads); returns the
// prefix, writes the total to *total.
__device__ int block_scan_1024(int v, int* warp_tot, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = warp_tot[lane];
        int s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_tot[lane] = s - w;
        if (lane == 31) *total = s;
    }
    __syncthreads();
    const int r = x - v + warp_tot[warp];
    __syncthreads();
    return r;
}

// Route plan of one chunk (recipe-lna/lna2/lna_moe_ticket.cu:147-214 builds
// the same kind of plan per CTA for decode; recipe-lna/vllm_exl3_exl3.py.lna:1617-1629
// is the argsort / count glue it replaces).  Pairs are ordered by expert,
// then token, so results do not depend on timing; an expert listed twice in
// one token's slots is one pair used by both slots.
__global__ void __launch_bounds__(1024) pf_plan_kernel(RouteIn route, int64_t slot0, int T, int topk, int E, int H,
                                                       int I, uint32_t* ctrl, PfPlan plan) {
    extern __shared__ uint32_t pf_mask[];   // [E][W]
    __shared__ int warp_tot[32];
    __shared__ int totals[4];
    __shared__ int s_pair[kPfMaxExperts + 1], s_pass[kPfMaxExperts + 1];
    pdl_launch_dependents();
    const int tid = threadIdx.x;
    const int W = (T + 31) >> 5;
    for (int i = tid; i < E * W; i += 1024) pf_mask[i] = 0u;
    __syncthreads();
    for (int q = tid; q < T * topk; q += 1024) {
        const int e = route_local_id(route, slot0 + q, E), t = q / topk;
        if (e >= 0) atomicOr(&pf_mask[e * W + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    // per expert: pairs, passes, units; E <= 1024 = one expert per thread
    int c = 0;
    if (tid < E)
        for (int w = 0; w < W; ++w) c += __popc(pf_mask[tid * W + w]);
    const int passes = (c + kPfRows - 1) / kPfRows;
    const int o_pair = block_scan_1024(c, warp_tot, &totals[0]);
    const int o_pass = block_scan_1024(passes, warp_tot, &totals[1]);
    const int o_gu = block_scan_1024(passes * (I / 128), warp_tot, &totals[2]);
    const int o_dn = block_scan_1024(passes * (H / 128), warp_tot, &totals[3]);
    if (tid < E) {
        plan.e_off[tid] = o_pair;
        plan.pass_off[tid] = o_pass;
        plan.gu_off[tid] = o_gu;
        plan.dn_off[tid] = o_dn;
        s_pair[tid] = o_pair;
        s_pass[tid] = o_pass;
    }
    if (tid == 0) {
        plan.e_off[E] = totals[0];
        plan.pass_off[E] = totals[1];
        plan.gu_off[E] = totals[2];
        plan.dn_off[E] = totals[3];
        s_pair[E] = totals[0];
        s_pass[E] = totals[1];
    }
    __syncthreads();
    // unit table: gate/up units (expert, strip, pass), then down units; one
    // expert per thread, so each thread still holds its own unit offsets
    if (totals[2] + totals[3] <= plan.unit_cap) {
        for (int e = tid; e < E; e += 1024) {
            const int pe = s_pair[e], ce = s_pair[e + 1] - pe;
            const int pass0 = s_pass[e], np = s_pass[e + 1] - pass0;
            for (int ph = 0; ph < 2; ++ph) {
                const int strips = ph == 0 ? I / 128 : H / 128;
                int4* dst = plan.units + (ph == 0 ? o_gu : totals[2] + o_dn);
                for (int st = 0; st < strips; ++st)
                    for (int ps = 0; ps < np; ++ps) {
                        const int rows = min(kPfRows, ce - ps * kPfRows);
                        dst[st * np + ps] = make_int4(e, st, pe + ps * kPfRows, rows | ((pass0 + ps) << 8));
                    }
            }
        }
    }
    // pairs: one (expert, token word) item per thread
    for (int it = tid; it < E * W; it += 1024) {
        const int e = it / W, w = it % W;
        uint32_t m = pf_mask[it];
        if (!m) continue;
        int base = s_pair[e];
        for (int w2 = 0; w2 < w; ++w2) base += __popc(pf_mask[e * W + w2]);
        while (m) {
            const int b = __ffs(m) - 1;
            m &= m - 1;
            plan.pair_tok[base] = w * 32 + b;
            plan.pair_exp[base] = e;
            ++base;
        }
    }
    // slot -> pair
    for (int q = tid; q < T * topk; q += 1024) {
        const int e = route_local_id(route, slot0 + q, E), t = q / topk;
        int pr = -1;
        if (e >= 0) {
            const int w = t >> 5;
            pr = s_pair[e] + __popc(pf_mask[e * W + w] & ((1u << (t & 31)) - 1u));
            for (int w2 = 0; w2 < w; ++w2) pr += __popc(pf_mask[e * W + w2]);
        }
        plan.slot_pair[q] = pr;
    }
    // the GEMM's ticket and per-pass counters start at zero
    const int npass = totals[1] < kPfMaxPasses ? totals[1] : kPfMaxPasses;
    for (int i = tid; i < npass; i += 1024) ctrl[kPfCtrlWords + i] = 0u;
    if (tid == 0) {
        ctrl[0] = 0u;
        ctrl[4] = (uint32_t) totals[2];
        ctrl[5] = (uint32_t) totals[3];
        ctrl[6] = (uint32_t) totals[0];
        if (totals[1] > kPfMaxPasses || totals[2] + totals[3] > plan.unit_cap) {
            // more passes than counters: run no units (reported as a plan overflow)
            ctrl[4] = 0u;
            ctrl[5] = 0u;
            atomicOr(&ctrl[2], ERR_PLAN);
        }
    }
}

// ------------------------------------------------------------------ 2. input
// Four consecutive activations of x (fp16 or bf16) as fp16, one 8-byte load.
__device__ __forceinline__ void load4_act(const void* x, int dtype, int64_t i, __half (&h)[4]) {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(x) + i * 2);
    if (dtype == 0) {
        *reinterpret_cast<uint2*>(h) = v;
    } else {
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) h[q] = __float2half_rn(__bfloat162float(b[q]));
    }
}

// fp16 activations -> one transformed 128-block: fp16(x) * suh (fp16),
// Hadamard in fp32, / sqrt(128), -> fp16, stored as 4 halves per lane.
__device__ __forceinline__ void pf_transform_store(const __half (&xh)[4], const __half* suh, int64_t k0, __half* dst,
                                                   int lane) {
    __half sh[4];
    if ((reinterpret_cast<uintptr_t>(suh) & 7u) == 0) {
        *reinterpret_cast<uint2*>(sh) = *reinterpret_cast<const uint2*>(suh + k0);
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) sh[q] = suh[k0 + q];
    }
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = __half2float(__hmul(xh[q], sh[q]));
    wht128_warp(v, lane);
    __half2 h0 = __floats2half2_rn(v[0] * kHadNorm, v[1] * kHadNorm);
    __half2 h1 = __floats2half2_rn(v[2] * kHadNorm, v[3] * kHadNorm);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(dst + k0) = o;
}

// One CTA per pair (grid-stride); warp w transforms the 128-blocks w, w + 8,
// ... of the pair's token row for gate and up
// (recipe-lna/lna2/lna_moe_ticket.cu:119-144).
__global__ void __launch_bounds__(256) pf_input_kernel(const void* x, int x_dtype, int H, const uint32_t* ctrl,
                                                       const int* pair_tok, const int* pair_exp,
                                                       const int64_t* gsuh_tab, const int64_t* usuh_tab,
                                                       __half* xg, __half* xu) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int npairs = (int) __ldcg(ctrl + 6);
    for (int pr = blockIdx.x; pr < npairs; pr += gridDim.x) {
        const int t = pair_tok[pr], e = pair_exp[pr];
        const __half* gs = reinterpret_cast<const __half*>(gsuh_tab[e]);
        const __half* us = reinterpret_cast<const __half*>(usuh_tab[e]);
        for (int kb = warp; kb < H / 128; kb += 8) {
            const int64_t k0 = (int64_t) kb * 128 + lane * 4;
            __half xh[4];
            load4_act(x, x_dtype, (int64_t) t * H + k0, xh);
            pf_transform_store(xh, gs, k0, xg + (int64_t) pr * H, lane);
            pf_transform_store(xh, us, k0, xu + (int64_t) pr * H, lane);
        }
    }
}

// ------------------------------------------------------------------ 3. GEMM
// Decoders: one unit's k-steps at bit width K.  Warp w decodes, per step,
// gate/up (MODE 0): matrix w / 8, n-tile w % 8, k-slices 0..3; down (MODE 1):
// n-tile w % 8, k-slices 2 (w / 8) .. +1.  Each 16x16 tile leaves the
// registers in the m16n8k16 fragment layout it was decoded in, as one
// stmatrix.x4 into the K-major 128-byte-swizzled A tile (lane l gives the
// address of row (l % 8) + 8 (l / 16), 8-element chunk (l / 8) % 2).
template <int K, int CB, int MODE>
__device__ bool pf_decode_unit(PfHead& H, uint8_t* Abuf, const uint8_t* Wring, int ksteps, uint32_t& gs,
                               const ShiftTable& st, int warp, int lane, uint32_t* status PFC_PARAM) {
    using F = TileFmt<K>;
    constexpr int NI = MODE == 0 ? 4 : 2;
    const LaneGeom<K> geom = lane_geom<K>(lane);
    const int ntile = warp & 7;
    const int m = MODE == 0 ? (warp >> 3) : 0;
    const int i0 = MODE == 0 ? 0 : (warp >> 3) * 2;
    const int row = ntile * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
    uint32_t off[NI];
#pragma unroll
    for (int ii = 0; ii < NI; ++ii) {
        const int chunk = (i0 + ii) * 2 + ((lane >> 3) & 1);
        off[ii] = (uint32_t) (m * (128 * 128) + row * 128 + ((chunk ^ (row & 7)) << 4));
    }
    const uint32_t abase = smem_u32(Abuf);
    // ring positions as running counters (one division per unit, not per step)
    int ws = (int) (gs % kPfWStages), as = (int) (gs % kPfAStages);
    uint32_t wph = (gs / kPfWStages) & 1u, aph = (gs / kPfAStages) & 1u;
    for (int s = 0; s < ksteps; ++s, ++gs) {
        PFC_RESET();
        if (!mbar_wait_lanes(&H.wfull[ws], wph, status)) return false;
        PFC_MARK(PF_DEC_W);
        if (!mbar_wait_lanes(&H.sfree[as], aph ^ 1u, status)) return false;
        PFC_MARK(PF_DEC_AFREE);
        const uint32_t* wst = reinterpret_cast<const uint32_t*>(Wring + ws * kPfWStage);
        const uint32_t a = abase + (uint32_t) (as * kPfAStage);
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) {
            const uint32_t* t = wst + ((m * 4 + i0 + ii) * 8 + ntile) * F::WORDS;
            uint32_t whi[F::NG], wlo[F::NG], w[8], xv[8];
#pragma unroll
            for (int h = 0; h < F::NG; ++h) {
                whi[h] = t[geom.ihi[h]];
                wlo[h] = t[geom.ilo[h]];
            }
            tile_windows_f<K>(whi, wlo, geom, st, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) xv[j] = codebook_pair<CB>(w[j]);
            stmatrix_x4(a + off[ii], round_pair(xv[0], xv[1]), round_pair(xv[2], xv[3]), round_pair(xv[4], xv[5]),
                        round_pair(xv[6], xv[7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&H.aready[as]);
            mbar_arrive(&H.wempty[ws]);
        }
        if (++ws == kPfWStages) { ws = 0; wph ^= 1u; }
        if (++as == kPfAStages) { as = 0; aph ^= 1u; }
    }
    return true;
}

template <int CB, int MODE>
__device__ bool pf_decode_k(PfHead& H, uint8_t* Abuf, const uint8_t* Wring, const PfUnit& u, uint32_t& gs,
                            const ShiftTable& st, int warp, int lane, uint32_t* status PFC_PARAM) {
    switch (u.K) {
        case 1: return pf_decode_unit<1, CB, MODE>(H, Abuf, Wring, u.ksteps, gs, st, warp, lane, status PFC_FWD);
        case 2: return pf_decode_unit<2, CB, MODE>(H, Abuf, Wring, u.ksteps, gs, st, warp, lane, status PFC_FWD);
        case 3: return pf_decode_unit<3, CB, MODE>(H, Abuf, Wring, u.ksteps, gs, st, warp, lane, status PFC_FWD);
        default: return pf_decode_unit<4, CB, MODE>(H, Abuf, Wring, u.ksteps, gs, st, warp, lane, status PFC_FWD);
    }
}

template <int CB>
__device__ bool pf_decode_dispatch(PfHead& H, uint8_t* Abuf, const uint8_t* Wring, const PfUnit& u, uint32_t& gs,
                                   const ShiftTable& st, int warp, int lane, uint32_t* status PFC_PARAM) {
    return u.mode == 0 ? pf_decode_k<CB, 0>(H, Abuf, Wring, u, gs, st, warp, lane, status PFC_FWD)
                       : pf_decode_k<CB, 1>(H, Abuf, Wring, u, gs, st, warp, lane, status PFC_FWD);
}

// Unit of ticket `tk` (mode -1 once the tickets run out); ngu / ndn are
// the gate/up and down unit counts.
__device__ PfUnit pf_unit_of(const PfParams& p, int tk, int ngu, int ndn) {
    PfUnit u{};
    if (tk >= ngu + ndn) { u.mode = -1; return u; }
    const int4 r = __ldcg(p.plan.units + tk);
    u.mode = tk < ngu ? 0 : 1;
    u.e = r.x;
    u.strip = r.y;
    u.row0 = r.z;
    u.rows = r.w & 255;
    u.gp = r.w >> 8;
    u.K = p.ktab ? p.ktab[u.e] : p.Kscalar;
    u.ksteps = (u.mode == 0 ? p.H : p.I) / kPfKStep;
    return u;
}

template <int CB>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ PfParams p) {
    extern __shared__ uint8_t pf_raw[];
    uint8_t* base = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);
    uint8_t* Xbuf = base;
    uint8_t* Abuf = Xbuf + kPfXStages * kPfXStage;
    uint8_t* Wring = Abuf + kPfAStages * kPfAStage;
    float* Stg = reinterpret_cast<float*>(Wring + kPfWStages * kPfWStage);    // [2][32][128] fp32
    PfHead& H = *reinterpret_cast<PfHead*>(reinterpret_cast<uint8_t*>(Stg) + kPfStageBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* status = p.ctrl + 2;

    if (tid == 0) {
        for (int s = 0; s < kPfWStages; ++s) { mbar_init(&H.wfull[s], 1); mbar_init(&H.wempty[s], kPfDecWarps); }
        for (int s = 0; s < kPfAStages; ++s) {
            mbar_init(&H.aready[s], kPfDecWarps);
            mbar_init(&H.xfull[s], 1);
            mbar_init(&H.sfree[s], 1);
        }
        for (int s = 0; s < 2; ++s) { mbar_init(&H.accfull[s], 1); mbar_init(&H.accfree[s], kPfEpiWarps); }
        for (int s = 0; s < kPfDQ; ++s) {
            mbar_init(&H.dfull[s], 1);
            mbar_init(&H.dempty[s], kPfDecWarps + 1 + kPfEpiWarps + 1);
        }
        fence_barrier_init();
    }
    if (warp == kPfMmaWarp) tmem_alloc(&H.tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = H.tmem;

    if (warp == kPfProducerWarp) {
        // ------------------------------------------------------------ producer
        // Lane 0 claims tickets and issues the copies; the whole warp points
        // the unit's weight tensor maps at the expert (tensormap.replace in
        // shared memory, release to this CTA's global slot, acquire).  A slot
        // is reused kPfMapSlots units later, after more weight stages than
        // the ring holds have been issued, so no copy still reads it.
        pdl_wait();
        uint32_t gs = 0, issued_w = 0;
        bool ok = true;
        const int ngu = (int) __ldcg(p.ctrl + 4), ndn = (int) __ldcg(p.ctrl + 5);
        // the next ticket is claimed one unit ahead, so its latency overlaps
        // the current unit's copies (tickets still rise per CTA, so a down
        // unit never waits on a unit this CTA holds back)
        int tk_next = 0;
        if (lane == 0) tk_next = (int) atomicAdd(p.ctrl, 1u);
        PFC_DECL
        for (uint32_t n = 0; ok; ++n) {
            const int tk = __shfl_sync(0xffffffffu, tk_next, 0);
            PFC_RESET();
            PfUnit u = pf_unit_of(p, tk, ngu, ndn);
            if (u.mode >= 0 && lane == 0) tk_next = (int) atomicAdd(p.ctrl, 1u);
            if (u.mode >= 0 && (u.K < 1 || u.K > kPfKmax)) {
                if (lane == 0) set_error(status, ERR_BAD_K);
                u.mode = -1;
            }
            PFC_MARK(PF_PR_TICKET);
            const int d = n % kPfDQ;
            if (lane == 0) {
                ok = mbar_wait(&H.dempty[d], ((n / kPfDQ) + 1u) & 1u, status);
                if (ok) {
                    H.desc[d] = u;
                    mbar_arrive(&H.dfull[d]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            PFC_MARK(PF_PR_DEMPTY);
            if (!ok || u.mode < 0) break;
            const int nm = u.mode == 0 ? 2 : 1;
            // weight tensor maps of the unit's matrices
            const CUtensorMap* wmap[2] = {nullptr, nullptr};
            bool valid = true;
            for (int m = 0; m < nm; ++m) {
                const void* wp = reinterpret_cast<const void*>(p.tab[u.mode == 0 ? m * 3 : 6][u.e]);
                if (!aligned16_dev(wp) || wp == nullptr) { valid = false; continue; }
                CUtensorMap* gtm = p.maps + ((size_t) blockIdx.x * kPfMapSlots + n % kPfMapSlots) * 2 + m;
                const uint4* tsrc = reinterpret_cast<const uint4*>(&p.tmpl[u.mode * 4 + u.K - 1]);
                if (lane < 8) reinterpret_cast<uint4*>(&H.tmap[m])[lane] = tsrc[lane];
                __syncwarp();
                if (lane == 0) tmap_replace_address(&H.tmap[m], wp);
                __syncwarp();
                tmap_publish(gtm, &H.tmap[m]);
                if (lane == 0) tmap_acquire(gtm);
                wmap[m] = gtm;
            }
            if (!valid && lane == 0) set_error(status, ERR_MISALIGNED);
            if (lane == 0) {
                // weights do not depend on earlier units: down units' weights
                // stream while their input is still being written
                const uint32_t wbytes = (uint32_t) (nm * 4 * 8 * 32 * u.K);
                for (int s = 0; s < u.ksteps && ok; ++s, ++gs) {
                    const int ws = gs % kPfWStages;
                    PFC_RESET();
                    ok = mbar_wait(&H.wempty[ws], ((gs / kPfWStages) + 1u) & 1u, status);
                    PFC_MARK(PF_PR_WEMPTY);
                    if (!ok) break;
                    if (valid) {
                        mbar_arrive_expect_tx(&H.wfull[ws], wbytes);
                        for (int m = 0; m < nm; ++m)
                            tma_load_3d(Wring + ws * kPfWStage + m * (4 * 8 * 32 * u.K), wmap[m], 0, u.strip * 8,
                                        s * 4, &H.wfull[ws]);
                    } else {
                        mbar_arrive(&H.wfull[ws]);        // garbage weights; the error bit is set
                    }
                    issued_w = gs + 1;
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
        if (lane == 0) {
            PFC_FLUSH(PF_PR_TOTAL, 0);
            // no copy may still be in flight when the CTA retires
            for (uint32_t i = issued_w > kPfWStages ? issued_w - kPfWStages : 0; i < issued_w; ++i)
                if (!mbar_wait(&H.wfull[i % kPfWStages], (i / kPfWStages) & 1u, status)) break;
        }
    } else if (warp == kPfXWarp) {
        // ------------------------------------------------------------ activation producer
        // Follows the unit descriptors; a down unit first waits (bounded) until
        // every 128-column strip of its pass's down input is written.
        pdl_wait();
        if (lane == 0) {
            uint32_t gs = 0, issued_x = 0;
            bool ok = true;
            PFC_DECL
            for (uint32_t n = 0; ok; ++n) {
                const int d = n % kPfDQ;
                if (!mbar_wait(&H.dfull[d], (n / kPfDQ) & 1u, status)) break;
                const PfUnit u = H.desc[d];
                mbar_arrive(&H.dempty[d]);
                if (u.mode < 0) break;
                PFC_RESET();
                if (u.mode == 1) {
                    ok = wait_counter(p.ctrl + kPfCtrlWords + u.gp, (uint32_t) (p.I / 128), status);
                    fence_proxy_async_global();
                    if (!ok) break;
                }
                PFC_MARK(PF_PR_DEP);
                const int nm = u.mode == 0 ? 2 : 1;
                const CUtensorMap* xmap[2] = {u.mode == 0 ? &p.xg_map : &p.xd_map, &p.xu_map};
                const int nbox = (u.rows + kPfBoxRows - 1) / kPfBoxRows;
                for (int s = 0; s < u.ksteps && ok; ++s, ++gs) {
                    const int xs = gs % kPfXStages;
                    PFC_RESET();
                    ok = mbar_wait(&H.sfree[xs], ((gs / kPfXStages) + 1u) & 1u, status);
                    PFC_MARK(PF_PR_XFREE);
                    if (!ok) break;
                    mbar_arrive_expect_tx(&H.xfull[xs], (uint32_t) (nm * nbox * kPfBoxBytes));
                    for (int m = 0; m < nm; ++m)
                        for (int b = 0; b < nbox; ++b)
                            tma_load_2d(Xbuf + xs * kPfXStage + m * kPfXBox + b * kPfBoxBytes, xmap[m], s * kPfKStep,
                                        u.row0 + b * kPfBoxRows, &H.xfull[xs]);
                    issued_x = gs + 1;
                }
            }
            PFC_FLUSH(PF_XP_TOTAL, 0);
            for (uint32_t i = issued_x > kPfXStages ? issued_x - kPfXStages : 0; i < issued_x; ++i)
                if (!mbar_wait(&H.xfull[i % kPfXStages], (i / kPfXStages) & 1u, status)) break;
        }
    } else if (warp == kPfMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t gs = 0;
            bool ok = true;
            const uint64_t adesc0 = sdesc_sw128(smem_u32(Abuf)), xdesc0 = sdesc_sw128(smem_u32(Xbuf));
            PFC_DECL
            for (uint32_t n = 0; ok; ++n) {
                const int d = n % kPfDQ;
                PFC_RESET();
                if (!mbar_wait(&H.dfull[d], (n / kPfDQ) & 1u, status)) break;
                PFC_MARK(PF_MMA_DESC);
                const PfUnit u = H.desc[d];
                mbar_arrive(&H.dempty[d]);
                if (u.mode < 0) break;
                PFC_COUNT(PF_UNITS);
                const int a = n & 1;
                ok = mbar_wait(&H.accfree[a], ((n >> 1) + 1u) & 1u, status);
                PFC_MARK(PF_MMA_ACCFREE);
                if (!ok) break;
                tc_fence_after();
                const uint32_t idesc = idesc_f16(128, (u.rows + 15) & ~15);
                const uint32_t acc0 = tmem + (uint32_t) (a * 256);
                for (int s = 0; s < u.ksteps; ++s, ++gs) {
                    const int as = gs % kPfAStages, xs = gs % kPfXStages;
                    PFC_RESET();
                    ok = mbar_wait(&H.xfull[xs], (gs / kPfXStages) & 1u, status);
                    PFC_MARK(PF_MMA_X);
                    ok = ok && mbar_wait(&H.aready[as], (gs / kPfAStages) & 1u, status);
                    PFC_MARK(PF_MMA_A);
                    if (!ok) break;
                    tc_fence_after();
                    // descriptors advance in 16-byte units: +2 per 16-element k step
                    const uint64_t ad = adesc0 + (uint64_t) (as * (kPfAStage >> 4));
                    const uint64_t xd = xdesc0 + (uint64_t) (xs * (kPfXStage >> 4));
                    const uint32_t en = s != 0;
                    if (u.mode == 0) {
#pragma unroll
                        for (int kk = 0; kk < kPfKStep / 16; ++kk) {
                            tc_mma(acc0, ad + 2 * kk, xd + 2 * kk, idesc, en | kk);
                            tc_mma(acc0 + 128, ad + (128 * 128 >> 4) + 2 * kk, xd + (kPfXBox >> 4) + 2 * kk, idesc,
                                   en | kk);
                        }
                    } else {
#pragma unroll
                        for (int kk = 0; kk < kPfKStep / 16; ++kk) tc_mma(acc0, ad + 2 * kk, xd + 2 * kk, idesc, en | kk);
                    }
                    tc_commit(&H.sfree[as]);
                }
                tc_commit(&H.accfull[a]);
            }
            PFC_FLUSH(PF_MMA_TOTAL, 0);
        }
    } else if (warp < kPfDecWarps) {
        // ------------------------------------------------------------ decoders
        uint32_t gs = 0;
        PFC_DECL
        for (uint32_t n = 0;; ++n) {
            const int d = n % kPfDQ;
            PFC_RESET();
            if (!mbar_wait_lanes(&H.dfull[d], (n / kPfDQ) & 1u, status)) break;
            PFC_MARK(PF_DEC_DESC);
            const PfUnit u = H.desc[d];
            __syncwarp();
            if (lane == 0) mbar_arrive(&H.dempty[d]);
            if (u.mode < 0) break;
            if (!pf_decode_dispatch<CB>(H, Abuf, Wring, u, gs, p.st, warp, lane, status PFC_FWD)) break;
        }
        PFC_FLUSH(PF_DEC_TOTAL, lane);
    } else {
        // ------------------------------------------------------------ epilogue
        const int lg = warp & 3;               // TMEM lane group of this warp
        const int ew = warp - kPfEpiWarp0;     // 0..3
        float* SG = Stg;
        float* SU = Stg + kPfChunkRows * 128;
        PFC_DECL
        for (uint32_t n = 0;; ++n) {
            const int d = n % kPfDQ;
            PFC_RESET();
            mbar_wait_lanes(&H.dfull[d], (n / kPfDQ) & 1u, status);
            PFC_MARK(PF_EP_DESC);
            // the four warps take one verdict: a completed phase stays complete
            // until these warps have released the slot
            named_bar(1, kPfEpiWarps * 32);
            if (!__all_sync(0xffffffffu, mbar_try_wait(&H.dfull[d], (n / kPfDQ) & 1u))) break;
            const PfUnit u = H.desc[d];
            __syncwarp();
            if (lane == 0) mbar_arrive(&H.dempty[d]);
            if (u.mode < 0) break;
            const int a = n & 1;
            PFC_RESET();
            const bool ok = mbar_wait_lanes(&H.accfull[a], (n >> 1) & 1u, status);
            PFC_MARK(PF_EP_ACC);
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t) (lg * 32) << 16) + (uint32_t) (a * 256);
            const int col = lg * 32 + lane;
            const int e = u.e;
            for (int c0 = 0; c0 < u.rows; c0 += kPfChunkRows) {
                {
                    float v[32];
                    tc_ld32(tbase + (uint32_t) c0, v);
#pragma unroll
                    for (int r = 0; r < 32; ++r) SG[r * 128 + col] = v[r];
                    if (u.mode == 0) {
                        tc_ld32(tbase + 128u + (uint32_t) c0, v);
#pragma unroll
                        for (int r = 0; r < 32; ++r) SU[r * 128 + col] = v[r];
                    }
                }
                named_bar(1, kPfEpiWarps * 32);
                for (int r = ew * 8; r < ew * 8 + 8; ++r) {
                    const int row = c0 + r;
                    if (row >= u.rows || !ok) break;
                    const int64_t pr = u.row0 + row;
                    float gv[4];
                    *reinterpret_cast<float4*>(gv) = *reinterpret_cast<const float4*>(SG + r * 128 + lane * 4);
                    if (u.mode == 0) {
                        float uv[4];
                        *reinterpret_cast<float4*>(uv) = *reinterpret_cast<const float4*>(SU + r * 128 + lane * 4);
                        const __half* gsv = reinterpret_cast<const __half*>(p.tab[2][e]) + u.strip * 128;
                        const __half* usv = reinterpret_cast<const __half*>(p.tab[5][e]) + u.strip * 128;
                        const __half* dsu = reinterpret_cast<const __half*>(p.tab[7][e]) + u.strip * 128;
                        out_transform(gv, gsv, lane);
                        out_transform(uv, usv, lane);
                        float dv[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            float gg = gv[q], uu = uv[q];
                            if (gg > p.limit) gg = p.limit;
                            if (uu < -p.limit) uu = -p.limit;
                            if (uu > p.limit) uu = p.limit;
                            const __half ah = __float2half_rn((gg / (1.0f + __expf(-gg))) * uu);
                            dv[q] = __half2float(__hmul(ah, dsu[lane * 4 + q]));
                        }
                        wht128_warp(dv, lane);
                        __half2 h0 = __floats2half2_rn(dv[0] * kHadNorm, dv[1] * kHadNorm);
                        __half2 h1 = __floats2half2_rn(dv[2] * kHadNorm, dv[3] * kHadNorm);
                        uint2 o;
                        o.x = *reinterpret_cast<uint32_t*>(&h0);
                        o.y = *reinterpret_cast<uint32_t*>(&h1);
                        *reinterpret_cast<uint2*>(p.xd + pr * p.I + u.strip * 128 + lane * 4) = o;
                    } else {
                        const __half* dsv = reinterpret_cast<const __half*>(p.tab[8][e]) + u.strip * 128;
                        out_transform(gv, dsv, lane);
                        __stcg(reinterpret_cast<float4*>(p.dn + pr * p.H + u.strip * 128 + lane * 4),
                               make_float4(gv[0], gv[1], gv[2], gv[3]));
                    }
                }
                named_bar(1, kPfEpiWarps * 32);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&H.accfree[a]);
            if (u.mode == 0) {
                // release this strip of the pass's down input to the down units
                fence_proxy_async_global();
                __threadfence();
                named_bar(1, kPfEpiWarps * 32);
                if (ew == 0 && lane == 0) atom_add_release_gpu(p.ctrl + kPfCtrlWords + u.gp, 1u);
            }
        }
        if (ew == 0) PFC_FLUSH(PF_EP_TOTAL, lane);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kPfMmaWarp) {
        tc_fence_after();
        tmem_free(tmem, 512);
    }
}

// ------------------------------------------------------------------ 4. gather
// out[t][c] = sum over slots j, in slot order, of weights[t][j] * dn[pair][c]
// (recipe-lna/lna2/lna_moe_ticket.cu:409-428), fp32, one cast.
__global__ void __launch_bounds__(256) pf_gather_kernel(const float* dn, const int* slot_pair, RouteIn route,
                                                        int64_t slot0, int T, int topk, int H, void* out,
                                                        int out_dtype) {
    pdl_wait();
    const int64_t n4 = (int64_t) T * (H / 4);
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t) gridDim.x * blockDim.x) {
        const int t = (int) (i / (H / 4));
        const int c = (int) (i % (H / 4)) * 4;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < topk; ++j) {
            const int pr = slot_pair[t * topk + j];
            if (pr < 0) continue;
            const float w = route_weight(route, slot0 + t * topk + j);
            const float4 d = __ldcg(reinterpret_cast<const float4*>(dn + (int64_t) pr * H + c));
            v[0] += w * d.x; v[1] += w * d.y; v[2] += w * d.z; v[3] += w * d.w;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) store_out(out, out_dtype, (int64_t) t * H + c + q, v[q]);
    }
}

// ------------------------------------------------------------------ host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 pf_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// Weight tensor-map templates for (hidden, inter): [gate/up, down][K - 1],
// dims [16K, n/16, k/16] u16, box [16K, 8, 4] (4 k-slices of 8 tiles), with
// a placeholder address every unit replaces.  Cached per shape.
struct PfTemplates {
    CUtensorMap t[8];
};

int pf_templates(int64_t H, int64_t I, void* placeholder, PfTemplates* out) {
    static std::mutex mu;
    static std::map<std::pair<int64_t, int64_t>, PfTemplates> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({H, I});
    if (it != cache.end()) {
        *out = it->second;
        return EXL3_OK;
    }
    auto encode = pf_encoder();
    EXL3_REQUIRE(encode != nullptr, EXL3_ERR_CUDA, "exl3_moe_prefill: cuTensorMapEncodeTiled is not available");
    PfTemplates T{};
    for (int kind = 0; kind < 2; ++kind)
        for (int K = 1; K <= kPfKmax; ++K) {
            const int64_t k = kind == 0 ? H : I, n = kind == 0 ? I : H;
            const cuuint64_t dims[3] = {(cuuint64_t) (16 * K), (cuuint64_t) (n / 16), (cuuint64_t) (k / 16)};
            const cuuint64_t strides[2] = {(cuuint64_t) (32 * K), (cuuint64_t) (n / 16) * (cuuint64_t) (32 * K)};
            const cuuint32_t box[3] = {(cuuint32_t) (16 * K), 8u, 4u};
            const cuuint32_t estr[3] = {1u, 1u, 1u};
            const CUresult r = encode(&T.t[kind * 4 + K - 1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, placeholder, dims,
                                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_moe_prefill: weight tensor map failed (%d)", (int) r);
        }
    cache[{H, I}] = T;
    *out = T;
    return EXL3_OK;
}

template <typename... Args>
cudaError_t pf_launch(void (*kern)(Args...), dim3 grid, dim3 block, int smem, cudaStream_t s, bool pdl,
                      const std::decay_t<Args>&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = (size_t) smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Tokens per plan: at most 2048, and the bitmasks must fit shared memory.
int64_t pf_chunk_tokens(int64_t E) {
    int64_t t = (int64_t) kPfMaskWords / E * 32;
    if (t > kPfMaxTokens) t = kPfMaxTokens;
    return t;
}

struct PfGeom {
    int64_t cap;                  // pair capacity of one chunk = chunk tokens x topk
    int64_t unit_cap;             // work units of one chunk, upper bound
    int64_t off_plan, off_units, off_maps, off_xg, off_xu, off_xd, off_dn, total;
};

PfGeom pf_geom(int64_t m, int64_t topk, int64_t H, int64_t I, int64_t E) {
    PfGeom g{};
    int64_t ct = pf_chunk_tokens(E);
    if (m < ct) ct = m;
    g.cap = ct * topk;
    // passes: one per expert with rows plus one per 128 rows
    const int64_t passes = (E < g.cap ? E : g.cap) + g.cap / kPfRows + 1;
    g.unit_cap = passes * (H / 128 + I / 128);
    int64_t o = kPfCtrlBytes;
    g.off_plan = o;
    o += align_up((4 * (E + 1) + 2 * g.cap + g.cap) * 4, 256);
    g.off_units = o;
    o += align_up(g.unit_cap * 16, 256);
    g.off_maps = o;
    o += (int64_t) kPfMaxGrid * kPfMapSlots * 2 * 128;
    g.off_xg = o;
    o += align_up(g.cap * H * 2, 256);
    g.off_xu = o;
    o += align_up(g.cap * H * 2, 256);
    g.off_xd = o;
    o += align_up(g.cap * I * 2, 256);
    g.off_dn = o;
    o += align_up(g.cap * H * 4, 256);
    g.total = o;
    return g;
}

template <int CB>
int pf_set_attr() {
    static std::once_flag once[64];
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    cudaError_t attr = cudaSuccess;
    std::call_once(once[dev & 63], [&] {
        attr = cudaFuncSetAttribute(pf_gemm_kernel<CB>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
        if (attr == cudaSuccess)
            attr = cudaFuncSetAttribute(pf_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfMaskWords * 4);
    });
    EXL3_CUDA(attr);
    return EXL3_OK;
}

}  // namespace

#ifdef EXL3_PHASE_CLOCK
extern "C" int exl3_pf_phase_read(unsigned long long* out, int n, int reset) {
    EXL3_REQUIRE(out && n >= 1 && n <= PF_N, EXL3_ERR_ARG, "phase clock: bad output");
    EXL3_CUDA(cudaDeviceSynchronize());
    EXL3_CUDA(cudaMemcpyFromSymbol(out, g_pf_phase, sizeof(unsigned long long) * n));
    if (reset) {
        static const unsigned long long zero[PF_N] = {};
        EXL3_CUDA(cudaMemcpyToSymbol(g_pf_phase, zero, sizeof(zero)));
    }
    return EXL3_OK;
}
#endif

extern "C" int64_t exl3_moe_prefill_scratch_bytes(int64_t m, int64_t topk, int64_t hidden, int64_t inter,
                                                  int64_t n_experts) {
    if (m < 1 || topk < 1 || topk > kPfMaxTopk || hidden < 128 || inter < 128 || n_experts < 1 ||
        n_experts > kPfMaxExperts)
        return -1;
    return pf_geom(m, topk, hidden, inter, n_experts).total;
}

extern "C" int64_t exl3_moe_prefill_chunk_tokens(int64_t n_experts) {
    if (n_experts < 1 || n_experts > kPfMaxExperts) return -1;
    return pf_chunk_tokens(n_experts);
}

int route_from_abi(const exl3_moe_route* r, RouteIn* out);   // moe.cu

static int moe_prefill_impl(const void* x, int x_dtype, void* out, int out_dtype, int64_t m, int64_t hidden,
                            int64_t inter, const int64_t* gate_trellis, const int64_t* gate_suh,
                            const int64_t* gate_svh, const int64_t* up_trellis, const int64_t* up_suh,
                            const int64_t* up_svh, const int64_t* down_trellis, const int64_t* down_suh,
                            const int64_t* down_svh, int64_t n_experts, const int32_t* k_table, int K, int kmax,
                            int cb, const RouteIn& route, int64_t topk, float swiglu_limit, void* scratch,
                            int64_t scratch_bytes, void* stream) {
    EXL3_REQUIRE(x && out && route.ids && route.weights && scratch, EXL3_ERR_ARG,
                 "exl3_moe_prefill: null pointer argument");
    EXL3_REQUIRE(gate_trellis && gate_suh && gate_svh && up_trellis && up_suh && up_svh && down_trellis &&
                     down_suh && down_svh,
                 EXL3_ERR_ARG, "exl3_moe_prefill: null pointer table");
    EXL3_REQUIRE(m >= 1, EXL3_ERR_ARG, "exl3_moe_prefill: m must be >= 1");
    EXL3_REQUIRE(hidden % 128 == 0 && inter % 128 == 0 && hidden > 0 && inter > 0, EXL3_ERR_ARG,
                 "exl3_moe_prefill: hidden and inter must be positive multiples of 128");
    EXL3_REQUIRE(n_experts >= 1 && n_experts <= kPfMaxExperts, EXL3_ERR_ARG,
                 "exl3_moe_prefill: n_experts must be in 1..%d", kPfMaxExperts);
    EXL3_REQUIRE(topk >= 1 && topk <= kPfMaxTopk, EXL3_ERR_ARG, "exl3_moe_prefill: topk must be in 1..%d",
                 kPfMaxTopk);
    EXL3_REQUIRE(kmax >= 1 && kmax <= kPfKmax, EXL3_ERR_ARG, "exl3_moe_prefill: kmax must be in 1..%d", kPfKmax);
    EXL3_REQUIRE(k_table || (K >= 1 && K <= kmax), EXL3_ERR_ARG, "exl3_moe_prefill: K must be in 1..kmax");
    EXL3_REQUIRE(cb >= 0 && cb <= 2, EXL3_ERR_ARG, "exl3_moe_prefill: codebook must be 0, 1 or 2");
    EXL3_REQUIRE(x_dtype >= 0 && x_dtype <= 1 && out_dtype >= 0 && out_dtype <= 2, EXL3_ERR_ARG,
                 "exl3_moe_prefill: x must be fp16/bf16, out fp16/bf16/fp32");
    EXL3_REQUIRE(swiglu_limit > 0.f, EXL3_ERR_ARG, "exl3_moe_prefill: swiglu_limit must be > 0");
    EXL3_REQUIRE(aligned16(scratch), EXL3_ERR_ARG, "exl3_moe_prefill: scratch must be 16-byte aligned");
    EXL3_REQUIRE(aligned16(x), EXL3_ERR_ARG, "exl3_moe_prefill: x must be 16-byte aligned");
    const PfGeom g = pf_geom(m, topk, hidden, inter, n_experts);
    EXL3_REQUIRE(scratch_bytes >= g.total, EXL3_ERR_ARG, "exl3_moe_prefill: scratch too small (%lld < %lld bytes)",
                 (long long) scratch_bytes, (long long) g.total);
    auto encode = pf_encoder();
    EXL3_REQUIRE(encode != nullptr, EXL3_ERR_CUDA, "exl3_moe_prefill: cuTensorMapEncodeTiled is not available");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    DeviceInfo di;
    {
        const int drc = device_info(dev, &di);
        if (drc != EXL3_OK) return drc;
    }
    int rc = cb == 0 ? pf_set_attr<0>() : cb == 1 ? pf_set_attr<1>() : pf_set_attr<2>();
    if (rc != EXL3_OK) return rc;

    uint8_t* sb = static_cast<uint8_t*>(scratch);
    PfParams p{};
    {
        const int64_t rows_cap = g.cap;
        __half* bufs[3] = {reinterpret_cast<__half*>(sb + g.off_xg), reinterpret_cast<__half*>(sb + g.off_xu),
                           reinterpret_cast<__half*>(sb + g.off_xd)};
        const int64_t widths[3] = {hidden, hidden, inter};
        CUtensorMap* maps[3] = {&p.xg_map, &p.xu_map, &p.xd_map};
        for (int i = 0; i < 3; ++i) {
            const cuuint64_t dims[2] = {(cuuint64_t) widths[i], (cuuint64_t) rows_cap};
            const cuuint64_t strides[1] = {(cuuint64_t) widths[i] * 2};
            const cuuint32_t box[2] = {(cuuint32_t) kPfKStep, (cuuint32_t) kPfBoxRows};
            const cuuint32_t estr[2] = {1u, 1u};
            const CUresult r = encode(maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, bufs[i], dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_moe_prefill: activation tensor map failed (%d)",
                         (int) r);
        }
    }
    const int64_t* tabs[9] = {gate_trellis, gate_suh, gate_svh, up_trellis, up_suh, up_svh,
                              down_trellis, down_suh, down_svh};
    for (int i = 0; i < 9; ++i) p.tab[i] = tabs[i];
    p.ktab = k_table;
    p.Kscalar = K;
    shift_table_init(p.st);
    p.E = (int) n_experts;
    p.H = (int) hidden;
    p.I = (int) inter;
    p.limit = swiglu_limit;
    p.ctrl = reinterpret_cast<uint32_t*>(sb);
    int* pl = reinterpret_cast<int*>(sb + g.off_plan);
    const int64_t E1 = n_experts + 1;
    p.plan.e_off = pl;
    p.plan.pass_off = pl + E1;
    p.plan.gu_off = pl + 2 * E1;
    p.plan.dn_off = pl + 3 * E1;
    p.plan.pair_tok = pl + 4 * E1;
    p.plan.pair_exp = pl + 4 * E1 + g.cap;
    p.plan.slot_pair = pl + 4 * E1 + 2 * g.cap;
    p.plan.units = reinterpret_cast<int4*>(sb + g.off_units);
    p.plan.unit_cap = (int) g.unit_cap;
    p.xd = reinterpret_cast<__half*>(sb + g.off_xd);
    p.dn = reinterpret_cast<float*>(sb + g.off_dn);
    p.maps = reinterpret_cast<CUtensorMap*>(sb + g.off_maps);
    {
        PfTemplates T{};
        const int trc = pf_templates(hidden, inter, sb + g.off_xg, &T);
        if (trc != EXL3_OK) return trc;
        for (int i = 0; i < 8; ++i) p.tmpl[i] = T.t[i];
    }
    const int grid = di.sms < kPfMaxGrid ? di.sms : kPfMaxGrid;

    // the status word reports this call
    EXL3_CUDA(cudaMemsetAsync(p.ctrl + 2, 0, sizeof(uint32_t), s));
    const int64_t ct = g.cap / topk;
    const int xb = 2;   // fp16 or bf16
    const int ob = out_dtype == 2 ? 4 : 2;
    for (int64_t t0 = 0; t0 < m; t0 += ct) {
        const int T = (int) (m - t0 < ct ? m - t0 : ct);
        const void* xc = static_cast<const uint8_t*>(x) + t0 * hidden * xb;
        void* oc = static_cast<uint8_t*>(out) + t0 * hidden * ob;
        const int64_t slot0 = t0 * topk;
        const int W = (T + 31) / 32;
        EXL3_CUDA(pf_launch(pf_plan_kernel, dim3(1), dim3(1024), (int) (n_experts * W * 4), s, false, route, slot0,
                            T, (int) topk, (int) n_experts, (int) hidden, (int) inter, p.ctrl, p.plan));
        int64_t ib = (int64_t) T * topk;
        if (ib > (int64_t) di.sms * 8) ib = (int64_t) di.sms * 8;
        EXL3_CUDA(pf_launch(pf_input_kernel, dim3((unsigned) ib), dim3(256), 0, s, true, xc, x_dtype, (int) hidden,
                            (const uint32_t*) p.ctrl, (const int*) p.plan.pair_tok,
                            (const int*) p.plan.pair_exp, gate_suh, up_suh, reinterpret_cast<__half*>(sb + g.off_xg),
                            reinterpret_cast<__half*>(sb + g.off_xu)));
        switch (cb) {
            case 0: EXL3_CUDA(pf_launch(pf_gemm_kernel<0>, dim3(grid), dim3(kPfThreads), kPfSmem, s, true, p)); break;
            case 1: EXL3_CUDA(pf_launch(pf_gemm_kernel<1>, dim3(grid), dim3(kPfThreads), kPfSmem, s, true, p)); break;
            default: EXL3_CUDA(pf_launch(pf_gemm_kernel<2>, dim3(grid), dim3(kPfThreads), kPfSmem, s, true, p)); break;
        }
        int64_t gb = ((int64_t) T * (hidden / 4) + 255) / 256;
        if (gb > (int64_t) di.sms * 8) gb = (int64_t) di.sms * 8;
        EXL3_CUDA(pf_launch(pf_gather_kernel, dim3((unsigned) gb), dim3(256), 0, s, true, (const float*) p.dn,
                            (const int*) p.plan.slot_pair, route, slot0, T, (int) topk, (int) hidden, oc,
                            out_dtype));
    }
    return EXL3_OK;
}

extern "C" int exl3_moe_prefill(const void* x, int x_dtype, void* out, int out_dtype, int64_t m, int64_t hidden,
                                int64_t inter, const int64_t* gate_trellis, const int64_t* gate_suh,
                                const int64_t* gate_svh, const int64_t* up_trellis, const int64_t* up_suh,
                                const int64_t* up_svh, const int64_t* down_trellis, const int64_t* down_suh,
                                const int64_t* down_svh, int64_t n_experts, const int32_t* k_table, int K, int kmax,
                                int cb, const int32_t* ids, const float* weights, int64_t topk, float swiglu_limit,
                                void* scratch, int64_t scratch_bytes, void* stream) {
    const RouteIn route{ids, weights, nullptr, 0, 0, 2};
    return moe_prefill_impl(x, x_dtype, out, out_dtype, m, hidden, inter, gate_trellis, gate_suh, gate_svh,
                            up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh, n_experts, k_table, K, kmax,
                            cb, route, topk, swiglu_limit, scratch, scratch_bytes, stream);
}

extern "C" int exl3_moe_prefill_routed(const void* x, int x_dtype, void* out, int out_dtype, int64_t m,
                                       int64_t hidden, int64_t inter, const int64_t* gate_trellis,
                                       const int64_t* gate_suh, const int64_t* gate_svh, const int64_t* up_trellis,
                                       const int64_t* up_suh, const int64_t* up_svh, const int64_t* down_trellis,
                                       const int64_t* down_suh, const int64_t* down_svh, int64_t n_experts,
                                       const int32_t* k_table, int K, int kmax, int cb, const exl3_moe_route* route,
                                       int64_t topk, float swiglu_limit, void* scratch, int64_t scratch_bytes,
                                       void* stream) {
    RouteIn r;
    if (int rc = route_from_abi(route, &r)) return rc;
    return moe_prefill_impl(x, x_dtype, out, out_dtype, m, hidden, inter, gate_trellis, gate_suh, gate_svh,
                            up_trellis, up_suh, up_svh, down_trellis, down_suh, down_svh, n_experts, k_table, K, kmax,
                            cb, r, topk, swiglu_limit, scratch, scratch_bytes, stream);
}

}  // namespace exl3
