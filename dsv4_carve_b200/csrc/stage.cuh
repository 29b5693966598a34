// stage.cuh -- the consumer side of a TMA ring shared by the routed-MoE and
// dense EXL3 kernels: one ring stage holds SK k-slices of 8 weight tiles
// (the weight part, `wpart` bytes) followed by the matching B fragments of
// the unit's rows; consumer warp w decodes tile w of every k-slice in
// registers and runs the MMAs against those fragments.
#pragma once

#include "engine.cuh"

// With -DEXL3_PHASE_CLOCK the consumer also accumulates the cycles it spends
// waiting for stage data into the caller's counter.
#ifdef EXL3_PHASE_CLOCK
#define PH_PARAM , unsigned long long& ph_wait
#define PH_FWD , ph_wait
#else
#define PH_PARAM
#define PH_FWD
#endif

namespace exl3 {

constexpr int kStageSK = 8;   // k-slices per ring stage

struct RingGeom {
    int slot_bytes;           // bytes per stage
    int ns;                   // stages in the ring
    int wpart;                // weight part of a stage
    ShiftTable st;            // IMAD shift multipliers of the window extraction (shift_table_init)
};

// B-fragment words per lane per row-slice: fast arithmetic keeps every
// activation duplicated into both halves of a word (4 words: k = 2t, 2t+8,
// 2t+1, 2t+9), the precise path packs pairs (2 words: (2t, 2t+1), (2t+8, 2t+9)).
template <bool PRECISE> struct Frag { static constexpr int FW = PRECISE ? 2 : 4; };

// Store one transformed activation (row-slice base `rs`, words) at in-slice
// position kk (0..15) in the fragment layout of Frag<PRECISE>.
template <bool PRECISE>
__device__ __forceinline__ void store_frag(uint32_t* rs, int kk, __half h) {
    const int t = (kk & 7) >> 1;
    if constexpr (PRECISE) {
        reinterpret_cast<__half*>(rs)[t * 4 + 2 * (kk >= 8 ? 1 : 0) + (kk & 1)] = h;
    } else {
        rs[t * 4 + ((kk & 1) ? 2 : 0) + (kk >= 8 ? 1 : 0)] = dup_half(h);
    }
}

// Decode + MMA over `nst` ring stages of one unit; bit width K and row-block
// count RB are compile-time so the inner loop carries no predicated MMAs.
// The B fragments come from each stage after its weight part, or, when
// `bext` is given, from that shared-memory array (the unit's fragments,
// kStageSK k-slices per stage, consecutive).
template <int K, int RB, int CB, bool PRECISE>
__device__ __forceinline__ bool ring_consume(const RingGeom& p, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                            uint32_t& it, int nst, int nrows, float (&acc)[4][4], int cwarp,
                                            int lane, uint32_t* status, const uint32_t* bext PH_PARAM) {
    using F = TileFmt<K>;
    constexpr int FW = Frag<PRECISE>::FW;
    constexpr int ROWW = 8 * F::WORDS;                 // words per k-slice row (8 tiles)
    const LaneGeom<K> geom = lane_geom<K>(lane);
    const int t4 = lane & 3, gr = lane >> 2;
    int boff[RB];
#pragma unroll
    for (int rb = 0; rb < RB; ++rb) boff[rb] = min(rb * 8 + gr, nrows - 1) * 4 * FW + t4 * FW;
    const int bstride = nrows * 4 * FW;                 // words per row-slice block of the unit
    float acc_odd[RB][4];                               // odd-k MMAs (fast path), added to acc at the end
#pragma unroll
    for (int rb = 0; rb < RB; ++rb)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc_odd[rb][q] = 0.f;
    // ring position as running counters (one division per unit, not per stage)
    int slot = (int) (it % (uint32_t) p.ns);
    uint32_t phase = (it / (uint32_t) p.ns) & 1u;
    for (int st = 0; st < nst; ++st) {
#ifdef EXL3_PHASE_CLOCK
        const unsigned long long w0_ = clock64();
#endif
        if (!mbar_wait_lanes(&full[slot], phase, status)) return false;
#ifdef EXL3_PHASE_CLOCK
        ph_wait += clock64() - w0_;
#endif
        const uint32_t* base = reinterpret_cast<const uint32_t*>(ring + (size_t) slot * p.slot_bytes);
        const uint32_t* phi[F::NG];
        const uint32_t* plo[F::NG];
#pragma unroll
        for (int h = 0; h < F::NG; ++h) {
            phi[h] = base + cwarp * F::WORDS + geom.ihi[h];
            plo[h] = base + cwarp * F::WORDS + geom.ilo[h];
        }
        const uint32_t* bf = bext != nullptr ? bext + st * kStageSK * bstride : base + p.wpart / 4;
#pragma unroll
        for (int i = 0; i < kStageSK; ++i) {
            uint32_t whi[F::NG], wlo[F::NG];
#pragma unroll
            for (int h = 0; h < F::NG; ++h) {
                whi[h] = phi[h][i * ROWW];
                wlo[h] = plo[h][i * ROWW];
            }
            uint32_t w[8], x[8];
            tile_windows_f<K>(whi, wlo, geom, p.st, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = codebook_pair<CB>(w[j]);
            const uint32_t* bs = bf + i * bstride;
#pragma unroll
            for (int rb = 0; rb < RB; ++rb) {
                if constexpr (PRECISE) {
                    mma_tile_precise(acc[rb], x, *reinterpret_cast<const uint2*>(bs + boff[rb]));
                } else {
                    mma_tile2(acc[rb], acc_odd[rb], x, *reinterpret_cast<const uint4*>(bs + boff[rb]));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++it;
        if (++slot == p.ns) { slot = 0; phase ^= 1u; }
    }
    if constexpr (!PRECISE) {
#pragma unroll
        for (int rb = 0; rb < RB; ++rb)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[rb][q] += acc_odd[rb][q];
    }
    return true;
}

template <int K, int CB, bool PRECISE>
__device__ __forceinline__ bool ring_consume_rb(int RB, const RingGeom& p, uint8_t* ring, uint64_t* full,
                                               uint64_t* empty, uint32_t& it, int nst, int nrows, float (&acc)[4][4],
                                               int cwarp, int lane, uint32_t* status, const uint32_t* bext PH_PARAM) {
    switch (RB) {
        case 1: return ring_consume<K, 1, CB, PRECISE>(p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, bext PH_FWD);
        case 2: return ring_consume<K, 2, CB, PRECISE>(p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, bext PH_FWD);
        case 3: return ring_consume<K, 3, CB, PRECISE>(p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, bext PH_FWD);
        default: return ring_consume<K, 4, CB, PRECISE>(p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, bext PH_FWD);
    }
}

template <int CB, bool PRECISE>
__device__ __forceinline__ bool ring_consume_any(int K, int RB, const RingGeom& p, uint8_t* ring, uint64_t* full,
                                                uint64_t* empty, uint32_t& it, int nst, int nrows, float (&acc)[4][4],
                                                int cwarp, int lane, uint32_t* status PH_PARAM) {
    switch (K) {
        case 1: return ring_consume_rb<1, CB, PRECISE>(RB, p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, nullptr PH_FWD);
        case 2: return ring_consume_rb<2, CB, PRECISE>(RB, p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, nullptr PH_FWD);
        case 3: return ring_consume_rb<3, CB, PRECISE>(RB, p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, nullptr PH_FWD);
        default: return ring_consume_rb<4, CB, PRECISE>(RB, p, ring, full, empty, it, nst, nrows, acc, cwarp, lane, status, nullptr PH_FWD);
    }
}

}  // namespace exl3
