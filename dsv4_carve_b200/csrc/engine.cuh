// engine.cuh -- the streaming GEMV engine shared by the dense linear and the
// routed-MoE decode kernels.
//
// One CTA = 8 consumer warps + 1 producer warp (288 threads), persistent.
// Work is cut into UNITS: (matrix, 128 output columns, k-chunk).  The
// producer warp claims units with a global ticket counter and streams each
// unit's packed trellis rows into a shared-memory ring with 1-D bulk copies
// (cp.async.bulk, completion on an mbarrier).  Consumer warp w owns the 16
// output columns of n-tile w of the unit; per k-slice it decodes its tile in
// registers (decode.cuh) and runs the MMAs against the unit's activations,
// which are prepared once per unit as B fragments in shared memory.
//
// A unit that covers only part of k writes an fp32 partial; the LAST unit of
// a column block (atomic counter) sums all partials in fixed chunk order, so
// results are bitwise reproducible, and applies the output transform.  No
// grid-wide barrier and no co-residency assumption anywhere.
#pragma once

#include "decode.cuh"

namespace exl3 {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kDQ = 4;                 // descriptor queue depth
constexpr int kActBytes = 32768;       // B-fragment buffer
constexpr int kMaxRows = 32;           // rows per unit on the small-R path
constexpr int kCols = 128;             // output columns per unit (one Hadamard block)
constexpr uint32_t kBarConsumers = 1;  // named barrier id (consumer warps only)

__host__ __device__ constexpr int stage_slices(int K) {
    // k-slices per ring stage: 8 slices = one 128-wide Hadamard block of k
    // (so every 128-multiple k-chunk is a whole number of stages), 4 for K >= 7
    // to keep a stage <= 8 KB.
    return K <= 6 ? 8 : 4;
}

__host__ __device__ constexpr int row_blocks(int rows) { return (rows + 7) >> 3; }

// k-slices of activations that fit in the B-fragment buffer for rb blocks.
__host__ __device__ constexpr int act_slices(int rb) { return kActBytes / (rb * 512); }

__device__ __forceinline__ void consumers_sync() { named_sync(kBarConsumers, kConsumerThreads); }
__device__ __forceinline__ bool consumers_all(bool v) { return named_all(kBarConsumers, kConsumerThreads, v); }

// ------------------------------------------------------------ activations
// Fill the B-fragment buffer for k-slices [ks0, ks0 + nks) of the unit.
//   rows[i]   : row index of unit row i in `src`
//   src       : activations, row-major with leading dimension `ld` (elements)
//   suh       : input sign/scale vector; when null, src is already fp16 and
//               transformed (the MoE down input) and is copied as is.
// Element (row i, k) of the slice range lands in fragment
//   ((ks * RB + i/8) * 32 + 4*(i%8) + (kk%8)/2), component (kk odd ? 2 : 0) + (kk >= 8)
// with ks = (k - k0)/16, kk = k % 16, matching mma_tile()'s B registers.
// PRECISE layout (mma_tile_precise): one uint2 per lane, element (i, k) at
//   u16 index (((ks * RB + i/8) * 32 + 4*(i%8) + (kk%8)/2) * 4 + 2*(kk >= 8) + (kk & 1)).
template <bool PRECISE>
__device__ __forceinline__ void build_bfrag(uint4* bfrag, int RB, int nrows, const int* rows,
                                            const void* src, int src_dtype, int64_t ld,
                                            int ks0, int nks, const __half* suh,
                                            int cwarp, int lane) {
    uint32_t* bf32 = reinterpret_cast<uint32_t*>(bfrag);
    // Padding rows (i >= nrows) are not written: column n of an MMA's D
    // depends only on column n of B, so whatever their B columns hold only
    // reaches accumulator columns that are never read.
    const int nblk = nks / 8;                 // 128-wide blocks in the range
    const int items = nrows * nblk;
    for (int it = cwarp; it < items; it += kConsumerWarps) {
        const int i = it / nblk;              // unit row
        const int b = it % nblk;
        const int kloc = b * 128 + lane * 4;  // offset inside the slice range
        const int64_t kglob = (int64_t) ks0 * 16 + kloc;
        __half h[4];
        {
            const int64_t base = (int64_t) rows[i] * ld + kglob;
            if (suh != nullptr) {
                float v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const __half a = load_act_half(src, src_dtype, base + q);
                    v[q] = __half2float(__hmul(a, suh[kglob + q]));
                }
                wht128_warp(v, lane);
#pragma unroll
                for (int q = 0; q < 4; ++q) h[q] = __float2half_rn(v[q] * kHadNorm);
            } else {
                const __half* s = reinterpret_cast<const __half*>(src) + base;
                const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(s));
                h[0] = __ushort_as_half((uint16_t) (raw.x & 0xffffu));
                h[1] = __ushort_as_half((uint16_t) (raw.x >> 16));
                h[2] = __ushort_as_half((uint16_t) (raw.y & 0xffffu));
                h[3] = __ushort_as_half((uint16_t) (raw.y >> 16));
            }
        }
        const int rb = i >> 3, g = i & 7;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int kl = kloc + q;
            const int ks = kl >> 4, kk = kl & 15;
            const int frag = (ks * RB + rb) * 32 + 4 * g + ((kk & 7) >> 1);
            if constexpr (PRECISE) {
                __half* bf16 = reinterpret_cast<__half*>(bfrag);
                bf16[frag * 4 + (kk >= 8 ? 2 : 0) + (kk & 1)] = h[q];
            } else {
                const int comp = ((kk & 1) ? 2 : 0) + (kk >= 8 ? 1 : 0);
                bf32[frag * 4 + comp] = dup_half(h[q]);
            }
        }
    }
}

// ------------------------------------------------------------ main loop
// Consume `nst` ring stages of one unit.  Each stage holds SK k-slices, each
// k-slice the 8 tiles (8 * 32K bytes) of the unit's 128 columns.  Warp w
// decodes tile w of every k-slice.  `ksl` is the k-slice index (within the
// current B-fragment range) of the stage's first slice.
template <int K, int CB, int RB, int NS, int STAGE_BYTES, int SK, bool PRECISE>
__device__ __forceinline__ bool consume_stages(uint8_t (*ring)[STAGE_BYTES], uint64_t* full,
                                               uint64_t* empty, uint32_t& it, int nst, int ksl,
                                               const uint4* bfrag, float (&acc)[4][4],
                                               const LaneGeom<K>& geom, int cwarp, int lane,
                                               uint32_t* status) {
    // SK = k-slices per ring stage as packed by the producer (a property of the
    // ring, not of K: the MoE ring is shared by experts of different K).
    // Per stage, each lane forms one pointer per word it reads; inside the
    // fully unrolled k-slice loop every shared-memory load then uses a
    // compile-time offset.
    using F = TileFmt<K>;
    constexpr int ROWW = 8 * F::WORDS;          // uint32 words per k-slice row (8 tiles)
    constexpr int BFW = PRECISE ? 2 : 4;        // uint32 words of B fragment per lane
    const uint32_t* bfbase = reinterpret_cast<const uint32_t*>(bfrag) + lane * BFW;
    for (int st = 0; st < nst; ++st) {
        const int slot = it % NS;
        if (!mbar_wait_warp(&full[slot], (it / NS) & 1u, status, lane)) return false;
        const uint32_t* tile0 = reinterpret_cast<const uint32_t*>(ring[slot]) + cwarp * F::WORDS;
        const uint32_t* phi[F::NG];
        const uint32_t* plo[F::NG];
#pragma unroll
        for (int h = 0; h < F::NG; ++h) {
            phi[h] = tile0 + geom.ihi[h];
            plo[h] = tile0 + geom.ilo[h];
        }
        const uint32_t* bfs = bfbase + (ksl + st * SK) * RB * 32 * BFW;
#pragma unroll
        for (int i = 0; i < SK; ++i) {
            uint32_t whi[F::NG], wlo[F::NG];
#pragma unroll
            for (int h = 0; h < F::NG; ++h) {
                whi[h] = phi[h][i * ROWW];
                wlo[h] = plo[h][i * ROWW];
            }
            uint32_t w[8], x[8];
            tile_windows_w<K>(whi, wlo, geom, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = codebook_pair<CB>(w[j]);
#pragma unroll
            for (int rb = 0; rb < RB; ++rb) {
                const uint32_t* b = bfs + (i * RB + rb) * 32 * BFW;
                if constexpr (PRECISE) {
                    const uint2 bf = *reinterpret_cast<const uint2*>(b);
                    mma_tile_precise(acc[rb], x, bf);
                } else {
                    const uint4 bf = *reinterpret_cast<const uint4*>(b);
                    mma_tile(acc[rb], x, bf);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++it;
    }
    return true;
}

// Accumulators -> cbuf[row][128] (fp32).  acc[rb] = D[ch][row] fragments:
// (ch g, row 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1) of n-tile cwarp.
__device__ __forceinline__ void acc_to_cbuf(float* cbuf, const float (&acc)[4][4], int RB, int cwarp,
                                            int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int ch = cwarp * 16 + g;
    for (int rb = 0; rb < RB; ++rb) {
        const int r = rb * 8 + 2 * t;
        cbuf[r * kCols + ch] = acc[rb][0];
        cbuf[(r + 1) * kCols + ch] = acc[rb][1];
        cbuf[r * kCols + ch + 8] = acc[rb][2];
        cbuf[(r + 1) * kCols + ch + 8] = acc[rb][3];
    }
}

// ------------------------------------------------------------ producer
// Issue the bulk copies for one ring stage: SK rows of `rowbytes` bytes from
// src + s * rowstride.  Lane 0 arms the barrier, lanes 0..SK-1 copy.  When
// `valid` is false (a bad pointer was detected) the stage is completed
// without data so the consumers never wait forever.
template <int NS, int STAGE_BYTES>
__device__ __forceinline__ bool produce_stage(uint8_t (*ring)[STAGE_BYTES], uint64_t* full,
                                              uint64_t* empty, uint32_t& it, const uint8_t* src,
                                              int64_t rowstride, int rowbytes, int nrows, bool valid,
                                              int lane, uint32_t* status) {
    const int slot = it % NS;
    bool ok = true;
    if (lane == 0) {
        ok = mbar_wait(&empty[slot], ((it / NS) + 1u) & 1u, status);
        if (ok) {
            if (valid) mbar_arrive_expect_tx(&full[slot], (uint32_t) (rowbytes * nrows));
            else mbar_arrive(&full[slot]);
        }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (!ok) return false;
    if (valid && lane < nrows)
        bulk_g2s(ring[slot] + lane * rowbytes, src + lane * rowstride, (uint32_t) rowbytes, &full[slot]);
    ++it;
    return true;
}

// Before the producer warp exits, wait (bounded) until every stage it issued
// has landed, so no bulk copy is still writing into shared memory when the
// CTA retires.  On the normal path the consumers have already waited on all
// of them and this returns at once; it matters only after an error made the
// consumers stop early.  Stage i occupies slot i % NS in phase i / NS.
template <int NS>
__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t it, int lane, uint32_t* status) {
    if (lane != 0) return;
    const uint32_t first = it > (uint32_t) NS ? it - (uint32_t) NS : 0u;
    for (uint32_t i = first; i < it; ++i)
        if (!mbar_wait(&full[i % NS], (i / NS) & 1u, status)) break;
}

// Next unit ticket.  Every ticket, the first included, comes from the global
// counter, so a unit is only ever owned by a CTA that is already running.
__device__ __forceinline__ int claim_ticket(uint32_t* counter, int lane) {
    int t = 0;
    if (lane == 0) t = (int) atomicAdd(counter, 1u);
    return __shfl_sync(0xffffffffu, t, 0);
}

// ------------------------------------------------------------ epilogue helpers
// Output transform of one 128-column row held as 4 values per lane:
// v <- H128(v) / sqrt(128) * svh.
__device__ __forceinline__ void out_transform(float (&v)[4], const __half* svh_blk, int lane) {
    wht128_warp(v, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = v[q] * kHadNorm * __half2float(svh_blk[lane * 4 + q]);
}

}  // namespace exl3
