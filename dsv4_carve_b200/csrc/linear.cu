// linear.cu -- dense EXL3 linear (GEMV form) and trellis dequant for sm_100a.
//
// exl3_linear: y = x . W for small row counts, the dense 6-bit path of the
// attention / shared-expert linears (reference: LinearEXL3.forward ->
// BC_LinearEXL3.run_alloc -> exl3_gemm_gr, recipe-lna/exllamav3/exl3.py.lna:114-139,
// recipe-lna/exllamav3/exl3_gemm.cu.lna:123-334).  Same arithmetic boundaries
// as the reference: input fp16(x) * suh in fp16, 128-block Hadamard in fp32
// rounded to fp16, fp32 accumulation, output Hadamard and svh in fp32, one
// cast to the output dtype.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "host.hpp"
#include "stage.cuh"

namespace exl3 {

// ------------------------------------------------------------------ dequant
// One warp per tile; W' element (16a + k, 16b + n) = RN(lo + hi).
template <int K, int CB>
__global__ void __launch_bounds__(256) decode_kernel(const uint8_t* __restrict__ trellis, int64_t kt,
                                                     int64_t nt, __half* __restrict__ wprime) {
    const int lane = threadIdx.x & 31;
    const LaneGeom<K> geom = lane_geom<K>(lane);
    const int64_t ntiles = kt * nt;
    const int64_t cols = nt * 16;
    const int q = lane & 3, g = lane >> 2;
    for (int64_t tile = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5); tile < ntiles;
         tile += (int64_t) gridDim.x * 8) {
        const uint32_t* tw = reinterpret_cast<const uint32_t*>(trellis + tile * TileFmt<K>::BYTES);
        uint32_t w[8];
        tile_windows<K>(tw, geom, w);
        const int64_t a = tile / nt, b = tile % nt;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = 2 * q + (j & 1) + 8 * ((j >> 1) & 1);
            const int n = g + 8 * (j >> 2);
            wprime[(a * 16 + k) * cols + b * 16 + n] = codebook_value<CB>(w[j]);
        }
    }
}

// One CTA per 128x128 block: decode, row transform, column transform with
// suh/svh, in the float order of the reference's dequant_cpu
// (recipe-lna/lna2/bindings.cpp:79-99): rows first, then columns, value =
// ((h * norm) * su) * sv, one rounding to fp16.
constexpr int kRecPitch = 129;
template <int K, int CB>
__global__ void __launch_bounds__(256) reconstruct_kernel(const uint8_t* __restrict__ trellis, int64_t nt,
                                                          const __half* __restrict__ suh,
                                                          const __half* __restrict__ svh,
                                                          __half* __restrict__ w) {
    extern __shared__ float m[];   // [128][kRecPitch]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bk = blockIdx.y, bn = blockIdx.x;
    const int64_t cols = nt * 16;
    const LaneGeom<K> geom = lane_geom<K>(lane);
    const int q = lane & 3, g = lane >> 2;
    for (int tt = warp; tt < 64; tt += 8) {
        const int a = tt >> 3, b = tt & 7;
        const int64_t tile = (bk * 8 + a) * nt + bn * 8 + b;
        const uint32_t* tw = reinterpret_cast<const uint32_t*>(trellis + tile * TileFmt<K>::BYTES);
        uint32_t wv[8];
        tile_windows<K>(tw, geom, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = 2 * q + (j & 1) + 8 * ((j >> 1) & 1);
            const int n = g + 8 * (j >> 2);
            m[(a * 16 + k) * kRecPitch + b * 16 + n] = __half2float(codebook_value<CB>(wv[j]));
        }
    }
    __syncthreads();
    for (int r = warp; r < 128; r += 8) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = m[r * kRecPitch + lane * 4 + i];
        wht128_warp(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) m[r * kRecPitch + lane * 4 + i] = __fmul_rn(v[i], kHadNorm);
    }
    __syncthreads();
    for (int c = warp; c < 128; c += 8) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = m[(lane * 4 + i) * kRecPitch + c];
        wht128_warp(v, lane);
        const float sv = __half2float(svh[bn * 128 + c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float su = __half2float(suh[bk * 128 + lane * 4 + i]);
            m[(lane * 4 + i) * kRecPitch + c] = __fmul_rn(__fmul_rn(__fmul_rn(v[i], kHadNorm), su), sv);
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 128 * 128; idx += 256) {
        const int r = idx >> 7, c = idx & 127;
        w[(bk * 128 + r) * cols + bn * 128 + c] = __float2half_rn(m[r * kRecPitch + c]);
    }
}

// ------------------------------------------------------------------ linear
// One persistent launch per (<= 32-row) block of rows.  Warps 0-7 decode +
// MMA, warp 8 produces (unit tickets, one 3-D TMA box of weights per ring
// stage), warp 9 stores each unit's partial tile, counts completions per
// 128-column block and finishes the block.  Units are (128-column block,
// k-chunk) in block-major order; a CTA's first unit is its block index, the
// rest come from a ticket counter.
//
// Launched with programmatic dependent launch: the producer streams its first
// unit's weights before griddepcontrol.wait (weights never depend on the
// preceding kernel), and every access to the input, the scratch and the output
// comes after it.  The consumers transform the unit's own k-chunk of the input
// (x -> fp16, * suh in fp16, 128-point Hadamard in fp32 -> fp16) straight into
// B-fragment order in shared memory, so no unit waits on another CTA's input
// work.  The finisher sums a block's chunk partials in fixed order and applies
// Hadamard * svh and the cast, so results are bitwise reproducible.
constexpr int kLinConsumerWarps = 8;
constexpr int kLinProducerWarp = 8;
constexpr int kLinEpilogueWarp = 9;
constexpr int kLinThreads = 320;
constexpr int kLinMaxRows = 32;
constexpr int kLinMaxChunks = 16;            // k-chunks per 128-column block
constexpr int kLinRingBytes = 98304;         // weight ring + partial tiles + the unit's input fragments
constexpr int kLinFragBytes = 32768;         // most shared memory the unit's input fragments may take
constexpr int kLinMaxStages = 12;
constexpr int kLinDQ = 4;
constexpr int kLinMaxMats = 8;               // matrices of one grouped launch (shared input)
// control words: [0] unit ticket [1] retired CTAs [2] status; block counters
// (over all matrices' 128-column blocks) from word 16
constexpr int kLinOffCnt = 16;

// One launch applies nmat matrices (same k, K and codebook) to the same input
// rows: matrix j has its own trellis map, suh, svh, width n[j] and output
// y[j]; its 128-column blocks are blocks blk0[j] .. blk0[j+1]-1 of the launch.
struct LinearParams {
    CUtensorMap tmap[kLinMaxMats];   // trellis as [k/16][n/16][16K] u16, box [16K, 8, SK]
    const void* x;
    int x_dtype;
    int rows;
    int k, nmat, ntot;               // ntot = sum of n[j] (row stride of the partials)
    int n[kLinMaxMats];
    int blk0[kLinMaxMats + 1];
    const __half* suh[kLinMaxMats];
    const __half* svh[kLinMaxMats];
    void* y[kLinMaxMats];
    int y_dtype;
    int kc, nk;                 // k-chunk per unit, chunk count
    RingGeom ring;              // stages hold weights only (slot_bytes == wpart)
    uint32_t* ctrl;
    float* partial;             // [nk][rows][ntot]
};

struct alignas(128) LinHead {
    uint64_t full[kLinMaxStages];
    uint64_t empty[kLinMaxStages];
    uint64_t dqf[kLinDQ];
    uint64_t dqe[kLinDQ];
    uint64_t pfull[2];
    uint64_t pempty[2];
    uint64_t xfree;             // every consumer warp is done with the previous unit's input fragments
    uint64_t xready;            // every consumer warp has written its share of this unit's fragments
    uint64_t fin_bar;           // the epilogue warp has published fin_blk (after its last unit)
    int desc[kLinDQ][4];        // valid, block, chunk
    int fin_blk;                // block whose rows every warp finishes at the end, or -1
    int last_cta;
};
constexpr int kLinHeadBytes = (int) ((sizeof(LinHead) + 127) / 128 * 128);

// Per-CTA timeline of the trace build (-DEXL3_PHASE_CLOCK; %globaltimer ns):
// entry, past griddepcontrol.wait (consumer warp 0), first unit's input
// fragments ready, first unit decoded, epilogue's first partial counted,
// epilogue done, exit.  Read with exl3_linear_timeline_read.
#ifdef EXL3_PHASE_CLOCK
static __device__ unsigned long long g_ltl[512][8];
#define LTL_MARK(i) do { if ((threadIdx.x & 31) == 0 && blockIdx.x < 512) g_ltl[blockIdx.x][i] = globaltimer_ns(); } while (0)
#else
#define LTL_MARK(i)
#endif

// Matrix of launch-wide 128-column block blk.
__device__ __forceinline__ int lin_matrix(const LinearParams& p, int blk) {
    int mat = 0;
    while (mat + 1 < p.nmat && blk >= p.blk0[mat + 1]) ++mat;
    return mat;
}

// Row r of block blk's epilogue, by one warp: the k-chunk partials summed in
// chunk order (all in flight at once), Hadamard * svh, one cast into y.
__device__ __noinline__ void lin_finish_row(const LinearParams& p, int blk, int r, int lane) {
    const int mat = lin_matrix(p, blk);
    const int lb = blk - p.blk0[mat];   // the block within its matrix
    const float* col0 = p.partial + blk * kCols + lane * 4;
    float4 a[kLinMaxChunks];
#pragma unroll
    for (int c2 = 0; c2 < kLinMaxChunks; ++c2)
        if (c2 < p.nk) a[c2] = __ldcg(reinterpret_cast<const float4*>(col0 + ((int64_t) c2 * p.rows + r) * p.ntot));
    float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c2 = 0; c2 < kLinMaxChunks; ++c2)
        if (c2 < p.nk) { v[0] += a[c2].x; v[1] += a[c2].y; v[2] += a[c2].z; v[3] += a[c2].w; }
    out_transform(v, p.svh[mat] + lb * kCols, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) store_out(p.y[mat], p.y_dtype, (int64_t) r * p.n[mat] + lb * kCols + lane * 4 + q, v[q]);
}

// Bounded rendezvous of the consumer warps on an mbarrier of count 8.
__device__ __forceinline__ bool lin_rendezvous(uint64_t* bar, uint32_t parity, int lane, uint32_t* status) {
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
    return mbar_wait_lanes(bar, parity, status);
}

template <int K, int CB, bool PRECISE>
__global__ void __launch_bounds__(kLinThreads, 2) linear_kernel(const __grid_constant__ LinearParams p) {
    constexpr int FW = Frag<PRECISE>::FW;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    LinHead& S = *reinterpret_cast<LinHead*>(smem_raw);
    uint8_t* ring = smem_raw + kLinHeadBytes;
    const int rows = p.rows;
    float* ptile = reinterpret_cast<float*>(ring + (size_t) p.ring.ns * p.ring.slot_bytes);   // [2][rows][128]
    uint32_t* xfrag = reinterpret_cast<uint32_t*>(ptile + 2 * rows * kCols);                   // [kc/16][rows][4*FW]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* status = p.ctrl + 2;
    uint32_t* cnt = p.ctrl + kLinOffCnt;
    const int NB = p.blk0[p.nmat];
    const int total = NB * p.nk;

    if (tid == 0) LTL_MARK(0);
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < p.ring.ns; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], kLinConsumerWarps); }
        for (int s = 0; s < kLinDQ; ++s) { mbar_init(&S.dqf[s], 1); mbar_init(&S.dqe[s], kLinConsumerWarps + 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&S.pfull[s], kLinConsumerWarps); mbar_init(&S.pempty[s], 1); }
        mbar_init(&S.xfree, kLinConsumerWarps);
        mbar_init(&S.xready, kLinConsumerWarps);
        mbar_init(&S.fin_bar, 1);
        S.fin_blk = -1;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kLinProducerWarp) {
        // ------------------------------------------------------------ producer
        int ticket = (int) blockIdx.x;   // the grid never exceeds the unit count
        uint32_t it = 0, du = 0;
        bool ok = true, waited = false;
        const uint32_t wbytes = (uint32_t) (kStageSK * 8 * 32 * K);
        const int nst = p.kc / (16 * kStageSK);
        while (ok) {
            const bool end = ticket >= total;
            const int blk = end ? 0 : ticket / p.nk, s = end ? 0 : ticket % p.nk;   // blk over all matrices
            const int mat = lin_matrix(p, blk);
            if (lane == 0) {
                const int slot = du % kLinDQ;
                ok = mbar_wait(&S.dqe[slot], ((du / kLinDQ) + 1u) & 1u, status);
                if (ok) {
                    S.desc[slot][0] = end ? 0 : 1;
                    S.desc[slot][1] = blk;
                    S.desc[slot][2] = s;
                    mbar_arrive(&S.dqf[slot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            ++du;
            if (end || !ok) break;
            const int ks0 = s * (p.kc / 16);
            for (int st = 0; st < nst && ok; ++st) {
                const int slot = (int) (it % (uint32_t) p.ring.ns);
                if (lane == 0) {
                    ok = mbar_wait(&S.empty[slot], ((it / (uint32_t) p.ring.ns) + 1u) & 1u, status);
                    if (ok) {
                        uint8_t* dst = ring + (size_t) slot * p.ring.slot_bytes;
                        mbar_arrive_expect_tx(&S.full[slot], wbytes);
                        tma_load_3d(dst, &p.tmap[mat], 0, (blk - p.blk0[mat]) * 8, ks0 + st * kStageSK, &S.full[slot]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
                ++it;
            }
            if (!waited) {
                pdl_wait();   // the ticket counter is in the scratch the preceding launch restores
                waited = true;
            }
            int next_raw = 0;
            if (lane == 0) next_raw = (int) gridDim.x + (int) atomicAdd(&p.ctrl[0], 1u);
            ticket = __shfl_sync(0xffffffffu, next_raw, 0);
        }
        if (!waited) pdl_wait();
        // no bulk copy may still be writing shared memory when the CTA retires
        if (lane == 0) {
            const uint32_t first = it > (uint32_t) p.ring.ns ? it - (uint32_t) p.ring.ns : 0u;
            for (uint32_t i = first; i < it; ++i)
                if (!mbar_wait(&S.full[i % p.ring.ns], (i / p.ring.ns) & 1u, status)) break;
        }
    } else if (warp == kLinEpilogueWarp) {
        // ------------------------------------------------------------ epilogue
        pdl_wait();
        uint32_t du = 0, uu = 0;
        int pend_fin = -1;      // block whose epilogue this CTA owes
        while (true) {
            const int slot = du % kLinDQ;
            if (!mbar_wait_lanes(&S.dqf[slot], (du / kLinDQ) & 1u, status)) break;
            const int valid = S.desc[slot][0], blk = S.desc[slot][1], s = S.desc[slot][2];
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.dqe[slot]);
            ++du;
            if (!valid) break;
            if (pend_fin >= 0) {   // more units follow: finish the owed block alone
                for (int r = 0; r < rows; ++r) lin_finish_row(p, pend_fin, r, lane);
                pend_fin = -1;
            }
            const int ps = (int) (uu & 1u);
            if (!mbar_wait_lanes(&S.pfull[ps], (uu >> 1) & 1u, status)) break;
            const float* tile = ptile + (size_t) ps * rows * kCols;
            for (int r = 0; r < rows; ++r) {
                const float4 v = *reinterpret_cast<const float4*>(tile + r * kCols + lane * 4);
                __stcg(reinterpret_cast<float4*>(p.partial + ((int64_t) s * rows + r) * p.ntot + blk * kCols + lane * 4),
                       v);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.pempty[ps]);
            ++uu;
            int last = 0;
            if (lane == 0) {
                // release this unit's partial; the last unit also acquires the others'
                const uint32_t old = atom_add_acq_rel_gpu(&cnt[blk], 1u);
                last = old == (uint32_t) (p.nk - 1);
                if (last) atomicExch(&cnt[blk], 0u);
            }
            if (uu == 1) LTL_MARK(4);
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            if (rows <= 2) {       // nothing worth sharing: finish now
                for (int r = 0; r < rows; ++r) lin_finish_row(p, blk, r, lane);
                continue;
            }
            pend_fin = blk;   // finished when the next descriptor is in (alone) or after the last (shared)
        }
        // The block this CTA finishes last goes to all its warps: the
        // consumers have no units left and split its rows with this warp.
        if (lane == 0) S.fin_blk = pend_fin;
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.fin_bar);
        if (pend_fin >= 0)
            for (int r = kLinConsumerWarps; r < rows; r += kLinConsumerWarps + 1) lin_finish_row(p, pend_fin, r, lane);
        LTL_MARK(5);
    } else {
        // ------------------------------------------------------------ consumers
        pdl_wait();   // the input is the preceding kernel's output
        if (warp == 0) LTL_MARK(1);
        uint32_t it = 0, du = 0, uu = 0;
        const int t4 = lane & 3, gr = lane >> 2;
        const int RB = row_blocks(rows);
        const int nst = p.kc / (16 * kStageSK);
        const int cb = p.kc / kCols;                   // 128-blocks of k per unit
        while (true) {
            const int slot = du % kLinDQ;
            if (!mbar_wait_lanes(&S.dqf[slot], (du / kLinDQ) & 1u, status)) break;
            const int valid = S.desc[slot][0], blk = S.desc[slot][1], s = S.desc[slot][2];
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.dqe[slot]);
            ++du;
            if (!valid) break;
            // The unit's input chunk into B-fragment order in shared memory, one
            // (128-block, row) item per warp at a time, once every warp is done
            // with the previous unit's fragments.
            if (uu > 0 && !lin_rendezvous(&S.xfree, (uu - 1) & 1u, lane, status)) break;
            {
                // items (128-block kb of the chunk, row r), up to four per warp
                // at a time with all their loads issued before any is used
                constexpr int kBatch = 4;
                const int mat = lin_matrix(p, blk);
                const __half* su = p.suh[mat];
                const int nitems = cb * rows;
                for (int i0 = warp; i0 < nitems; i0 += kBatch * kLinConsumerWarps) {
                    __half xa[kBatch][4], sa[kBatch][4];
#pragma unroll
                    for (int b = 0; b < kBatch; ++b) {
                        const int item = i0 + b * kLinConsumerWarps;
                        if (item < nitems) {
                            const int r = item % rows, kb = item / rows;
                            const int k0 = (s * cb + kb) * kCols + lane * 4;
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                xa[b][q] = load_act_half(p.x, p.x_dtype, (int64_t) r * p.k + k0 + q);
                                sa[b][q] = su[k0 + q];
                            }
                        }
                    }
#pragma unroll
                    for (int b = 0; b < kBatch; ++b) {
                        const int item = i0 + b * kLinConsumerWarps;
                        if (item >= nitems) break;
                        const int r = item % rows, kb = item / rows;
                        float v[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) v[q] = __half2float(__hmul(xa[b][q], sa[b][q]));
                        wht128_warp(v, lane);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int kl = lane * 4 + q;
                            const int ks = kb * 8 + (kl >> 4);   // k-slice within the unit
                            store_frag<PRECISE>(xfrag + ((size_t) ks * rows + r) * 4 * FW, kl & 15,
                                                __float2half_rn(v[q] * kHadNorm));
                        }
                    }
                }
            }
            if (!lin_rendezvous(&S.xready, uu & 1u, lane, status)) break;
            if (warp == 0 && uu == 0) LTL_MARK(2);
            float acc[4][4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
#ifdef EXL3_PHASE_CLOCK
            unsigned long long ph_wait = 0;   // the dense kernel records no phases
#endif
            if (!ring_consume_rb<K, CB, PRECISE>(RB, p.ring, ring, S.full, S.empty, it, nst, rows, acc, warp, lane,
                                                 status, xfrag PH_FWD)) break;
            if (warp == 0 && uu == 0) LTL_MARK(3);
            const int ps = (int) (uu & 1u);
            if (!mbar_wait_lanes(&S.pempty[ps], ((uu >> 1) + 1u) & 1u, status)) break;
            float* tile = ptile + (size_t) ps * rows * kCols;
            const int col = warp * 16 + gr;
#pragma unroll
            for (int rb = 0; rb < 4; ++rb)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = rb * 8 + 2 * t4 + h;
                    if (r < rows) {
                        tile[r * kCols + col] = acc[rb][h];
                        tile[r * kCols + col + 8] = acc[rb][2 + h];
                    }
                }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.pfull[ps]);
            ++uu;
        }
        // rows of the block the epilogue warp shares out at the end (bounded wait)
        if (mbar_wait_lanes(&S.fin_bar, 0u, status)) {
            const int fb = *reinterpret_cast<volatile int*>(&S.fin_blk);
            if (fb >= 0)
                for (int r = warp; r < rows; r += kLinConsumerWarps + 1) lin_finish_row(p, fb, r, lane);
        }
    }

    // Retire: the last CTA out restores the control words for the next launch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&p.ctrl[1], 1u);
        S.last_cta = old == gridDim.x - 1;
    }
    __syncthreads();
    if (S.last_cta && tid == 0) {
        __threadfence();
        atomicExch(&p.ctrl[0], 0u);
        atomicExch(&p.ctrl[1], 0u);
    }
    if (tid == 0) LTL_MARK(6);
}

// ------------------------------------------------------------------ host side
// Tensor-core path for >= 64 rows (tc.cu).
int64_t linear_tc_scratch_bytes(int64_t rows, int64_t k, int64_t n);
bool linear_tc_eligible(int64_t rows, int64_t k, int64_t n);
int linear_tc(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t n, const void* trellis, int K, int cb,
              const void* suh, const void* svh, void* y, int y_dtype, void* scratch, cudaStream_t s);

namespace {

struct LinPrepared {
    bool ready = false;
    int grid = 0;
};
std::mutex g_lin_mu;
LinPrepared g_lin_prep[64][8][3][2];

template <int K, int CB, bool PRECISE>
int launch_linear(const LinearParams& p, int units, int smem, cudaStream_t stream) {
    // programmatic stream serialization: see the kernel's prologue
    auto kern = linear_kernel<K, CB, PRECISE>;
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    EXL3_REQUIRE(dev < 64, EXL3_ERR_UNSUPPORTED, "device index >= 64");
    int grid_max = 0;
    {
        std::lock_guard<std::mutex> lock(g_lin_mu);
        LinPrepared& pr = g_lin_prep[dev][K - 1][CB][PRECISE ? 1 : 0];
        if (!pr.ready) {
            DeviceInfo di;
            if (int rc = device_info(dev, &di)) return rc;
            const int smax = kLinHeadBytes + kLinRingBytes;
            EXL3_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
            int res = 0;
            EXL3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, kern, kLinThreads, smax));
            EXL3_REQUIRE(res > 0, EXL3_ERR_UNSUPPORTED, "linear kernel has no resident CTA");
            pr.grid = di.sms * res;
            pr.ready = true;
        }
        grid_max = pr.grid;
    }
    const int grid = units < grid_max ? units : grid_max;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned) grid);
    cfg.blockDim = dim3((unsigned) kLinThreads);
    cfg.dynamicSmemBytes = (size_t) smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    EXL3_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
    return EXL3_OK;
}

template <int K, bool PRECISE>
int launch_linear_cb(int cb, const LinearParams& p, int units, int smem, cudaStream_t s) {
    switch (cb) {
        case 0: return launch_linear<K, 0, PRECISE>(p, units, smem, s);
        case 1: return launch_linear<K, 1, PRECISE>(p, units, smem, s);
        default: return launch_linear<K, 2, PRECISE>(p, units, smem, s);
    }
}

template <bool PRECISE>
int launch_linear_k(int K, int cb, const LinearParams& p, int units, int smem, cudaStream_t s) {
    switch (K) {
        case 1: return launch_linear_cb<1, PRECISE>(cb, p, units, smem, s);
        case 2: return launch_linear_cb<2, PRECISE>(cb, p, units, smem, s);
        case 3: return launch_linear_cb<3, PRECISE>(cb, p, units, smem, s);
        case 4: return launch_linear_cb<4, PRECISE>(cb, p, units, smem, s);
        case 5: return launch_linear_cb<5, PRECISE>(cb, p, units, smem, s);
        case 6: return launch_linear_cb<6, PRECISE>(cb, p, units, smem, s);
        case 7: return launch_linear_cb<7, PRECISE>(cb, p, units, smem, s);
        default: return launch_linear_cb<8, PRECISE>(cb, p, units, smem, s);
    }
}

int launch_linear_any(int K, int cb, bool precise, const LinearParams& p, int units, int smem, cudaStream_t s) {
    return precise ? launch_linear_k<true>(K, cb, p, units, smem, s) : launch_linear_k<false>(K, cb, p, units, smem, s);
}

// k-chunks per 128-column block: among the chunk counts that divide k into
// whole 128-blocks (at most kLinMaxChunks) and keep a unit's input fragments
// (k/c x rows x fw bytes) within kLinFragBytes, the most that still fit one
// wave (a CTA per unit: no CTA runs a second unit while its block waits on
// it), else the fewest allowed.  -1 when none is allowed.
int pick_chunks(int64_t k, int64_t n, int grid, int64_t rows, int fw) {
    const int kb = (int) (k / 128);
    const int64_t nb = n / 128;
    int best = -1, fewest = -1;
    for (int c = 1; c <= kb && c <= kLinMaxChunks; ++c) {
        if (kb % c) continue;
        if ((k / c) * rows * fw > kLinFragBytes) continue;
        if (fewest < 0) fewest = c;
        if (nb * c <= (int64_t) grid) best = c;
    }
    return best > 0 ? best : fewest;
}

int assumed_grid() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    DeviceInfo di;
    if (device_info(dev, &di) != EXL3_OK || di.sms <= 0) return 296;
    return di.sms * 2;
}

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
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

template <int K, int CB>
void launch_dequant(const uint8_t* t, int64_t kt, int64_t nt, const __half* suh, const __half* svh,
                    __half* w, int full, cudaStream_t s, int sms) {
    if (full) {
        const int smem = 128 * kRecPitch * 4;
        cudaFuncSetAttribute(reconstruct_kernel<K, CB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        dim3 grid((unsigned) (nt / 8), (unsigned) (kt / 8));
        reconstruct_kernel<K, CB><<<grid, 256, smem, s>>>(t, nt, suh, svh, w);
    } else {
        int64_t blocks = (kt * nt + 7) / 8;
        if (blocks > (int64_t) sms * 16) blocks = (int64_t) sms * 16;
        decode_kernel<K, CB><<<(unsigned) blocks, 256, 0, s>>>(t, kt, nt, w);
    }
}

template <int K>
void launch_dequant_cb(int cb, const uint8_t* t, int64_t kt, int64_t nt, const __half* suh,
                       const __half* svh, __half* w, int full, cudaStream_t s, int sms) {
    switch (cb) {
        case 0: launch_dequant<K, 0>(t, kt, nt, suh, svh, w, full, s, sms); break;
        case 1: launch_dequant<K, 1>(t, kt, nt, suh, svh, w, full, s, sms); break;
        default: launch_dequant<K, 2>(t, kt, nt, suh, svh, w, full, s, sms); break;
    }
}

}  // namespace
}  // namespace exl3

using namespace exl3;

extern "C" int exl3_dequant(const void* trellis, int64_t kt, int64_t nt, int K, int cb, const void* suh,
                            const void* svh, void* w, int full, void* stream) {
    EXL3_REQUIRE(trellis && w, EXL3_ERR_ARG, "exl3_dequant: null trellis or output");
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_ARG, "exl3_dequant: K must be in 1..8 (got %d)", K);
    EXL3_REQUIRE(cb >= 0 && cb <= 2, EXL3_ERR_ARG, "exl3_dequant: codebook must be 0, 1 or 2");
    EXL3_REQUIRE(kt > 0 && nt > 0, EXL3_ERR_ARG, "exl3_dequant: trellis dimensions must be positive");
    EXL3_REQUIRE(((reinterpret_cast<uintptr_t>(trellis) & 3u) == 0), EXL3_ERR_ARG,
                 "exl3_dequant: trellis must be 4-byte aligned");
    if (full) {
        EXL3_REQUIRE(kt % 8 == 0 && nt % 8 == 0, EXL3_ERR_ARG,
                     "trellis dimensions must reconstruct whole 128-element Hadamard blocks");
        EXL3_REQUIRE(suh && svh, EXL3_ERR_ARG, "exl3_dequant: suh and svh are required when full = 1");
    }
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    DeviceInfo di;
    if (int rc = device_info(dev, &di)) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    auto t = static_cast<const uint8_t*>(trellis);
    auto su = static_cast<const __half*>(suh);
    auto sv = static_cast<const __half*>(svh);
    auto wo = static_cast<__half*>(w);
    switch (K) {
        case 1: launch_dequant_cb<1>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        case 2: launch_dequant_cb<2>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        case 3: launch_dequant_cb<3>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        case 4: launch_dequant_cb<4>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        case 5: launch_dequant_cb<5>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        case 6: launch_dequant_cb<6>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        case 7: launch_dequant_cb<7>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
        default: launch_dequant_cb<8>(cb, t, kt, nt, su, sv, wo, full, s, di.sms); break;
    }
    EXL3_CUDA(cudaGetLastError());
    return EXL3_OK;
}

// Scratch: control words and the chunk partials over all matrices' columns
// (sized for the most chunks either arithmetic can pick).
static int64_t linear_scratch_for(int64_t rows_blk, int64_t k, int64_t ntot, int grid) {
    int nk = pick_chunks(k, ntot, grid, rows_blk, 2);
    const int nk4 = pick_chunks(k, ntot, grid, rows_blk, 4);
    if (nk4 > nk) nk = nk4;
    if (nk < 1) nk = kLinMaxChunks;
    return EXL3_LINEAR_CTRL_BYTES + align_up((int64_t) nk * rows_blk * ntot * 4, 256);
}

// Scratch for `rows` rows: the tensor-core path's (>= 64 rows, one matrix at a
// time) or the GEMV path's.
static int64_t linear_group_need(int64_t rows, int64_t k, int nmat, const int64_t* n, int grid) {
    int64_t ntot = 0, tc = 0;
    bool all_tc = true;
    for (int j = 0; j < nmat; ++j) {
        ntot += n[j];
        if (linear_tc_eligible(rows, k, n[j])) {
            const int64_t b = linear_tc_scratch_bytes(rows, k, n[j]);
            tc = b > tc ? b : tc;
        } else {
            all_tc = false;
        }
    }
    if (all_tc) return tc;
    const int64_t rb = rows < kLinMaxRows ? rows : kLinMaxRows;
    const int64_t g = linear_scratch_for(rb, k, ntot, grid);
    return g > tc ? g : tc;
}

static int64_t linear_need(int64_t rows, int64_t k, int64_t n, int grid) {
    return linear_group_need(rows, k, 1, &n, grid);
}

extern "C" int64_t exl3_linear_scratch_bytes(int64_t rows, int64_t k, int64_t n, int K) {
    if (rows < 1 || k < 128 || n < 128 || K < 1 || K > 8) return -1;
    return linear_need(rows, k, n, assumed_grid());
}

extern "C" int64_t exl3_linear_group_scratch_bytes(int64_t rows, int64_t k, int nmat, const int64_t* n, int K) {
    if (rows < 1 || k < 128 || nmat < 1 || nmat > kLinMaxMats || !n || K < 1 || K > 8) return -1;
    for (int j = 0; j < nmat; ++j)
        if (n[j] < 128) return -1;
    return linear_group_need(rows, k, nmat, n, assumed_grid());
}

namespace exl3 {
namespace {

// The GEMV engine over a group of nmat matrices sharing x (checked by the
// callers): one launch per block of 32 rows.  Matrices that the tensor-core
// path takes (>= 64 rows) run one after another on it instead.
int linear_group_impl(const char* who, const void* x, int x_dtype, int64_t rows, int64_t k, int nmat,
                      const int64_t* n, const void* const* trellis, int K, int cb, const void* const* suh,
                      const void* const* svh, void* const* y, int y_dtype, void* scratch, int64_t scratch_bytes,
                      int precise, void* stream) {
    EXL3_REQUIRE(x && scratch && n && trellis && suh && svh && y, EXL3_ERR_ARG, "%s: null pointer argument", who);
    EXL3_REQUIRE(nmat >= 1 && nmat <= kLinMaxMats, EXL3_ERR_ARG, "%s: 1 to %d matrices (got %d)", who, kLinMaxMats,
                 nmat);
    EXL3_REQUIRE(rows >= 1, EXL3_ERR_ARG, "%s: rows must be >= 1", who);
    EXL3_REQUIRE(k % 128 == 0 && k > 0, EXL3_ERR_ARG, "%s: k and n must be positive multiples of 128 (k = %lld)",
                 who, (long long) k);
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_ARG, "%s: K must be in 1..8 (got %d)", who, K);
    EXL3_REQUIRE(cb >= 0 && cb <= 2, EXL3_ERR_ARG, "%s: codebook must be 0, 1 or 2", who);
    EXL3_REQUIRE(x_dtype >= 0 && x_dtype <= 2 && y_dtype >= 0 && y_dtype <= 2, EXL3_ERR_ARG,
                 "%s: dtype codes are 0 (fp16), 1 (bf16), 2 (fp32)", who);
    EXL3_REQUIRE(aligned16(scratch), EXL3_ERR_ARG, "%s: scratch must be 16-byte aligned", who);
    int64_t ntot = 0;
    for (int j = 0; j < nmat; ++j) {
        EXL3_REQUIRE(trellis[j] && suh[j] && svh[j] && y[j], EXL3_ERR_ARG, "%s: null pointer for matrix %d", who, j);
        EXL3_REQUIRE(n[j] % 128 == 0 && n[j] > 0, EXL3_ERR_ARG,
                     "%s: k and n must be positive multiples of 128 (matrix %d: n = %lld)", who, j, (long long) n[j]);
        EXL3_REQUIRE(aligned16(trellis[j]), EXL3_ERR_ARG, "%s: trellis must be 16-byte aligned", who);
        ntot += n[j];
    }
    EXL3_REQUIRE(ntot / 128 + kLinOffCnt <= EXL3_LINEAR_CTRL_BYTES / 4, EXL3_ERR_UNSUPPORTED, "%s: n too large", who);
    const int grid = assumed_grid();
    const int64_t rb = rows < kLinMaxRows ? rows : kLinMaxRows;
    const int64_t need = linear_group_need(rows, k, nmat, n, grid);
    EXL3_REQUIRE(scratch_bytes >= need, EXL3_ERR_ARG, "%s: scratch too small (%lld < %lld bytes)", who,
                 (long long) scratch_bytes, (long long) need);
    auto s = static_cast<cudaStream_t>(stream);
    // matrices for the tensor-core path, one launch sequence each
    int gm = 0;
    int64_t gn[kLinMaxMats];
    const void* gt[kLinMaxMats];
    const void* gsu[kLinMaxMats];
    const void* gsv[kLinMaxMats];
    void* gy[kLinMaxMats];
    for (int j = 0; j < nmat; ++j) {
        if (linear_tc_eligible(rows, k, n[j])) {
            if (int rc = linear_tc(x, x_dtype, rows, k, n[j], trellis[j], K, cb, suh[j], svh[j], y[j], y_dtype, scratch,
                                   s))
                return rc;
        } else {
            gn[gm] = n[j]; gt[gm] = trellis[j]; gsu[gm] = suh[j]; gsv[gm] = svh[j]; gy[gm] = y[j];
            ++gm;
        }
    }
    if (gm == 0) return EXL3_OK;
    auto encode = tmap_encoder();
    EXL3_REQUIRE(encode != nullptr, EXL3_ERR_CUDA, "%s: cuTensorMapEncodeTiled is not available", who);

    LinearParams p{};
    shift_table_init(p.ring.st);
    int64_t gtot = 0;
    for (int j = 0; j < gm; ++j) {
        const cuuint64_t dims[3] = {(cuuint64_t) (16 * K), (cuuint64_t) (gn[j] / 16), (cuuint64_t) (k / 16)};
        const cuuint64_t strides[2] = {(cuuint64_t) (32 * K), (cuuint64_t) (gn[j] / 16) * (cuuint64_t) (32 * K)};
        const cuuint32_t box[3] = {(cuuint32_t) (16 * K), 8u, (cuuint32_t) kStageSK};
        const cuuint32_t estr[3] = {1u, 1u, 1u};
        const CUresult r = encode(&p.tmap[j], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(gt[j]), dims,
                                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", who, (int) r);
        p.n[j] = (int) gn[j];
        p.blk0[j] = (int) (gtot / kCols);
        p.suh[j] = static_cast<const __half*>(gsu[j]);
        p.svh[j] = static_cast<const __half*>(gsv[j]);
        gtot += gn[j];
    }
    p.blk0[gm] = (int) (gtot / kCols);
    p.nmat = gm;
    p.ntot = (int) gtot;
    p.k = (int) k;
    p.x_dtype = x_dtype;
    p.y_dtype = y_dtype;
    const int fw = precise ? 2 : 4;
    p.nk = pick_chunks(k, gtot, grid, rb, fw);
    EXL3_REQUIRE(p.nk >= 1, EXL3_ERR_UNSUPPORTED, "%s: k = %lld has no k-chunk small enough for %lld rows", who,
                 (long long) k, (long long) rb);
    p.kc = (int) (k / p.nk);
    uint8_t* sb = static_cast<uint8_t*>(scratch);
    p.ctrl = reinterpret_cast<uint32_t*>(sb);
    p.partial = reinterpret_cast<float*>(sb + EXL3_LINEAR_CTRL_BYTES);
    const int esz_x = x_dtype == 2 ? 4 : 2, esz_y = y_dtype == 2 ? 4 : 2;
    const int64_t units = (gtot / kCols) * p.nk;
    for (int64_t r0 = 0; r0 < rows; r0 += kLinMaxRows) {
        p.rows = (int) ((rows - r0) < kLinMaxRows ? (rows - r0) : kLinMaxRows);
        p.ring.wpart = kStageSK * 8 * 32 * K;
        p.ring.slot_bytes = p.ring.wpart;
        const int xbytes = p.kc * p.rows * fw;          // the unit's input fragments
        const int budget = kLinRingBytes - 2 * p.rows * kCols * 4 - xbytes;
        const int nsl = budget / p.ring.slot_bytes;
        p.ring.ns = nsl < 2 ? 2 : (nsl > kLinMaxStages ? kLinMaxStages : nsl);
        const int smem = kLinHeadBytes + p.ring.ns * p.ring.slot_bytes + 2 * p.rows * kCols * 4 + xbytes;
        EXL3_REQUIRE(smem <= kLinHeadBytes + kLinRingBytes, EXL3_ERR_UNSUPPORTED, "%s: stage too large", who);
        p.x = static_cast<const uint8_t*>(x) + r0 * k * esz_x;
        for (int j = 0; j < gm; ++j) p.y[j] = static_cast<uint8_t*>(gy[j]) + r0 * gn[j] * esz_y;
        if (int rc = launch_linear_any(K, cb, precise != 0, p, (int) units, smem, s)) return rc;
    }
    return EXL3_OK;
}

}  // namespace
}  // namespace exl3

#ifdef EXL3_PHASE_CLOCK
extern "C" int exl3_linear_timeline_read(unsigned long long* out, int n) {
    EXL3_REQUIRE(out && n >= 1 && n <= 512 * 8, EXL3_ERR_ARG, "linear timeline: bad output");
    EXL3_CUDA(cudaDeviceSynchronize());
    EXL3_CUDA(cudaMemcpyFromSymbol(out, exl3::g_ltl, sizeof(unsigned long long) * n));
    return EXL3_OK;
}
#endif

extern "C" int exl3_linear(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t n, const void* trellis,
                           int K, int cb, const void* suh, const void* svh, void* y, int y_dtype, void* scratch,
                           int64_t scratch_bytes, int precise, void* stream) {
    EXL3_REQUIRE(x && trellis && suh && svh && y && scratch, EXL3_ERR_ARG, "exl3_linear: null pointer argument");
    EXL3_REQUIRE(n % 128 == 0 && n > 0, EXL3_ERR_ARG, "exl3_linear: k and n must be positive multiples of 128 (got %lld, %lld)",
                 (long long) k, (long long) n);
    return linear_group_impl("exl3_linear", x, x_dtype, rows, k, 1, &n, &trellis, K, cb, &suh, &svh, &y, y_dtype,
                             scratch, scratch_bytes, precise, stream);
}

extern "C" int exl3_linear_group(const void* x, int x_dtype, int64_t rows, int64_t k, int nmat, const int64_t* n,
                                 const void* const* trellis, int K, int cb, const void* const* suh,
                                 const void* const* svh, void* const* y, int y_dtype, void* scratch,
                                 int64_t scratch_bytes, int precise, void* stream) {
    return linear_group_impl("exl3_linear_group", x, x_dtype, rows, k, nmat, n, trellis, K, cb, suh, svh, y, y_dtype,
                             scratch, scratch_bytes, precise, stream);
}

