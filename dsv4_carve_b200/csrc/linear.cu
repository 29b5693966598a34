// linear.cu -- dense EXL3 linear (GEMV form) and trellis dequant for sm_100a.
//
// exl3_linear: y = x . W for small row counts, the dense 6-bit path of the
// attention / shared-expert linears (reference: LinearEXL3.forward ->
// BC_LinearEXL3.run_alloc -> exl3_gemm_gr, recipe-lna/exllamav3/exl3.py.lna:114-139,
// recipe-lna/exllamav3/exl3_gemm.cu.lna:123-334).  Same arithmetic boundaries
// as the reference: input fp16(x) * suh in fp16, 128-block Hadamard in fp32
// rounded to fp16, fp32 accumulation, output Hadamard and svh in fp32, one
// cast to the output dtype.
#include <mutex>

#include "engine.cuh"
#include "host.hpp"

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
struct LinearParams {
    const void* x;
    int x_dtype;
    int rows;            // <= kMaxRows
    int64_t k, n;
    const uint8_t* trellis;
    const __half* suh;
    const __half* svh;
    void* y;
    int y_dtype;
    int kc;              // k-chunk per unit (multiple of 128 and of the stage depth)
    int nchunks;         // k / kc
    float* partial;      // [nchunks][rows][n]
    uint32_t* colcnt;    // [n/128]
    uint32_t* ctrl;      // [0] ticket, [1] retire, [2] status
};

template <int K> struct LinCfg {
    static constexpr int SK = stage_slices(K);
    static constexpr int STAGE = SK * 8 * TileFmt<K>::BYTES;
    static constexpr int NS = (49152 / STAGE) > 8 ? 8 : (49152 / STAGE);
};

template <int K>
struct alignas(128) LinSmem {
    uint8_t ring[LinCfg<K>::NS][LinCfg<K>::STAGE];
    uint4 bfrag[kActBytes / 16];
    float cbuf[kMaxRows * kCols];
    uint64_t full[LinCfg<K>::NS];
    uint64_t empty[LinCfg<K>::NS];
    uint64_t dqf[kDQ];
    uint64_t dqe[kDQ];
    int desc[kDQ][2];
    int rows[kMaxRows];
    int flag;
};

template <int K, int CB, int RB, bool PRECISE>
__device__ __forceinline__ bool lin_consume(LinSmem<K>& S, uint32_t& it, int nst, float (&acc)[4][4],
                                            const LaneGeom<K>& geom, int cwarp, int lane, uint32_t* status) {
    return consume_stages<K, CB, RB, LinCfg<K>::NS, LinCfg<K>::STAGE, LinCfg<K>::SK, PRECISE>(
        S.ring, S.full, S.empty, it, nst, 0, S.bfrag, acc, geom, cwarp, lane, status);
}

template <int K, int CB, bool PRECISE>
__global__ void __launch_bounds__(kThreads, 2) linear_kernel(LinearParams p) {
    using C = LinCfg<K>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    LinSmem<K>& S = *reinterpret_cast<LinSmem<K>*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* status = p.ctrl + 2;

    if (tid == 0) {
        for (int s = 0; s < C::NS; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], kConsumerWarps); }
        for (int s = 0; s < kDQ; ++s) { mbar_init(&S.dqf[s], 1); mbar_init(&S.dqe[s], 1); }
        fence_barrier_init();
    }
    if (tid < kMaxRows) S.rows[tid] = tid;
    __syncthreads();

    const int nbn = (int) (p.n / kCols);
    const int total = nbn * p.nchunks;
    const int kslices = p.kc / 16;
    const int nst = kslices / C::SK;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------- producer
        const int rowbytes = 8 * TileFmt<K>::BYTES;
        const int64_t rowstride = (p.n / 16) * TileFmt<K>::BYTES;
        int ticket = claim_ticket(&p.ctrl[0], lane);
        uint32_t it = 0, du = 0;
        bool ok = true;
        while (ok) {
            const bool end = ticket >= total;
            const int j = end ? -1 : ticket / p.nchunks;
            const int s = end ? -1 : ticket % p.nchunks;
            if (lane == 0) {
                const int slot = du % kDQ;
                ok = mbar_wait(&S.dqe[slot], ((du / kDQ) + 1u) & 1u, status);
                if (ok) {
                    S.desc[slot][0] = j;
                    S.desc[slot][1] = s;
                    mbar_arrive(&S.dqf[slot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            ++du;
            if (end || !ok) break;
            const uint8_t* src = p.trellis + (int64_t) s * kslices * rowstride + (int64_t) j * rowbytes;
            const bool valid = aligned16_dev(src) && (rowstride & 15) == 0;
            if (!valid && lane == 0) set_error(status, ERR_MISALIGNED);
            for (int st = 0; st < nst && ok; ++st)
                ok = produce_stage<C::NS, C::STAGE>(S.ring, S.full, S.empty, it, src + (int64_t) st * C::SK * rowstride,
                                                    rowstride, rowbytes, C::SK, valid, lane, status);
            ticket = claim_ticket(&p.ctrl[0], lane);
        }
        drain_ring<C::NS>(S.full, it, lane, status);
    } else {
        // ---------------------------------------------------------- consumers
        const int ctid = tid;
        const LaneGeom<K> geom = lane_geom<K>(lane);
        const int RB = row_blocks(p.rows);
        const int sub = (act_slices(RB) / 16) * 16 < kslices ? (act_slices(RB) / 16) * 16 : kslices;
        uint32_t it = 0, du = 0;
        while (true) {
            const int slot = du % kDQ;
            if (!consumers_all(mbar_wait_warp(&S.dqf[slot], (du / kDQ) & 1u, status, lane))) break;
            const int j = S.desc[slot][0], s = S.desc[slot][1];
            consumers_sync();
            if (ctid == 0) mbar_arrive(&S.dqe[slot]);
            ++du;
            if (j < 0) break;

            float acc[4][4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
            bool ok = true;
            for (int ks0 = 0; ks0 < kslices && ok; ks0 += sub) {
                const int nks = min(sub, kslices - ks0);
                if (ks0 > 0) consumers_sync();
                build_bfrag<PRECISE>(S.bfrag, RB, p.rows, S.rows, p.x, p.x_dtype, p.k, s * kslices + ks0, nks,
                                     p.suh, warp, lane);
                consumers_sync();
                const int n_st = nks / C::SK;
                switch (RB) {
                    case 1: ok = lin_consume<K, CB, 1, PRECISE>(S, it, n_st, acc, geom, warp, lane, status); break;
                    case 2: ok = lin_consume<K, CB, 2, PRECISE>(S, it, n_st, acc, geom, warp, lane, status); break;
                    case 3: ok = lin_consume<K, CB, 3, PRECISE>(S, it, n_st, acc, geom, warp, lane, status); break;
                    default: ok = lin_consume<K, CB, 4, PRECISE>(S, it, n_st, acc, geom, warp, lane, status); break;
                }
                ok = consumers_all(ok);
            }
            if (!consumers_all(ok)) break;
            acc_to_cbuf(S.cbuf, acc, RB, warp, lane);
            consumers_sync();

            bool finalize = true;
            if (p.nchunks > 1) {
                const int64_t col0 = (int64_t) j * kCols;
                for (int idx = ctid; idx < p.rows * kCols; idx += kConsumerThreads) {
                    const int r = idx / kCols, c = idx % kCols;
                    p.partial[((int64_t) s * p.rows + r) * p.n + col0 + c] = S.cbuf[idx];
                }
                consumers_sync();
                if (ctid == 0) {
                    __threadfence();   // release: covers every consumer's writes (ordered by the barrier)
                    const uint32_t old = atomicAdd(&p.colcnt[j], 1u);
                    const int last = old == (uint32_t) (p.nchunks - 1);
                    if (last) {
                        atomicExch(&p.colcnt[j], 0u);
                        __threadfence();   // acquire: the other chunks' partials
                    }
                    S.flag = last;
                }
                consumers_sync();
                finalize = S.flag != 0;
                if (finalize) {
                    for (int idx = ctid; idx < p.rows * kCols; idx += kConsumerThreads) {
                        const int r = idx / kCols, c = idx % kCols;
                        float v = 0.f;
                        for (int c2 = 0; c2 < p.nchunks; ++c2)
                            v += __ldcg(&p.partial[((int64_t) c2 * p.rows + r) * p.n + col0 + c]);
                        S.cbuf[idx] = v;
                    }
                    consumers_sync();
                }
            }
            if (finalize) {
                for (int r = warp; r < p.rows; r += kConsumerWarps) {
                    float v[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) v[q] = S.cbuf[r * kCols + lane * 4 + q];
                    out_transform(v, p.svh + (int64_t) j * kCols, lane);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        store_out(p.y, p.y_dtype, (int64_t) r * p.n + (int64_t) j * kCols + lane * 4 + q, v[q]);
                }
            }
            consumers_sync();
        }
    }

    // Retire: the last CTA out restores the ticket counters for the next launch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&p.ctrl[1], 1u);
        if (old == gridDim.x - 1) {
            atomicExch(&p.ctrl[0], 0u);
            atomicExch(&p.ctrl[1], 0u);
        }
    }
}

// ------------------------------------------------------------------ host side
namespace {

template <int K, int CB, bool PRECISE>
int launch_linear(const LinearParams& p, int grid, cudaStream_t stream) {
    auto kern = linear_kernel<K, CB, PRECISE>;
    const int smem = (int) sizeof(LinSmem<K>);
    static std::once_flag once[64];
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    cudaError_t attr = cudaSuccess;
    std::call_once(once[dev & 63], [&] {
        attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    EXL3_CUDA(attr);
    kern<<<grid, kThreads, smem, stream>>>(p);
    EXL3_CUDA(cudaGetLastError());
    return EXL3_OK;
}

template <int K, bool PRECISE>
int launch_linear_cb(int cb, const LinearParams& p, int grid, cudaStream_t s) {
    switch (cb) {
        case 0: return launch_linear<K, 0, PRECISE>(p, grid, s);
        case 1: return launch_linear<K, 1, PRECISE>(p, grid, s);
        default: return launch_linear<K, 2, PRECISE>(p, grid, s);
    }
}

template <bool PRECISE>
int launch_linear_k(int K, int cb, const LinearParams& p, int grid, cudaStream_t s) {
    switch (K) {
        case 1: return launch_linear_cb<1, PRECISE>(cb, p, grid, s);
        case 2: return launch_linear_cb<2, PRECISE>(cb, p, grid, s);
        case 3: return launch_linear_cb<3, PRECISE>(cb, p, grid, s);
        case 4: return launch_linear_cb<4, PRECISE>(cb, p, grid, s);
        case 5: return launch_linear_cb<5, PRECISE>(cb, p, grid, s);
        case 6: return launch_linear_cb<6, PRECISE>(cb, p, grid, s);
        case 7: return launch_linear_cb<7, PRECISE>(cb, p, grid, s);
        default: return launch_linear_cb<8, PRECISE>(cb, p, grid, s);
    }
}

int launch_linear_any(int K, int cb, bool precise, const LinearParams& p, int grid, cudaStream_t s) {
    return precise ? launch_linear_k<true>(K, cb, p, grid, s) : launch_linear_k<false>(K, cb, p, grid, s);
}

int stage_k(int K) { return stage_slices(K) * 16; }

// k-chunk: a multiple of 128 and of the stage depth that divides k, chosen so
// the unit count fills the grid about twice, between 256 and 1024 elements.
int pick_kc(int64_t k, int64_t n, int K, int grid) {
    const int64_t nbn = n / kCols;
    const int step = stage_k(K) > 128 ? stage_k(K) : 128;
    int best = -1;
    for (int64_t kc = step; kc <= k; kc += step) {
        if (k % kc) continue;
        if (best < 0) best = (int) kc;
        if (kc > 1024) break;
        if (nbn * (k / kc) >= 2 * grid || kc <= 256) best = (int) kc;
    }
    return best < 0 ? (int) k : best;
}

int64_t linear_chunks(int64_t k, int64_t n, int K, int grid) { return k / pick_kc(k, n, K, grid); }

int grid_for(int device) {
    DeviceInfo di;
    if (device_info(device, &di) != EXL3_OK) return 0;
    return di.sms * 2;
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

static int64_t linear_scratch_for(int64_t rows_blk, int64_t k, int64_t n, int K, int grid) {
    const int64_t chunks = linear_chunks(k, n, K, grid);
    const int64_t part = chunks > 1 ? chunks * rows_blk * n * 4 : 0;
    return EXL3_LINEAR_CTRL_BYTES + align_up(part, 256);
}

extern "C" int64_t exl3_linear_scratch_bytes(int64_t rows, int64_t k, int64_t n, int K) {
    if (rows < 1 || k < 128 || n < 128 || K < 1 || K > 8) return -1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    int grid = grid_for(dev);
    if (grid <= 0) grid = 296;
    const int64_t rb = rows < kMaxRows ? rows : kMaxRows;
    return linear_scratch_for(rb, k, n, K, grid);
}

extern "C" int exl3_linear(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t n, const void* trellis,
                           int K, int cb, const void* suh, const void* svh, void* y, int y_dtype, void* scratch,
                           int64_t scratch_bytes, int precise, void* stream) {
    EXL3_REQUIRE(x && trellis && suh && svh && y && scratch, EXL3_ERR_ARG, "exl3_linear: null pointer argument");
    EXL3_REQUIRE(rows >= 1, EXL3_ERR_ARG, "exl3_linear: rows must be >= 1");
    EXL3_REQUIRE(k % 128 == 0 && n % 128 == 0 && k > 0 && n > 0, EXL3_ERR_ARG,
                 "exl3_linear: k and n must be positive multiples of 128 (got %lld, %lld)", (long long) k,
                 (long long) n);
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_ARG, "exl3_linear: K must be in 1..8 (got %d)", K);
    EXL3_REQUIRE(cb >= 0 && cb <= 2, EXL3_ERR_ARG, "exl3_linear: codebook must be 0, 1 or 2");
    EXL3_REQUIRE(x_dtype >= 0 && x_dtype <= 2 && y_dtype >= 0 && y_dtype <= 2, EXL3_ERR_ARG,
                 "exl3_linear: dtype codes are 0 (fp16), 1 (bf16), 2 (fp32)");
    EXL3_REQUIRE(aligned16(trellis), EXL3_ERR_ARG, "exl3_linear: trellis must be 16-byte aligned");
    EXL3_REQUIRE(aligned16(scratch), EXL3_ERR_ARG, "exl3_linear: scratch must be 16-byte aligned");
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    const int grid_max = grid_for(dev);
    EXL3_REQUIRE(grid_max > 0, EXL3_ERR_CUDA, "exl3_linear: cannot query the device");
    const int64_t rb = rows < kMaxRows ? rows : kMaxRows;
    const int64_t need = linear_scratch_for(rb, k, n, K, grid_max);
    EXL3_REQUIRE(scratch_bytes >= need, EXL3_ERR_ARG, "exl3_linear: scratch too small (%lld < %lld bytes)",
                 (long long) scratch_bytes, (long long) need);
    EXL3_REQUIRE(n / 128 + 16 <= EXL3_LINEAR_CTRL_BYTES / 4, EXL3_ERR_UNSUPPORTED, "exl3_linear: n too large");

    LinearParams p{};
    p.k = k;
    p.n = n;
    p.trellis = static_cast<const uint8_t*>(trellis);
    p.suh = static_cast<const __half*>(suh);
    p.svh = static_cast<const __half*>(svh);
    p.x_dtype = x_dtype;
    p.y_dtype = y_dtype;
    p.kc = pick_kc(k, n, K, grid_max);
    p.nchunks = (int) (k / p.kc);
    EXL3_REQUIRE(p.kc % (stage_slices(K) * 16) == 0 && p.kc % 128 == 0 && k % p.kc == 0, EXL3_ERR_UNSUPPORTED,
                 "exl3_linear: internal k-chunk %d does not tile k = %lld", p.kc, (long long) k);
    uint8_t* sb = static_cast<uint8_t*>(scratch);
    p.ctrl = reinterpret_cast<uint32_t*>(sb);
    p.colcnt = reinterpret_cast<uint32_t*>(sb) + 16;
    p.partial = reinterpret_cast<float*>(sb + EXL3_LINEAR_CTRL_BYTES);
    const int esz_x = x_dtype == 2 ? 4 : 2, esz_y = y_dtype == 2 ? 4 : 2;
    const int64_t units = (n / kCols) * p.nchunks;
    const int grid = (int) (units < grid_max ? units : grid_max);
    auto s = static_cast<cudaStream_t>(stream);
    for (int64_t r0 = 0; r0 < rows; r0 += kMaxRows) {
        p.rows = (int) ((rows - r0) < kMaxRows ? (rows - r0) : kMaxRows);
        p.x = static_cast<const uint8_t*>(x) + r0 * k * esz_x;
        p.y = static_cast<uint8_t*>(y) + r0 * n * esz_y;
        if (int rc = launch_linear_any(K, cb, precise != 0, p, grid, s)) return rc;
    }
    return EXL3_OK;
}
