// tc.cu -- tensor-core (tcgen05) path of the dense EXL3 linear for >= 64 rows
// (prefill chunks), where y = x . W is a real contraction.  Reference: the
// prefill branch of LinearEXL3.forward, reconstruct + hgemm
// (recipe-lna/exllamav3/exl3.py.lna:161-218), and the M16 panel GEMM of
// exl3_gemm_kernel (orders/F1-ref/exl3_gemm_kernel.cuh:8-80).
//
// Dequant-then-MMA, one CTA per 128-row x 128-column output tile over the
// whole k:
//   warp 8 (producer)  TMA: per k-step of 128, the 8 k-slices x 8 tiles of
//                      packed weights (3-D box) into a 3-stage ring, and the
//                      transformed activations (two 128-row x 64-element
//                      boxes, 128-byte swizzle) into a double-buffered A tile;
//   warps 0-7          decode n-tile w of every k-slice in registers, round
//                      each weight to fp16 (the reference decoder's value) and
//                      write it into the double-buffered B tile, K-major with
//                      the 128-byte swizzle the MMA descriptor names;
//   warp 9             allocates 128 TMEM columns; lane 0 issues
//                      tcgen05.mma (M 128, N 128, K 16, fp16 in, fp32 out) and
//                      commits each k-step to the mbarrier that frees its A/B
//                      buffers;
//   epilogue           warps 0-3 read the accumulator (tcgen05.ld, one row per
//                      thread) into shared memory; warps 0-7 apply the output
//                      transform (Hadamard * svh) per row and store y.
// The input transform (x -> fp16, * suh, Hadamard -> fp16, row-major) runs as
// a separate small kernel first.  Every wait is bounded; TMEM is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "engine.cuh"
#include "host.hpp"

namespace exl3 {

constexpr int kTcThreads = 320;
constexpr int kTcTile = 128;                       // M and N of the CTA tile
constexpr int kTcKStep = 128;                      // k per pipeline step (8 k-slices)
constexpr int kTcAtom = 128 * 128;                 // 128 rows x 64 fp16 (128-byte rows), one swizzle block
constexpr int kTcAB = 2 * kTcAtom;                 // one A or B buffer: 128 x 128 fp16 = 32 KB
constexpr int kTcWStages = 3;
constexpr int kTcWStageMax = 8 * 8 * 32 * 8;       // 8 k-slices x 8 tiles x 32K bytes at K = 8
constexpr int kTcDPitch = kTcTile + 1;             // fp32 staging pitch of the accumulator
constexpr int kTcMinRows = 64;

struct TcHead {
    uint64_t wfull[kTcWStages];
    uint64_t wempty[kTcWStages];
    uint64_t afull[2];
    uint64_t bready[2];
    uint64_t bfree[2];
    uint64_t done;
    uint32_t tmem;
};
constexpr int kTcSmem = 1024 /* alignment slack */ + 4 * kTcAB + kTcWStages * kTcWStageMax + 256;

struct TcParams {
    CUtensorMap wmap;      // trellis [k/16][n/16][16K] u16, box [16K, 8, 8]
    CUtensorMap amap;      // transformed x [M][k] fp16, box [64, 128], 128-byte swizzle
    int M, k, n;
    const __half* svh;
    void* y;
    int y_dtype;
    uint32_t* status;
};

// ------------------------------------------------------------------ tcgen05 wrappers
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle (8-row groups
// 1024 bytes apart), start address at `addr`.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr) {
    return (uint64_t) ((addr & 0x3FFFFu) >> 4)          // start address
         | ((uint64_t) 1 << 16)                          // leading byte offset (unused for swizzled K-major)
         | ((uint64_t) (1024 >> 4) << 32)                // stride byte offset: 8 rows x 128 B
         | ((uint64_t) 1 << 46)                          // descriptor version
         | ((uint64_t) 2 << 61);                         // 128-byte swizzle
}

// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(dtmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (row, k) of a 128-row, 128-k K-major tile made of two
// 64-element swizzle blocks: 16-byte chunk index XOR (row mod 8).
__device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
    const int atom = k >> 6, col = k & 63;
    return (uint32_t) (atom * kTcAtom + row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

// ------------------------------------------------------------------ input transform
// xt[r][k] = fp16( H128( fp16(x[r][k]) * suh[k] ) / sqrt(128) ), one warp per
// (row, 128-block) (recipe-lna/lna2/lna_moe_ticket.cu:119-144).
__global__ void __launch_bounds__(256) input_transform_kernel(const void* x, int x_dtype, int M, int k,
                                                              const __half* suh, __half* xt) {
    const int lane = threadIdx.x & 31;
    const int kb_count = k / 128;
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= M * kb_count) return;
    const int r = item / kb_count, kb = item % kb_count;
    const int64_t k0 = (int64_t) kb * 128 + lane * 4;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const __half a = load_act_half(x, x_dtype, (int64_t) r * k + k0 + q);
        v[q] = __half2float(__hmul(a, suh[k0 + q]));
    }
    wht128_warp(v, lane);
    __half2 h0 = __floats2half2_rn(v[0] * kHadNorm, v[1] * kHadNorm);
    __half2 h1 = __floats2half2_rn(v[2] * kHadNorm, v[3] * kHadNorm);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(xt + (int64_t) r * k + k0) = o;
}

// ------------------------------------------------------------------ GEMM
template <int K, int CB>
__global__ void __launch_bounds__(kTcThreads, 1) linear_tc_kernel(const __grid_constant__ TcParams p) {
    using F = TileFmt<K>;
    extern __shared__ uint8_t tc_raw[];
    uint8_t* base = tc_raw + ((1024u - (smem_u32(tc_raw) & 1023u)) & 1023u);
    uint8_t* Abuf = base;                              // [2][32 KB]
    uint8_t* Bbuf = base + 2 * kTcAB;                  // [2][32 KB]
    uint8_t* Wring = base + 4 * kTcAB;                 // [3][16 KB]
    TcHead& H = *reinterpret_cast<TcHead*>(Wring + kTcWStages * kTcWStageMax);
    float* Dst = reinterpret_cast<float*>(base);       // accumulator staging [128][129], after the last MMA
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = blockIdx.x, mb = blockIdx.y;
    const int KS = p.k / kTcKStep;
    uint32_t* status = p.status;

    if (tid == 0) {
        for (int s = 0; s < kTcWStages; ++s) { mbar_init(&H.wfull[s], 1); mbar_init(&H.wempty[s], 8); }
        for (int s = 0; s < 2; ++s) { mbar_init(&H.afull[s], 1); mbar_init(&H.bready[s], 8); mbar_init(&H.bfree[s], 1); }
        mbar_init(&H.done, 1);
        fence_barrier_init();
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&H.tmem)), "r"(kTcTile) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = H.tmem;

    if (warp == 8) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t wbytes = (uint32_t) (8 * 8 * 32 * K);
            uint32_t issued_w = 0, issued_a = 0;
            bool ok = true;
            for (int s = 0; s < KS && ok; ++s) {
                const int ws = s % kTcWStages, ab = s & 1;
                ok = mbar_wait(&H.wempty[ws], ((s / kTcWStages) + 1u) & 1u, status);
                if (!ok) break;
                mbar_arrive_expect_tx(&H.wfull[ws], wbytes);
                tma_load_3d(Wring + ws * kTcWStageMax, &p.wmap, 0, nb * 8, s * 8, &H.wfull[ws]);
                ++issued_w;
                ok = mbar_wait(&H.bfree[ab], ((s >> 1) + 1u) & 1u, status);
                if (!ok) break;
                mbar_arrive_expect_tx(&H.afull[ab], (uint32_t) kTcAB);
                tma_load_2d(Abuf + ab * kTcAB, &p.amap, s * kTcKStep, mb * kTcTile, &H.afull[ab]);
                tma_load_2d(Abuf + ab * kTcAB + kTcAtom, &p.amap, s * kTcKStep + 64, mb * kTcTile, &H.afull[ab]);
                ++issued_a;
            }
            // no copy may still be in flight when the CTA retires
            for (uint32_t i = issued_w > kTcWStages ? issued_w - kTcWStages : 0; i < issued_w; ++i)
                if (!mbar_wait(&H.wfull[i % kTcWStages], (i / kTcWStages) & 1u, status)) break;
            for (uint32_t i = issued_a > 2 ? issued_a - 2 : 0; i < issued_a; ++i)
                if (!mbar_wait(&H.afull[i & 1], (i >> 1) & 1u, status)) break;
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kTcTile, kTcTile);
            bool ok = true;
            for (int s = 0; s < KS && ok; ++s) {
                const int ab = s & 1;
                ok = mbar_wait(&H.afull[ab], (s >> 1) & 1u, status) && mbar_wait(&H.bready[ab], (s >> 1) & 1u, status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(Abuf + ab * kTcAB), b0 = smem_u32(Bbuf + ab * kTcAB);
#pragma unroll
                for (int kk = 0; kk < kTcKStep / 16; ++kk) {
                    const uint32_t off = (uint32_t) ((kk >> 2) * kTcAtom + (kk & 3) * 32);
                    tc_mma(tmem, sdesc_sw128(a0 + off), sdesc_sw128(b0 + off), idesc, (s | kk) != 0);
                }
                tc_commit(&H.bfree[ab]);
            }
            tc_commit(&H.done);
        }
    } else {
        // ------------------------------------------------------------ decoders
        const LaneGeom<K> geom = lane_geom<K>(lane);
        const int t4 = lane & 3, g = lane >> 2;
        const int n0 = warp * 16 + g;                  // this lane's output columns n0 and n0 + 8
        for (int s = 0; s < KS; ++s) {
            const int ws = s % kTcWStages, ab = s & 1;
            if (!mbar_wait_lanes(&H.wfull[ws], (s / kTcWStages) & 1u, status)) break;
            if (!mbar_wait_lanes(&H.bfree[ab], ((s >> 1) + 1u) & 1u, status)) break;
            const uint32_t* wst = reinterpret_cast<const uint32_t*>(Wring + ws * kTcWStageMax);
            uint8_t* B = Bbuf + ab * kTcAB;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t* t = wst + (i * 8 + warp) * F::WORDS;
                uint32_t w[8], x[8];
                tile_windows<K>(t, geom, w);
#pragma unroll
                for (int j = 0; j < 8; ++j) x[j] = codebook_pair<CB>(w[j]);
                const int kk = i * 16 + 2 * t4;
                *reinterpret_cast<uint32_t*>(B + sw128_offset(n0, kk)) = round_pair(x[0], x[1]);
                *reinterpret_cast<uint32_t*>(B + sw128_offset(n0, kk + 8)) = round_pair(x[2], x[3]);
                *reinterpret_cast<uint32_t*>(B + sw128_offset(n0 + 8, kk)) = round_pair(x[4], x[5]);
                *reinterpret_cast<uint32_t*>(B + sw128_offset(n0 + 8, kk + 8)) = round_pair(x[6], x[7]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor core reads
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&H.bready[ab]);
                mbar_arrive(&H.wempty[ws]);
            }
        }
    }

    // ---------------------------------------------------------------- epilogue
    __syncthreads();
    if (warp < 4) {
        mbar_wait_lanes(&H.done, 0u, status);
        tc_fence_after();
        const int row = warp * 32 + lane;
        for (int c0 = 0; c0 < kTcTile; c0 += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t) (warp * 32) << 16) + (uint32_t) c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) Dst[row * kTcDPitch + c0 + i] = v[i];
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kTcTile) : "memory");
    }
    if (warp < 8) {
        for (int r = warp; r < kTcTile; r += 8) {
            const int64_t grow = (int64_t) mb * kTcTile + r;
            if (grow >= p.M) break;
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = Dst[r * kTcDPitch + lane * 4 + q];
            out_transform(v, p.svh + (int64_t) nb * kTcTile, lane);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                store_out(p.y, p.y_dtype, grow * p.n + (int64_t) nb * kTcTile + lane * 4 + q, v[q]);
        }
    }
}

// ------------------------------------------------------------------ host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 tc_encoder() {
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
int launch_tc(const TcParams& p, cudaStream_t s) {
    auto kern = linear_tc_kernel<K, CB>;
    static std::once_flag once[64];
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    cudaError_t attr = cudaSuccess;
    std::call_once(once[dev & 63], [&] {
        attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    });
    EXL3_CUDA(attr);
    dim3 grid((unsigned) (p.n / kTcTile), (unsigned) ((p.M + kTcTile - 1) / kTcTile));
    kern<<<grid, kTcThreads, kTcSmem, s>>>(p);
    EXL3_CUDA(cudaGetLastError());
    return EXL3_OK;
}

template <int K>
int launch_tc_cb(int cb, const TcParams& p, cudaStream_t s) {
    switch (cb) {
        case 0: return launch_tc<K, 0>(p, s);
        case 1: return launch_tc<K, 1>(p, s);
        default: return launch_tc<K, 2>(p, s);
    }
}

}  // namespace

// Scratch bytes of the tensor-core path: the control words plus the
// transformed activations (fp16 [rows][k]).
int64_t linear_tc_scratch_bytes(int64_t rows, int64_t k) {
    return EXL3_LINEAR_CTRL_BYTES + align_up(rows * k * 2, 256);
}

bool linear_tc_eligible(int64_t rows, int64_t k, int64_t n) {
    return rows >= kTcMinRows && k % kTcKStep == 0 && n % kTcTile == 0;
}

// y = x . W for rows >= kTcMinRows through the tensor cores (weights rounded
// to fp16 as the reference decoder does).  Arguments are validated by the
// caller (exl3_linear).
int linear_tc(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t n, const void* trellis, int K, int cb,
              const void* suh, const void* svh, void* y, int y_dtype, void* scratch, cudaStream_t s) {
    auto encode = tc_encoder();
    EXL3_REQUIRE(encode != nullptr, EXL3_ERR_CUDA, "exl3_linear: cuTensorMapEncodeTiled is not available");
    uint8_t* sb = static_cast<uint8_t*>(scratch);
    __half* xt = reinterpret_cast<__half*>(sb + EXL3_LINEAR_CTRL_BYTES);
    TcParams p{};
    {
        const cuuint64_t dims[3] = {(cuuint64_t) (16 * K), (cuuint64_t) (n / 16), (cuuint64_t) (k / 16)};
        const cuuint64_t strides[2] = {(cuuint64_t) (32 * K), (cuuint64_t) (n / 16) * (cuuint64_t) (32 * K)};
        const cuuint32_t box[3] = {(cuuint32_t) (16 * K), 8u, 8u};
        const cuuint32_t estr[3] = {1u, 1u, 1u};
        const CUresult r = encode(&p.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(trellis), dims,
                                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_linear: weight tensor map failed (%d)", (int) r);
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t) k, (cuuint64_t) rows};
        const cuuint64_t strides[1] = {(cuuint64_t) k * 2};
        const cuuint32_t box[2] = {64u, (cuuint32_t) kTcTile};
        const cuuint32_t estr[2] = {1u, 1u};
        const CUresult r = encode(&p.amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xt, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_linear: activation tensor map failed (%d)", (int) r);
    }
    p.M = (int) rows;
    p.k = (int) k;
    p.n = (int) n;
    p.svh = static_cast<const __half*>(svh);
    p.y = y;
    p.y_dtype = y_dtype;
    p.status = reinterpret_cast<uint32_t*>(sb) + 2;
    const int64_t items = rows * (k / 128);
    input_transform_kernel<<<(unsigned) ((items + 7) / 8), 256, 0, s>>>(x, x_dtype, (int) rows, (int) k,
                                                                      static_cast<const __half*>(suh), xt);
    EXL3_CUDA(cudaGetLastError());
    switch (K) {
        case 1: return launch_tc_cb<1>(cb, p, s);
        case 2: return launch_tc_cb<2>(cb, p, s);
        case 3: return launch_tc_cb<3>(cb, p, s);
        case 4: return launch_tc_cb<4>(cb, p, s);
        case 5: return launch_tc_cb<5>(cb, p, s);
        case 6: return launch_tc_cb<6>(cb, p, s);
        case 7: return launch_tc_cb<7>(cb, p, s);
        default: return launch_tc_cb<8>(cb, p, s);
    }
}

}  // namespace exl3
