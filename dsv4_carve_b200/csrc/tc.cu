// tc.cu -- tensor-core (tcgen05) path of the dense EXL3 linear for >= 64 rows
// (prefill chunks), where y = x . W is a real contraction.  Reference: the
// prefill branch of LinearEXL3.forward, reconstruct + hgemm
// (recipe-lna/exllamav3/exl3.py.lna:161-218), and the M16 panel GEMM of
// exl3_gemm_kernel (orders/F1-ref/exl3_gemm_kernel.cuh:8-80).
//
// Dequant-then-MMA with the weights as the M operand: D[n][row] =
// sum_k W^T[n][k] x[row][k], so one CTA decodes each 128-column x 64-k weight
// tile ONCE and applies it to up to 512 activation rows (two N <= 256 MMAs
// into 512 TMEM columns).  A CTA owns (128-column strip, k-chunk, 512-row
// pass); the k-chunks split k so that the grid fills the SMs in one wave:
//   warp 16 (producer) TMA: per k-step of 64, the 4 k-slices x 8 tiles of
//                      packed weights (3-D box) into a 4-stage ring, and the
//                      transformed activations (one or two 64-element x
//                      <= 256-row boxes, 128-byte swizzle) into a 2-stage ring;
//   warps 0-15         decode n-tile w % 8 of k-slices 2 (w / 8), +1 of each
//                      step in registers, round each weight to fp16 (the
//                      reference decoder's value) and write it, K-major with the
//                      128-byte swizzle the MMA descriptor names, into a
//                      3-stage ring of weight tiles;
//   warp 17            allocates the TMEM columns; lane 0 issues tcgen05.mma
//                      (M 128, N <= 256, K 16, fp16 in, fp32 out) and commits
//                      each step to the mbarriers that free its buffers;
//   epilogue           warps 0-15 read the accumulator (tcgen05.ld; warp w
//                      reads TMEM lanes 32 (w % 4)..) and store it as this
//                      chunk's fp32 partial.
// Three launches, chained with programmatic dependent launch so that each
// kernel's prologue overlaps the previous one's tail:
//   tc_input_kernel    x -> fp16, * suh, Hadamard -> fp16 (row-major [M][k]);
//   linear_tc_kernel   the GEMM above (weight copies start before the input
//                      transform has finished; activation copies wait for it);
//   tc_finish_kernel   one warp per output row and strip: the chunk partials
//                      summed in chunk order (results do not depend on timing),
//                      output transform (Hadamard * svh), store y.
// Every wait is bounded; TMEM is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "host.hpp"
#include "tcgen05.cuh"

namespace exl3 {

constexpr int kTcDecWarps = 16;                    // decoder warps: 2 per n-tile, 2 k-slices each per step
constexpr int kTcProducerWarp = kTcDecWarps;
constexpr int kTcMmaWarp = kTcDecWarps + 1;
constexpr int kTcThreads = (kTcDecWarps + 2) * 32;
constexpr int kTcCols = 128;                       // weight columns per CTA (MMA M)
constexpr int kTcKStep = 64;                       // k per pipeline step: 4 k-slices, one 128-byte swizzle row
constexpr int kTcPassRows = 512;                   // activation rows per CTA (TMEM columns)
constexpr int kTcMaxN = 256;                       // MMA N / TMA box height
constexpr int kTcABytes = kTcCols * 128;           // decoded weight tile [128 n][64 k] fp16
constexpr int kTcAStages = 3;
constexpr int kTcXBytes = kTcPassRows * 128;       // activation tile [512 rows][64 k] fp16
constexpr int kTcXStages = 2;
constexpr int kTcWStages = 4;
constexpr int kTcWStageMax = 4 * 8 * 32 * 8;       // 4 k-slices x 8 tiles x 32K bytes at K = 8
constexpr int kTcMinRows = 64;
constexpr int kTcWave = 148;                       // CTAs per wave the k-split aims at (one per SM)
constexpr int kTcMinChunkSteps = 4;                // k-chunks of at least 256
constexpr int kTcFinishRows = 16;                  // rows per finisher CTA (one warp each)

struct TcHead {
    uint64_t wfull[kTcWStages];
    uint64_t wempty[kTcWStages];
    uint64_t aready[kTcAStages];
    uint64_t afree[kTcAStages];
    uint64_t xfull[kTcXStages];
    uint64_t xfree[kTcXStages];
    uint64_t done;
    uint32_t tmem;
};
constexpr int kTcSmem = 1024 /* alignment slack */ + kTcXStages * kTcXBytes + kTcAStages * kTcABytes +
                        kTcWStages * kTcWStageMax + 256;
static_assert(sizeof(TcHead) <= 256, "head must fit its slot");

struct TcParams {
    CUtensorMap wmap;      // trellis [k/16][n/16][16K] u16, box [16K, 8, 4]
    CUtensorMap xmap;      // transformed x [M][k] fp16, box [64, box_rows], 128-byte swizzle
    int M, k, n;
    int box_rows;          // TMA box height (<= 256, multiple of 16)
    int chunks;            // k-chunks per strip
    int tmem_cols;         // TMEM columns allocated (power of two >= 32)
    const __half* svh;
    float* part;           // [chunks][M][n] fp32 partials
    uint32_t* status;
    ShiftTable st;         // IMAD shift multipliers of the window extraction
};


// ------------------------------------------------------------------ input transform
// xt[r][k] = fp16( H128( fp16(x[r][k]) * suh[k] ) / sqrt(128) ), one warp per
// (row, 128-block) (recipe-lna/lna2/lna_moe_ticket.cu:119-144).
__global__ void __launch_bounds__(256) tc_input_kernel(const void* x, int x_dtype, int M, int k,
                                                       const __half* suh, __half* xt) {
    pdl_launch_dependents();
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
    uint8_t* Xbuf = base;                                          // [2][64 KB]
    uint8_t* Abuf = Xbuf + kTcXStages * kTcXBytes;                 // [3][16 KB]
    uint8_t* Wring = Abuf + kTcAStages * kTcABytes;                // [4][8 KB]
    TcHead& H = *reinterpret_cast<TcHead*>(Wring + kTcWStages * kTcWStageMax);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int strips = p.n / kTcCols;
    const int strip = (int) blockIdx.x % strips, chunk = (int) blockIdx.x / strips;
    const int pass = blockIdx.y;
    const int KS = p.k / kTcKStep;
    const int kbeg = chunk * KS / p.chunks, nsteps = (chunk + 1) * KS / p.chunks - kbeg;
    const int row0 = pass * kTcPassRows;
    const int rows = min(kTcPassRows, p.M - row0);
    const int nbox = (rows + p.box_rows - 1) / p.box_rows;
    const int n0 = min(kTcMaxN, (rows + 15) & ~15);                // MMA N of accumulator 0
    const int n1 = rows > kTcMaxN ? ((rows - kTcMaxN + 15) & ~15) : 0;
    uint32_t* status = p.status;

    if (tid == 0) {
        for (int s = 0; s < kTcWStages; ++s) { mbar_init(&H.wfull[s], 1); mbar_init(&H.wempty[s], kTcDecWarps); }
        for (int s = 0; s < kTcAStages; ++s) { mbar_init(&H.aready[s], kTcDecWarps); mbar_init(&H.afree[s], 1); }
        for (int s = 0; s < kTcXStages; ++s) { mbar_init(&H.xfull[s], 1); mbar_init(&H.xfree[s], 1); }
        mbar_init(&H.done, 1);
        fence_barrier_init();
    }
    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&H.tmem)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = H.tmem;

    if (warp == kTcProducerWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t wbytes = (uint32_t) (4 * 8 * 32 * K);
            const uint32_t xbytes = (uint32_t) (nbox * p.box_rows * 128);
            uint32_t issued_w = 0, issued_x = 0;
            bool ok = true;
            for (int s = 0; s < nsteps && ok; ++s) {
                const int ws = s % kTcWStages, xs = s % kTcXStages, ks = kbeg + s;
                ok = mbar_wait(&H.wempty[ws], ((s / kTcWStages) + 1u) & 1u, status);
                if (!ok) break;
                mbar_arrive_expect_tx(&H.wfull[ws], wbytes);
                tma_load_3d(Wring + ws * kTcWStageMax, &p.wmap, 0, strip * 8, ks * 4, &H.wfull[ws]);
                ++issued_w;
                if (s == 0) pdl_wait();                      // the transformed activations are complete
                ok = mbar_wait(&H.xfree[xs], ((s / kTcXStages) + 1u) & 1u, status);
                if (!ok) break;
                mbar_arrive_expect_tx(&H.xfull[xs], xbytes);
                for (int b = 0; b < nbox; ++b)
                    tma_load_2d(Xbuf + xs * kTcXBytes + b * p.box_rows * 128, &p.xmap, ks * kTcKStep,
                                row0 + b * p.box_rows, &H.xfull[xs]);
                ++issued_x;
            }
            // no copy may still be in flight when the CTA retires
            for (uint32_t i = issued_w > kTcWStages ? issued_w - kTcWStages : 0; i < issued_w; ++i)
                if (!mbar_wait(&H.wfull[i % kTcWStages], (i / kTcWStages) & 1u, status)) break;
            for (uint32_t i = issued_x > kTcXStages ? issued_x - kTcXStages : 0; i < issued_x; ++i)
                if (!mbar_wait(&H.xfull[i % kTcXStages], (i / kTcXStages) & 1u, status)) break;
        }
    } else if (warp == kTcMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id0 = idesc_f16(kTcCols, n0), id1 = idesc_f16(kTcCols, n1 > 0 ? n1 : 16);
            const uint64_t adesc0 = sdesc_sw128(smem_u32(Abuf)), xdesc0 = sdesc_sw128(smem_u32(Xbuf));
            bool ok = true;
            for (int s = 0; s < nsteps && ok; ++s) {
                const int as = s % kTcAStages, xs = s % kTcXStages;
                ok = mbar_wait(&H.xfull[xs], (s / kTcXStages) & 1u, status) &&
                     mbar_wait(&H.aready[as], (s / kTcAStages) & 1u, status);
                if (!ok) break;
                tc_fence_after();
                // descriptors advance in 16-byte units: +2 per 16-element k step
                const uint64_t ad = adesc0 + (uint64_t) (as * (kTcABytes >> 4));
                const uint64_t xd = xdesc0 + (uint64_t) (xs * (kTcXBytes >> 4));
                const uint32_t en = s != 0;
                if (n1 > 0) {
#pragma unroll
                    for (int kk = 0; kk < kTcKStep / 16; ++kk) {
                        tc_mma(tmem, ad + 2 * kk, xd + 2 * kk, id0, en | kk);
                        tc_mma(tmem + kTcMaxN, ad + 2 * kk, xd + (kTcMaxN * 128 >> 4) + 2 * kk, id1, en | kk);
                    }
                } else {
#pragma unroll
                    for (int kk = 0; kk < kTcKStep / 16; ++kk) tc_mma(tmem, ad + 2 * kk, xd + 2 * kk, id0, en | kk);
                }
                tc_commit(&H.afree[as]);
                tc_commit(&H.xfree[xs]);
            }
            tc_commit(&H.done);
        }
    } else {
        // ------------------------------------------------------------ decoders
        const LaneGeom<K> geom = lane_geom<K>(lane);
        const int t4 = lane & 3, g = lane >> 2;
        const int ntile = warp & 7, i0 = (warp >> 3) * 2;
        const int c0 = ntile * 16 + g;                 // this lane's weight columns c0 and c0 + 8
        for (int s = 0; s < nsteps; ++s) {
            const int ws = s % kTcWStages, as = s % kTcAStages;
            if (!mbar_wait_lanes(&H.wfull[ws], (s / kTcWStages) & 1u, status)) break;
            if (!mbar_wait_lanes(&H.afree[as], ((s / kTcAStages) + 1u) & 1u, status)) break;
            const uint32_t* wst = reinterpret_cast<const uint32_t*>(Wring + ws * kTcWStageMax);
            uint8_t* A = Abuf + as * kTcABytes;
#pragma unroll
            for (int i = i0; i < i0 + 2; ++i) {
                const uint32_t* t = wst + (i * 8 + ntile) * F::WORDS;
                uint32_t whi[F::NG], wlo[F::NG], w[8], x[8];
#pragma unroll
                for (int h = 0; h < F::NG; ++h) {
                    whi[h] = t[geom.ihi[h]];
                    wlo[h] = t[geom.ilo[h]];
                }
                tile_windows_f<K>(whi, wlo, geom, p.st, w);
#pragma unroll
                for (int j = 0; j < 8; ++j) x[j] = codebook_pair<CB>(w[j]);
                const int kk = i * 16 + 2 * t4;
                *reinterpret_cast<uint32_t*>(A + sw128_offset(c0, kk)) = round_pair(x[0], x[1]);
                *reinterpret_cast<uint32_t*>(A + sw128_offset(c0, kk + 8)) = round_pair(x[2], x[3]);
                *reinterpret_cast<uint32_t*>(A + sw128_offset(c0 + 8, kk)) = round_pair(x[4], x[5]);
                *reinterpret_cast<uint32_t*>(A + sw128_offset(c0 + 8, kk + 8)) = round_pair(x[6], x[7]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor core reads
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&H.aready[as]);
                mbar_arrive(&H.wempty[ws]);
            }
        }
    }

    // ---------------------------------------------------------------- epilogue
    __syncthreads();
    const int64_t ld = p.n;
    if (warp < kTcDecWarps) {
        // accumulator -> this chunk's partial: thread = weight column, 16 rows per load
        mbar_wait_lanes(&H.done, 0u, status);
        tc_fence_after();
        const int lg = warp & 3, col = strip * kTcCols + lg * 32 + lane;
        float* part = p.part + (int64_t) chunk * p.M * ld + col;
        for (int c = warp >> 2; c * 16 < rows; c += 4) {
            float v[16];
            tc_ld16(tmem + ((uint32_t) (lg * 32) << 16) + (uint32_t) (c * 16), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int r = c * 16 + i;
                if (r < rows) part[(int64_t) (row0 + r) * ld] = v[i];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

// One warp per (row, strip): y[row][strip cols] = out_transform(sum over
// chunks, in chunk order, of the partials).
__global__ void __launch_bounds__(kTcFinishRows * 32) tc_finish_kernel(const float* part, int chunks, int M, int n,
                                                                     const __half* svh, void* y, int y_dtype) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int strip = blockIdx.x;
    const int64_t row = (int64_t) blockIdx.y * kTcFinishRows + (threadIdx.x >> 5);
    if (row >= M) return;
    const int64_t plane = (int64_t) M * n;
    const float* src = part + row * n + strip * kTcCols + lane * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < chunks; ++c) {
        const float4 q = __ldcg(reinterpret_cast<const float4*>(src + c * plane));
        v[0] += q.x; v[1] += q.y; v[2] += q.z; v[3] += q.w;
    }
    out_transform(v, svh + (int64_t) strip * kTcCols, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) store_out(y, y_dtype, row * n + strip * kTcCols + lane * 4 + q, v[q]);
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

// Launch with the programmatic-stream-serialization attribute: the kernel may
// start once the previous kernel in the stream has triggered (or retired), and
// synchronises on it with griddepcontrol.wait.
template <typename... Args>
cudaError_t launch_pdl(void (*kern)(Args...), dim3 grid, dim3 block, int smem, cudaStream_t s,
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
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
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
    EXL3_CUDA(launch_pdl(kern, dim3((unsigned) (p.n / kTcCols * p.chunks),
                                    (unsigned) ((p.M + kTcPassRows - 1) / kTcPassRows)),
                         dim3(kTcThreads), kTcSmem, s, p));
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

// k-chunks per 128-column strip: enough (strip, chunk, pass) CTAs for about
// one wave, each chunk at least kTcMinChunkSteps k-steps.  A function of the
// shape only, so the scratch size does not depend on the device.
int tc_chunks(int64_t rows, int64_t k, int64_t n) {
    const int64_t base = (n / kTcCols) * ((rows + kTcPassRows - 1) / kTcPassRows);
    int64_t c = kTcWave / base;
    const int64_t cmax = (k / kTcKStep) / kTcMinChunkSteps;
    if (c > cmax) c = cmax;
    return c < 1 ? 1 : (int) c;
}

// Scratch bytes of the tensor-core path: the control words, the transformed
// activations (fp16 [rows][k]) and the chunk partials (fp32 [chunks][rows][n]).
int64_t linear_tc_scratch_bytes(int64_t rows, int64_t k, int64_t n) {
    return EXL3_LINEAR_CTRL_BYTES + align_up(rows * k * 2, 256) + align_up(tc_chunks(rows, k, n) * rows * n * 4, 256);
}

bool linear_tc_eligible(int64_t rows, int64_t k, int64_t n) {
    return rows >= kTcMinRows && k % kTcKStep == 0 && n % kTcCols == 0 && rows <= INT32_MAX / 2;
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
    const int64_t pass_rows = rows < kTcPassRows ? rows : kTcPassRows;
    p.box_rows = (int) ((pass_rows + 15) & ~15);
    if (p.box_rows > kTcMaxN) p.box_rows = kTcMaxN;
    p.chunks = tc_chunks(rows, k, n);
    p.tmem_cols = 32;
    while (p.tmem_cols < ((pass_rows + 15) & ~15)) p.tmem_cols <<= 1;
    if (pass_rows > kTcMaxN) p.tmem_cols = kTcPassRows;
    {
        const cuuint64_t dims[3] = {(cuuint64_t) (16 * K), (cuuint64_t) (n / 16), (cuuint64_t) (k / 16)};
        const cuuint64_t strides[2] = {(cuuint64_t) (32 * K), (cuuint64_t) (n / 16) * (cuuint64_t) (32 * K)};
        const cuuint32_t box[3] = {(cuuint32_t) (16 * K), 8u, 4u};
        const cuuint32_t estr[3] = {1u, 1u, 1u};
        const CUresult r = encode(&p.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(trellis), dims,
                                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_linear: weight tensor map failed (%d)", (int) r);
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t) k, (cuuint64_t) rows};
        const cuuint64_t strides[1] = {(cuuint64_t) k * 2};
        const cuuint32_t box[2] = {(cuuint32_t) kTcKStep, (cuuint32_t) p.box_rows};
        const cuuint32_t estr[2] = {1u, 1u};
        const CUresult r = encode(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xt, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        EXL3_REQUIRE(r == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_linear: activation tensor map failed (%d)", (int) r);
    }
    p.M = (int) rows;
    p.k = (int) k;
    p.n = (int) n;
    p.svh = static_cast<const __half*>(svh);
    p.status = reinterpret_cast<uint32_t*>(sb) + 2;
    shift_table_init(p.st);
    p.part = reinterpret_cast<float*>(sb + EXL3_LINEAR_CTRL_BYTES + align_up(rows * k * 2, 256));
    const int64_t items = rows * (k / 128);
    tc_input_kernel<<<(unsigned) ((items + 7) / 8), 256, 0, s>>>(x, x_dtype, (int) rows, (int) k,
                                                               static_cast<const __half*>(suh), xt);
    EXL3_CUDA(cudaGetLastError());
    int rc;
    switch (K) {
        case 1: rc = launch_tc_cb<1>(cb, p, s); break;
        case 2: rc = launch_tc_cb<2>(cb, p, s); break;
        case 3: rc = launch_tc_cb<3>(cb, p, s); break;
        case 4: rc = launch_tc_cb<4>(cb, p, s); break;
        case 5: rc = launch_tc_cb<5>(cb, p, s); break;
        case 6: rc = launch_tc_cb<6>(cb, p, s); break;
        case 7: rc = launch_tc_cb<7>(cb, p, s); break;
        default: rc = launch_tc_cb<8>(cb, p, s); break;
    }
    if (rc != EXL3_OK) return rc;
    EXL3_CUDA(launch_pdl(tc_finish_kernel, dim3((unsigned) (n / kTcCols), (unsigned) ((rows + kTcFinishRows - 1) / kTcFinishRows)),
                         dim3(kTcFinishRows * 32), 0, s, (const float*) p.part, p.chunks, (int) rows, (int) n,
                         (const __half*) svh, y, y_dtype));
    return EXL3_OK;
}

}  // namespace exl3
