// roof.cu -- decode-issue roof of the EXL3 GEMV engine.
//
// The routed-MoE and dense GEMV kernels stream few bytes per weight (K bits),
// so on B200 their ceiling is set by the integer work of the trellis decode,
// not by HBM.  decode_roof_kernel runs exactly the consumer inner loop of the
// ring engine (stage.cuh: tile_windows_f, codebook_pair, mma_tile2 into split
// accumulators) on weight tiles held in shared memory, with no global traffic
// and no synchronisation, at the MoE kernel's occupancy (2 CTAs of 8 decoding
// warps per SM).  Its rate is the most weights per second that decode loop can
// deliver: the "decode-issue" roof bench.py reports beside the HBM roof.  It is
// the B200 counterpart of the reference's null-decode measurement, which ran
// its kernel with the decode removed to separate memory from decode time
// (LNA2_NULL_DECODE, recipe-lna/lna2/lna_gemv_core.cuh:31-32,170;
// orders/reports/REPORT-F3.md:129,152-177).  Here the memory side is removed
// instead, so what remains is the decode.
#include "host.hpp"
#include "stage.cuh"

namespace exl3 {
namespace {

constexpr int kRoofWarps = 8;
constexpr int kRoofThreads = kRoofWarps * 32;
constexpr int kRoofTiles = 32;            // resident tiles: 4 groups of 8 (one k-slice row each)
constexpr int kRoofSlices = 8;            // k-slices per loop iteration (one ring stage)

template <int K, int CB>
__global__ void __launch_bounds__(kRoofThreads, 2)
    decode_roof_kernel(const uint32_t* __restrict__ words, float* __restrict__ out, int iters,
                       const __grid_constant__ ShiftTable st) {
    using F = TileFmt<K>;
    __shared__ uint32_t tiles[kRoofTiles * F::WORDS];
    __shared__ uint4 frag[kRoofSlices * 32];
    for (int i = threadIdx.x; i < kRoofTiles * F::WORDS; i += blockDim.x) tiles[i] = words[i];
    for (int i = threadIdx.x; i < kRoofSlices * 32; i += blockDim.x) {
        // duplicated-half activations of magnitude ~1 (fast-path fragment layout)
        const uint32_t h = 0x3c003c00u ^ ((uint32_t) i * 0x00010001u & 0x01ff01ffu);
        frag[i] = make_uint4(h, h ^ 0x00010001u, h ^ 0x00020002u, h);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const LaneGeom<K> geom = lane_geom<K>(lane);
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc_odd[4] = {0.f, 0.f, 0.f, 0.f};
    for (int it = 0; it < iters; ++it) {
        const uint32_t* row = tiles + ((it + warp) & (kRoofTiles / kRoofSlices - 1)) * kRoofSlices * F::WORDS;
#pragma unroll
        for (int i = 0; i < kRoofSlices; ++i) {
            const uint32_t* tw = row + i * F::WORDS;
            uint32_t whi[F::NG], wlo[F::NG];
#pragma unroll
            for (int h = 0; h < F::NG; ++h) {
                whi[h] = tw[geom.ihi[h]];
                wlo[h] = tw[geom.ilo[h]];
            }
            uint32_t w[8], x[8];
            tile_windows_f<K>(whi, wlo, geom, st, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = codebook_pair<CB>(w[j]);
            mma_tile2(acc, acc_odd, x, frag[i * 32 + lane]);
        }
    }
    out[(size_t) blockIdx.x * blockDim.x + threadIdx.x] =
        acc[0] + acc[1] + acc[2] + acc[3] + acc_odd[0] + acc_odd[1] + acc_odd[2] + acc_odd[3];
}

template <int CB>
int launch_cb(int K, dim3 grid, const uint32_t* words, float* out, int iters, const ShiftTable& st,
              cudaStream_t s) {
    switch (K) {
        case 1: decode_roof_kernel<1, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        case 2: decode_roof_kernel<2, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        case 3: decode_roof_kernel<3, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        case 4: decode_roof_kernel<4, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        case 5: decode_roof_kernel<5, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        case 6: decode_roof_kernel<6, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        case 7: decode_roof_kernel<7, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
        default: decode_roof_kernel<8, CB><<<grid, kRoofThreads, 0, s>>>(words, out, iters, st); break;
    }
    return EXL3_OK;
}

}  // namespace
}  // namespace exl3

extern "C" int64_t exl3_decode_roof_out_floats(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    exl3::DeviceInfo di;
    if (exl3::device_info(dev, &di)) return -1;
    return (int64_t) di.sms * 2 * exl3::kRoofThreads;
}

extern "C" int exl3_decode_roof(int K, int cb, int iters, const void* words, int64_t words_len, float* out,
                                int64_t out_len, int64_t* weights_decoded, void* stream) {
    using namespace exl3;
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_ARG, "exl3_decode_roof: K must be 1..8 (got %d)", K);
    EXL3_REQUIRE(cb == 0 || cb == 1, EXL3_ERR_ARG, "exl3_decode_roof: codebook must be 0 (3INST) or 1 (MCG)");
    EXL3_REQUIRE(iters >= 1, EXL3_ERR_ARG, "exl3_decode_roof: iters must be >= 1");
    EXL3_REQUIRE(words && out && weights_decoded, EXL3_ERR_ARG, "exl3_decode_roof: null pointer");
    EXL3_REQUIRE(words_len >= (int64_t) kRoofTiles * 8 * K, EXL3_ERR_ARG,
                 "exl3_decode_roof: words needs %d uint32 (got %lld)", kRoofTiles * 8 * K, (long long) words_len);
    int dev = 0;
    EXL3_CUDA(cudaGetDevice(&dev));
    DeviceInfo di;
    if (int rc = device_info(dev, &di)) return rc;
    const dim3 grid((unsigned) (di.sms * 2));
    EXL3_REQUIRE(out_len >= (int64_t) grid.x * kRoofThreads, EXL3_ERR_ARG,
                 "exl3_decode_roof: out needs %lld floats", (long long) grid.x * kRoofThreads);
    ShiftTable st;
    shift_table_init(st);
    auto s = static_cast<cudaStream_t>(stream);
    const auto* w = static_cast<const uint32_t*>(words);
    if (cb == 0) launch_cb<CB_3INST>(K, grid, w, out, iters, st, s);
    else launch_cb<CB_MCG>(K, grid, w, out, iters, st, s);
    EXL3_CUDA(cudaGetLastError());
    *weights_decoded = (int64_t) grid.x * kRoofWarps * iters * kRoofSlices * 256;
    return EXL3_OK;
}
