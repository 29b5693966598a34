// engine.cuh -- small pieces shared by the EXL3 kernels: work-ticket claims,
// row blocking and the per-128-column output transform.
#pragma once

#include "decode.cuh"

namespace exl3 {

constexpr int kConsumerWarps = 8;                       // decode + MMA warps per CTA
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kCols = 128;                              // output columns per unit (one Hadamard block)

// Row blocks of 8 (the n dimension of one m16n8k16 MMA).
__host__ __device__ constexpr int row_blocks(int rows) { return (rows + 7) >> 3; }

// Next unit ticket.  Every ticket, the first included, comes from the global
// counter, so a unit is only ever owned by a CTA that is already running.
__device__ __forceinline__ int claim_ticket(uint32_t* counter, int lane) {
    int t = 0;
    if (lane == 0) t = (int) atomicAdd(counter, 1u);
    return __shfl_sync(0xffffffffu, t, 0);
}

// Output transform of one 128-column row held as 4 values per lane:
// v <- H128(v) / sqrt(128) * svh.
__device__ __forceinline__ void out_transform(float (&v)[4], const __half* svh_blk, int lane) {
    wht128_warp(v, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = v[q] * kHadNorm * __half2float(svh_blk[lane * 4 + q]);
}

}  // namespace exl3
