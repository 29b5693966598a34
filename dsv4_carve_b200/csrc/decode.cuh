// decode.cuh -- EXL3 trellis decode for one 16x16 tile per warp, in registers.
//
// Format (restated from orders/F1-ref/exl3_dequant.cuh:110-128 and
// orders/F1-ref/exl3_dq.cuh:15-31): a tile is 16*K uint16 words viewed as 8K
// uint32 words (u32 i = u16[2i] | u16[2i+1] << 16).  They form a circular
// 256K-bit stream read most-significant-bit first.  Weight t (0..255) is the
// 16-bit window that ends at stream bit (t+257)*K - 1.
//
// Lane l of a warp decodes weights t = 8l .. 8l+7.  With j = t % 8 they sit at
//   k = 2(l%4) + (j&1) + 8((j>>1)&1),   n = l/4 + 8(j>>2)
// inside the tile (recipe-lna/lna2/bindings.cpp:52-76), which is exactly the
// A-operand fragment of mma.m16n8k16 when A = W^T (rows = output channels):
// every lane decodes its own fragment and no shuffle is needed.
//
// Codebooks (exl3_dequant.cuh:74-93, primitive_gate.cu:25-31):
//   3INST  x = w * 89226354 + 64248484
//   MCG    x = w * 0xCBAC1FED
//   then   x = (x & 0x8fff8fff) ^ 0x3b603b60      (lop3 LUT 0x6a)
//   value  = fp16(x & 0xffff) + fp16(x >> 16)
//   MUL1   s = 0x6400 + bytesum(w * 0x83DCD12D);  value = s * fp16(0x1eee) + fp16(0xc931)
// The fast GEMV path never forms `value`: the (lo, hi) half pair produced by
// the lop3 is used directly as one packed A element against a duplicated
// activation, so the tensor core computes x*lo + x*hi in fp32.  The PRECISE
// path rounds each weight to fp16 first (mma_tile_precise).
#pragma once

#include "common.cuh"

namespace exl3 {

enum Codebook : int { CB_3INST = 0, CB_MCG = 1, CB_MUL1 = 2 };

// Windows per 64-bit group: every group's 16 + (G-1)K stream bits fit in two
// consecutive uint32 words for any lane (checked for K = 1..8).  Groups are
// kept short enough that most windows sit at most 16 bits above the group's
// last one (K <= 5: all of them), which the extraction of tile_windows_f
// turns into one shift and one byte permute.
template <int K> struct TileFmt {
    static constexpr int G = (K <= 2) ? 8 : (K == 7 ? 2 : 4);
    static constexpr int NG = 8 / G;
    static constexpr int WORDS = 8 * K;         // uint32 words per tile
    static constexpr int BYTES = 32 * K;        // bytes per tile
};

// Per-lane constant geometry of a tile: for group h, the two words that hold
// it (hi = earlier stream bits) and the right shift that puts the group's last
// window at bit 0 of the 64-bit pair.  The shift is kept < 32 by moving the
// word pair when needed.
template <int K> struct LaneGeom {
    uint8_t ihi[TileFmt<K>::NG];
    uint8_t ilo[TileFmt<K>::NG];
    uint8_t sh[TileFmt<K>::NG];
};

template <int K>
__device__ __forceinline__ LaneGeom<K> lane_geom(int lane) {
    using F = TileFmt<K>;
    LaneGeom<K> g;
    const int nbits = 256 * K;
#pragma unroll
    for (int h = 0; h < F::NG; ++h) {
        const int first = 8 * lane + h * F::G;          // first weight of the group
        const int start = ((first + 257) * K - 16) % nbits;
        int i0 = start >> 5;                             // word holding the first bit
        // LSB position (in the 64-bit pair word[i0]:word[i0+1]) of the LAST window.
        int lsb = 48 - (start & 31) - (F::G - 1) * K;
        if (lsb >= 32) { i0 = (i0 + F::WORDS - 1) % F::WORDS; lsb -= 32; }
        g.ihi[h] = (uint8_t) i0;
        g.ilo[h] = (uint8_t) ((i0 + 1) % F::WORDS);
        g.sh[h] = (uint8_t) lsb;
    }
    return g;
}

// Extract window `off` bits above the group's last window from the pair
// (hi32:lo32), zero-extended to 16 bits.
template <int OFF>
__device__ __forceinline__ uint32_t window_at(uint32_t lo32, uint32_t hi32) {
    if constexpr (OFF == 0) return lo32 & 0xffffu;
    else if constexpr (OFF == 8) return __byte_perm(lo32, 0u, 0x4421);
    else if constexpr (OFF == 16) return lo32 >> 16;
    else if constexpr (OFF + 16 <= 32) return (lo32 >> OFF) & 0xffffu;
    else if constexpr (OFF < 32) return __funnelshift_r(lo32, hi32, OFF) & 0xffffu;
    else if constexpr (OFF == 32) return hi32 & 0xffffu;
    else if constexpr (OFF == 40) return __byte_perm(hi32, 0u, 0x4421);
    else return (hi32 >> (OFF - 32)) & 0xffffu;
}

template <int K, int G, int U>
__device__ __forceinline__ uint32_t window_u(uint32_t lo32, uint32_t hi32) {
    return window_at<(G - 1 - U) * K>(lo32, hi32);
}

// 16-bit windows of this lane's 8 weights, j = 0..7, from the already loaded
// word pairs of each group (whi[h] = tile word g.ihi[h], wlo[h] = g.ilo[h]).
template <int K>
__device__ __forceinline__ void tile_windows_w(const uint32_t (&whi_)[TileFmt<K>::NG],
                                               const uint32_t (&wlo_)[TileFmt<K>::NG], const LaneGeom<K>& g,
                                               uint32_t (&w)[8]) {
    using F = TileFmt<K>;
#pragma unroll
    for (int h = 0; h < F::NG; ++h) {
        const uint32_t whi = whi_[h];
        const uint32_t wlo = wlo_[h];
        const uint32_t lo32 = __funnelshift_r(wlo, whi, g.sh[h]);
        const uint32_t hi32 = whi >> g.sh[h];
        if constexpr (K == 2) {
            // Phase trick: three shifted copies make every window byte aligned.
            const uint32_t p2 = lo32 >> 2, p4 = lo32 >> 4, p6 = lo32 >> 6;
            w[0] = __byte_perm(p6, 0u, 0x4421);
            w[1] = __byte_perm(p4, 0u, 0x4421);
            w[2] = __byte_perm(p2, 0u, 0x4421);
            w[3] = __byte_perm(lo32, 0u, 0x4421);
            w[4] = p6 & 0xffffu;
            w[5] = p4 & 0xffffu;
            w[6] = p2 & 0xffffu;
            w[7] = lo32 & 0xffffu;
        } else {
            constexpr int G = F::G;
            w[h * G + 0] = window_u<K, G, 0>(lo32, hi32);
            if constexpr (G > 1) w[h * G + 1] = window_u<K, G, 1>(lo32, hi32);
            if constexpr (G > 2) w[h * G + 2] = window_u<K, G, 2>(lo32, hi32);
            if constexpr (G > 3) w[h * G + 3] = window_u<K, G, 3>(lo32, hi32);
            if constexpr (G > 4) w[h * G + 4] = window_u<K, G, 4>(lo32, hi32);
            if constexpr (G > 5) w[h * G + 5] = window_u<K, G, 5>(lo32, hi32);
            if constexpr (G > 6) w[h * G + 6] = window_u<K, G, 6>(lo32, hi32);
            if constexpr (G > 7) w[h * G + 7] = window_u<K, G, 7>(lo32, hi32);
        }
    }
}

// Powers of two 2^1 .. 2^15 held in kernel parameters.  A left shift written
// as a multiply by one of them stays an integer multiply-add (the FMA pipe),
// because the compiler cannot see the value; the same shift by a literal would
// be issued to the 16-lane integer ALU pipe, which the decode already fills
// with its byte permutes and codebook LOP3s.
struct ShiftTable {
    uint32_t mul[16];           // mul[i] = 1u << i
};

inline void shift_table_init(ShiftTable& t) {
    for (int i = 0; i < 16; ++i) t.mul[i] = 1u << i;
}

// Window `OFF` bits above the group's last window, zero-extended: byte
// permutes for byte-aligned offsets; otherwise the window is moved to the top
// half by an IMAD left shift and taken by a byte permute.  Offsets above 16
// (K = 6 and 8 only) fall back to the funnel shift of window_at.
template <int OFF>
__device__ __forceinline__ uint32_t window_f(uint32_t lo32, uint32_t hi32, const ShiftTable& st) {
    if constexpr (OFF == 0) return lo32 & 0xffffu;
    else if constexpr (OFF == 8) return __byte_perm(lo32, 0u, 0x4421);
    else if constexpr (OFF == 16) return __byte_perm(lo32, 0u, 0x4432);
    else if constexpr (OFF < 16) return __byte_perm(lo32 * st.mul[16 - OFF], 0u, 0x4432);
    else return window_at<OFF>(lo32, hi32);
}

// tile_windows_w with the extraction of window_f (the GEMV engine's decoder).
// K = 2: the eight windows sit 2 bits apart in one word, so three IMAD-shifted
// copies (by 2, 4 and 6) put every window at bit 0, 8 or 16 of some copy, where
// a byte permute takes it: 3 IMAD + 8 ALU instead of 6 + 8 (measured on B200:
// 5.76 against 5.54 T weights/s for the decode loop).
template <int K>
__device__ __forceinline__ void tile_windows_f(const uint32_t (&whi_)[TileFmt<K>::NG],
                                               const uint32_t (&wlo_)[TileFmt<K>::NG], const LaneGeom<K>& g,
                                               const ShiftTable& st, uint32_t (&w)[8]) {
    using F = TileFmt<K>;
    constexpr int G = F::G;
    if constexpr (K == 2) {
        const uint32_t lo32 = __funnelshift_r(wlo_[0], whi_[0], g.sh[0]);
        const uint32_t a2 = lo32 * st.mul[2], a4 = lo32 * st.mul[4], a6 = lo32 * st.mul[6];
        w[0] = __byte_perm(a2, 0u, 0x4432);     // window 14 bits above the last: bits 16..31 of a2
        w[1] = __byte_perm(a4, 0u, 0x4432);     // 12
        w[2] = __byte_perm(a6, 0u, 0x4432);     // 10
        w[3] = __byte_perm(lo32, 0u, 0x4421);   // 8
        w[4] = __byte_perm(a2, 0u, 0x4421);     // 6: bits 8..23 of a2
        w[5] = __byte_perm(a4, 0u, 0x4421);     // 4
        w[6] = __byte_perm(a6, 0u, 0x4421);     // 2
        w[7] = lo32 & 0xffffu;                  // 0
    } else {
#pragma unroll
    for (int h = 0; h < F::NG; ++h) {
        const uint32_t lo32 = __funnelshift_r(wlo_[h], whi_[h], g.sh[h]);
        const uint32_t hi32 = ((G - 1) * K > 16) ? (whi_[h] >> g.sh[h]) : 0u;
        w[h * G + 0] = window_f<(G - 1) * K>(lo32, hi32, st);
        if constexpr (G > 1) w[h * G + 1] = window_f<(G - 2) * K>(lo32, hi32, st);
        if constexpr (G > 2) w[h * G + 2] = window_f<(G > 2 ? G - 3 : 0) * K>(lo32, hi32, st);
        if constexpr (G > 3) w[h * G + 3] = window_f<(G > 3 ? G - 4 : 0) * K>(lo32, hi32, st);
        if constexpr (G > 4) w[h * G + 4] = window_f<(G > 4 ? G - 5 : 0) * K>(lo32, hi32, st);
        if constexpr (G > 5) w[h * G + 5] = window_f<(G > 5 ? G - 6 : 0) * K>(lo32, hi32, st);
        if constexpr (G > 6) w[h * G + 6] = window_f<(G > 6 ? G - 7 : 0) * K>(lo32, hi32, st);
        if constexpr (G > 7) w[h * G + 7] = window_f<(G > 7 ? G - 8 : 0) * K>(lo32, hi32, st);
    }
    }
}

// 16-bit windows of this lane's 8 weights, j = 0..7, reading the tile at tw.
template <int K>
__device__ __forceinline__ void tile_windows(const uint32_t* tw, const LaneGeom<K>& g, uint32_t (&w)[8]) {
    uint32_t whi[TileFmt<K>::NG], wlo[TileFmt<K>::NG];
#pragma unroll
    for (int h = 0; h < TileFmt<K>::NG; ++h) {
        whi[h] = tw[g.ihi[h]];
        wlo[h] = tw[g.ilo[h]];
    }
    tile_windows_w<K>(whi, wlo, g, w);
}

// Codebook -> packed (lo, hi) fp16 pair whose sum is the weight.
template <int CB>
__device__ __forceinline__ uint32_t codebook_pair(uint32_t w) {
    if constexpr (CB == CB_MUL1) {
        const uint32_t x = w * 0x83DCD12Du;
        const uint32_t s = __dp4a(x, 0x01010101u, 0x6400u);   // 0x6400 + byte sum
        const __half v = __hfma(__ushort_as_half((uint16_t) s), __ushort_as_half((uint16_t) 0x1eee),
                                __ushort_as_half((uint16_t) 0xc931));
        return (uint32_t) __half_as_ushort(v);                  // (value, +0)
    } else {
        uint32_t x;
        if constexpr (CB == CB_3INST) x = w * 89226354u + 64248484u;
        else x = w * 0xCBAC1FEDu;
        uint32_t y;
        asm("lop3.b32 %0, %1, 0x8fff8fff, 0x3b603b60, 0x6a;" : "=r"(y) : "r"(x));
        return y;
    }
}

// Exact fp16 weight (single nearest-even rounding of lo + hi).
template <int CB>
__device__ __forceinline__ __half codebook_value(uint32_t w) {
    const uint32_t p = codebook_pair<CB>(w);
    if constexpr (CB == CB_MUL1) return __ushort_as_half((uint16_t) p);
    return __hadd(__ushort_as_half((uint16_t) (p & 0xffffu)), __ushort_as_half((uint16_t) (p >> 16)));
}

// ------------------------------------------------------------------ MMA
// D[16 ch x 8 rows] += A[16 ch x 16] * B[16 x 8 rows], fp16 in, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One tile against one 8-row block of activations.  x[] are the decoded
// pairs; bf = (even-k b0, even-k b1, odd-k b0, odd-k b1) duplicated halves.
// Even tile-k rows go through the first MMA, odd ones through the second
// (each packed pair occupies two k slots of the k-doubled MMA).
__device__ __forceinline__ void mma_tile(float (&d)[4], const uint32_t (&x)[8], const uint4& bf) {
    mma_16816(d, x[0], x[4], x[2], x[6], bf.x, bf.y);
    mma_16816(d, x[1], x[5], x[3], x[7], bf.z, bf.w);
}

// mma_tile with the even and odd k rows summed into separate accumulators, so
// the two MMAs of a tile do not wait on each other; the caller adds d1 to d0
// at the end of its k range.
__device__ __forceinline__ void mma_tile2(float (&d0)[4], float (&d1)[4], const uint32_t (&x)[8], const uint4& bf) {
    mma_16816(d0, x[0], x[4], x[2], x[6], bf.x, bf.y);
    mma_16816(d1, x[1], x[5], x[3], x[7], bf.z, bf.w);
}

// PRECISE variant: the weights the reference actually uses, RN(lo + hi) in
// fp16, two consecutive k of one output channel per register (a standard,
// non-doubled A operand): 2 PRMT + 1 HADD2 per pair of weights.
__device__ __forceinline__ uint32_t round_pair(uint32_t xa, uint32_t xb) {
    const uint32_t lo = __byte_perm(xa, xb, 0x5410);   // (lo_a, lo_b)
    const uint32_t hi = __byte_perm(xa, xb, 0x7632);   // (hi_a, hi_b)
    const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
    return *reinterpret_cast<const uint32_t*>(&s);
}

// One tile against one 8-row block, fp16-rounded weights: b = (x[2t], x[2t+1]),
// (x[2t+8], x[2t+9]) of row g.
__device__ __forceinline__ void mma_tile_precise(float (&d)[4], const uint32_t (&x)[8], const uint2& bf) {
    mma_16816(d, round_pair(x[0], x[1]), round_pair(x[4], x[5]), round_pair(x[2], x[3]), round_pair(x[6], x[7]),
              bf.x, bf.y);
}

}  // namespace exl3
