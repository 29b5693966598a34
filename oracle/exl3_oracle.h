/*
 * exl3_oracle.h -- CPU oracle for the EXL3 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (dsv4_carve_b200/, the
 * C-ABI library, vllm_exl3_c) may call, link or load this code; only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and only as
 * the checker.
 *
 * Every function restates a reference behaviour and cites it (paths are
 * relative to the lna-lab/dsv4-carve project root):
 *   - trellis bit stream / 16-bit windows:  orders/F1-ref/exl3_dequant.cuh:110-128,
 *                                           orders/F1-ref/exl3_dq.cuh:15-31
 *   - codebooks 3INST / MCG / MUL1:         orders/F1-ref/exl3_dequant.cuh:74-93,
 *                                           recipe-lna/lna2/primitive_gate.cu:25-31
 *   - 16x16 tile fragment placement:        recipe-lna/lna2/bindings.cpp:33-77
 *   - two-sided 128-block Hadamard + su/sv: recipe-lna/lna2/bindings.cpp:79-99
 *   - GEMV form (input/output transforms):  recipe-lna/lna2/lna_moe_ticket.cu:119-144,
 *                                           orders/F1-ref/exl3_gemm_kernel.cuh:14-28
 *   - MoE numerics (fp32 boundaries, clamp-then-SiLU, slot-order sum):
 *                                           recipe-lna/lna2/lna_moe_ticket.cu:5-12,329-359,409-428,
 *                                           recipe-lna/vllm_exl3_exl3.py.lna:988-1027
 *
 * Deliberate correction: the reference's host helper float_to_half_bits
 * truncates the mantissa (exl3_dequant.cuh:41-55), which makes its half add
 * differ from the device __hadd.  This oracle rounds to nearest-even by
 * default; `trunc` = 1 reproduces the helper bit for bit, which is how the
 * oracle is pinned against the reference compiled from source.
 */
#ifndef EXL3_ORACLE_H
#define EXL3_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes shared with the product ABI: 0 fp16, 1 bf16, 2 fp32 */
enum { EXO_F16 = 0, EXO_BF16 = 1, EXO_F32 = 2 };

/* fp16 / bf16 helpers (bit patterns in uint16_t). */
float exo_half_to_float(uint16_t h);
uint16_t exo_half_from_double(double v);      /* round to nearest even */
uint16_t exo_half_from_float_trunc(float v);  /* the reference helper's truncation */
uint16_t exo_bf16_from_double(double v);      /* round to nearest even */

/* 16-bit window of weight t (0..255) in one tile of 16*K uint16 words. */
uint32_t exo_window(const uint16_t* tile, int K, int t);

/* Codebook value of a window as fp16 bits.  cb: 0 3INST, 1 MCG, 2 MUL1. */
uint16_t exo_codebook(uint32_t window, int cb, int trunc);

/* Codebook value with no fp16 rounding: lo + hi for 3INST / MCG (what the
 * fast GEMV path multiplies by), the fp16 value for MUL1. */
double exo_codebook_exact(uint32_t window, int cb);

/* Decode a packed trellis [kt, nt, 16K] int16 into W' [16kt, 16nt] fp16 bits
 * (row = input feature k, column = output feature n). */
void exo_decode(const int16_t* trellis, int64_t kt, int64_t nt, int K, int cb,
                int trunc, uint16_t* wprime);

/* Full weight W = diag(suh) H W' H diag(svh) / 128 -> fp16 bits, with the
 * reference's own float operation order (rows first, then columns). */
void exo_reconstruct(const uint16_t* wprime, const uint16_t* suh,
                     const uint16_t* svh, int64_t k, int64_t n, uint16_t* w);

/* Input transform: xh = fp16( H128( fp16(x) * suh ) / sqrt(128) ), [R, k]. */
void exo_input_transform(const void* x, int x_dtype, int64_t R, int64_t k,
                         const uint16_t* suh, uint16_t* xh);

/* Dense EXL3 linear in GEMV form, result in double [R, n]. */
void exo_gemv(const void* x, int x_dtype, int64_t R, const int16_t* trellis,
              const uint16_t* suh, const uint16_t* svh, int64_t k, int64_t n,
              int K, int cb, double* y);

/* exo_gemv with exact = 1: weights enter as lo + hi unrounded (the fast
 * kernel path's arithmetic); exact = 0 is exo_gemv. */
void exo_gemv_ex(const void* x, int x_dtype, int64_t R, const int16_t* trellis,
                 const uint16_t* suh, const uint16_t* svh, int64_t k, int64_t n,
                 int K, int cb, int exact, double* y);

/* Routed-MoE decode layer (one rank).  Per-expert tables are host arrays of
 * host pointers.  ids [T, topk] int32 (ids outside [0, E) are skipped),
 * weights [T, topk] fp32, out [T, H] double.  Ktab[e] is the bit width of
 * expert e.  Returns the number of unique (expert, row) pairs. */
int64_t exo_moe(const void* x, int x_dtype, int64_t T, int64_t H, int64_t I,
                const int16_t* const* gt, const uint16_t* const* gsu, const uint16_t* const* gsv,
                const int16_t* const* ut, const uint16_t* const* usu, const uint16_t* const* usv,
                const int16_t* const* dt, const uint16_t* const* dsu, const uint16_t* const* dsv,
                const int32_t* Ktab, int cb, int64_t E,
                const int32_t* ids, const float* weights, int64_t topk,
                double limit, double* out);

/* exo_moe with the weight rounding mode of exo_gemv_ex. */
int64_t exo_moe_ex(const void* x, int x_dtype, int64_t T, int64_t H, int64_t I,
                   const int16_t* const* gt, const uint16_t* const* gsu, const uint16_t* const* gsv,
                   const int16_t* const* ut, const uint16_t* const* usu, const uint16_t* const* usv,
                   const int16_t* const* dt, const uint16_t* const* dsu, const uint16_t* const* dsv,
                   const int32_t* Ktab, int cb, int64_t E,
                   const int32_t* ids, const float* weights, int64_t topk,
                   double limit, int exact, double* out);

#ifdef __cplusplus
}
#endif
#endif
