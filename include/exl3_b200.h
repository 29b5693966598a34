/*
 * exl3_b200.h -- C ABI of the B200 (sm_100a) EXL3 decode hot path.
 *
 * Library: dsv4_carve_b200/libexl3b200.so.  Plain pointers, sizes and a CUDA
 * stream (passed as void*, i.e. a cudaStream_t); no C++ or torch types.  All
 * device pointers must be on the device that is current on the calling
 * thread.  Every function returns EXL3_OK (0) or an exl3_status code; on
 * failure exl3_last_error() returns a message for the calling thread.  Calls
 * that launch work are asynchronous on `stream`.  The entry points that take
 * a caller scratch never allocate, copy or synchronize, so they may be
 * captured in a CUDA graph once the per-device state has been prepared
 * (exl3_*_prepare, or one eager call).
 *
 * Data formats (the EXL3 on-disk / in-memory layout used by the reference):
 *   trellis  int16 [k/16, n/16, 16*K]   packed trellis words of W' (k = in, n = out)
 *   suh      fp16  [k]                  input sign/scale vector
 *   svh      fp16  [n]                  output sign/scale vector
 *   W = diag(suh) . H . W' . H . diag(svh) / 128, H = 128-block Sylvester Hadamard.
 * Codebooks: 0 = 3INST, 1 = MCG (the production codebook), 2 = MUL1.
 * Activation / output dtypes: 0 = fp16, 1 = bf16, 2 = fp32.
 *
 * Each declaration cites the reference interface it replaces (paths relative
 * to the lna-lab/dsv4-carve project root).
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    EXL3_OK = 0,
    EXL3_ERR_ARG = 1,          /* invalid argument (shape, dtype, alignment, size) */
    EXL3_ERR_CUDA = 2,         /* a CUDA runtime call failed */
    EXL3_ERR_UNSUPPORTED = 3,  /* valid input outside what this build implements */
    EXL3_ERR_DEVICE = 4        /* the device-side status word reports a failure */
} exl3_status;

enum { EXL3_DTYPE_F16 = 0, EXL3_DTYPE_BF16 = 1, EXL3_DTYPE_F32 = 2 };
enum { EXL3_CB_3INST = 0, EXL3_CB_MCG = 1, EXL3_CB_MUL1 = 2 };

/* Version of this ABI (bumped on any signature change). */
int exl3_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* exl3_last_error(void);

/* ------------------------------------------------------------------ dequant
 * Replaces vllm_exl3_c.dequant_trellis (recipe-lna/lna2/bindings.cpp:118-133,
 * CPU dequant_cpu at :16-101) and the exllamav3_ext reconstruct call used by
 * LinearEXL3.reconstruct_hgemm (recipe-lna/exllamav3/exl3.py.lna:161-218).
 * full = 0: w = W' (inner decoded weights), fp16 [16*kt, 16*nt], bit-exact.
 * full = 1: w = W  (both Hadamards and suh/svh applied in the reference's
 *           float order), fp16.  suh/svh may be NULL when full = 0.
 * K in 1..8; kt and nt multiples of 8 when full = 1. */
int exl3_dequant(const void* trellis, int64_t kt, int64_t nt, int K, int cb,
                 const void* suh, const void* svh, void* w, int full, void* stream);

/* Arithmetic of the decode + MMA inner loop (`precise` argument below):
 *   precise = 1: each weight is rounded to fp16, RN(lo + hi), exactly the
 *                value the reference's decoder produces, before the fp16 MMA;
 *   precise = 0: the codebook's (lo, hi) fp16 halves go to the tensor core
 *                as one k-doubled element, so the weight enters as lo + hi
 *                unrounded (one fewer rounding, fewer instructions).
 * Both accumulate in fp32; they differ by the fp16 rounding of each weight. */

/* ------------------------------------------------------------------ dense linear
 * y[rows, n] = x[rows, k] . W   (GEMV form: input transform, decode + MMA,
 * output transform).  Below 64 rows the kernel is launched with programmatic
 * stream serialization: its CTAs may start while the previous kernel in the
 * stream is still running and stream the weights (`trellis`) before they
 * wait for it; x, the scratch and y are touched only after that kernel has
 * completed.  A preceding kernel that signals griddepcontrol.launch_dependents
 * early must therefore not write `trellis` after it signals.  Replaces vllm_exl3_c.exl3_gemv / exl3_gemm
 * (recipe-lna/lna2/bindings.cpp:104-109,135-148), exllamav3_ext.exl3_gemm
 * (recipe-lna/exllamav3/exl3_gemm.cu.lna:336-348) and
 * BC_LinearEXL3.run_alloc as called by LinearEXL3.forward
 * (recipe-lna/exllamav3/exl3.py.lna:114-139).
 * k, n multiples of 128; K in 1..8; x row-major with leading dimension k,
 * y row-major with leading dimension n.  Any rows >= 1 (processed in blocks
 * of 32 rows).  `scratch` is a device buffer of at least
 * exl3_linear_scratch_bytes(rows, k, n, K) bytes whose first
 * EXL3_LINEAR_CTRL_BYTES bytes are zero before first use; the kernel leaves
 * them zero again.  One launch at a time per scratch buffer. */
#define EXL3_LINEAR_CTRL_BYTES 4096
int64_t exl3_linear_scratch_bytes(int64_t rows, int64_t k, int64_t n, int K);
int exl3_linear(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t n,
                const void* trellis, int K, int cb, const void* suh, const void* svh,
                void* y, int y_dtype, void* scratch, int64_t scratch_bytes, int precise,
                void* stream);

/* Grouped dense linear: nmat (1..8) EXL3 matrices applied to the same input
 * rows in one launch, y_j[rows, n[j]] = x[rows, k] . W_j -- every matrix with
 * its own trellis [k/16, n[j]/16, 16K], suh [k], svh [n[j]] and output y[j]
 * (row-major, leading dimension n[j]); one k, K and codebook for the group.
 * Replaces exllamav3_ext.exl3_mgemm with a broadcast input (bszm_in = 1,
 * per-matrix suh / svh / width / output pointer:
 * recipe-lna/exllamav3/exl3_gemm.cu.lna:659-679, called by the plugin's
 * dense groups at recipe-lna/vllm_exl3_exl3.py.lna:546-613).  The k-chunked
 * units of all matrices share one ticket counter, so a group of small
 * matrices fills the GPU like one wide matrix.  Matrices that take the
 * tensor-core path (>= 64 rows) run one after another on it.  `scratch`:
 * >= exl3_linear_group_scratch_bytes(rows, k, nmat, n, K) bytes, first
 * EXL3_LINEAR_CTRL_BYTES zero before first use (left zero); sum of n[j] up to
 * 120,832.  `n`, `trellis`, `suh`, `svh` and `y` are host arrays of nmat
 * entries (device addresses in the pointer arrays). */
int64_t exl3_linear_group_scratch_bytes(int64_t rows, int64_t k, int nmat, const int64_t* n, int K);
int exl3_linear_group(const void* x, int x_dtype, int64_t rows, int64_t k, int nmat, const int64_t* n,
                      const void* const* trellis, int K, int cb, const void* const* suh, const void* const* svh,
                      void* const* y, int y_dtype, void* scratch, int64_t scratch_bytes, int precise, void* stream);

/* ------------------------------------------------------------------ routed MoE
 * One routed-expert decode layer on one rank (TP shard of the intermediate
 * dim): for every valid (row, slot), expert e = ids[row, slot]:
 *   g = x . Wgate_e, u = x . Wup_e            (fp32, output transform applied)
 *   a = fp16( silu(min(g, L)) * clamp(u, -L, L) )
 *   d = a . Wdown_e                           (fp32)
 *   out[row] = sum over slots, in slot order, of weights[row, slot] * d   (fp32),
 * then one cast to out_dtype.  An expert listed twice in one row is computed
 * once and added twice.  Ids outside [0, n_experts) are skipped.
 * Replaces vllm_exl3_c.lna2_moe_decode (recipe-lna/lna2/lna_moe_ticket.cu:507-581)
 * with its semantics (recipe-lna/vllm_exl3_exl3.py.lna:988-1027), generalised:
 *   - pointer tables: device int64 [n_experts] arrays of device addresses,
 *     in the reference's order gate/up/down x trellis/suh/svh; gate/up trellis
 *     [hidden/16, inter/16, 16K], down trellis [inter/16, hidden/16, 16K];
 *   - bits: k_table (device int32 [n_experts]) or, when k_table is NULL, the
 *     scalar K for all experts; kmax = largest K present (1..4);
 *   - m in 1..exl3_moe_max_rows(), topk in 1..16, m*topk <= 256,
 *     hidden and inter multiples of 128, n_experts <= 1024;
 *   - x fp16/bf16 [m, hidden]; out fp16/bf16/fp32 [m, hidden];
 *     ids int32 [m, topk]; weights fp32 [m, topk] (routing scale included).
 * `scratch`: >= exl3_moe_scratch_bytes(m, topk, hidden, inter) bytes, first
 * EXL3_MOE_CTRL_BYTES zero before first use (the kernel restores them).  One
 * launch at a time per scratch buffer.  The kernel is launched with
 * programmatic stream serialization: it may start while the previous kernel in
 * the stream is still retiring, reads only `ids` before waiting for that kernel
 * (griddepcontrol.wait), and waits before everything else.  A preceding kernel
 * that itself signals griddepcontrol.launch_dependents early must therefore
 * have written `ids` before it signals (kernels that never signal are waited
 * for in full, as without the attribute). */
#define EXL3_MOE_CTRL_BYTES 262144
int64_t exl3_moe_scratch_bytes(int64_t m, int64_t topk, int64_t hidden, int64_t inter);
/* Replaces lna2_moe_max_rows (recipe-lna/lna2/lna_moe_ticket.cu:491-492). */
int64_t exl3_moe_max_rows(void);
int exl3_moe_decode(const void* x, int x_dtype, void* out, int out_dtype,
                    int64_t m, int64_t hidden, int64_t inter,
                    const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                    const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                    const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh,
                    int64_t n_experts, const int32_t* k_table, int K, int kmax, int cb,
                    const int32_t* ids, const float* weights, int64_t topk,
                    float swiglu_limit, void* scratch, int64_t scratch_bytes, int precise,
                    void* stream);
/* Routed-MoE decode taking the router's outputs as the serving layer holds
 * them.  The reference's plugin turns them into the kernel's int32 local ids
 * and fp32 weights with torch operations before every layer -- the
 * global-to-local id mapping map_topk_to_local and the dtype casts
 * (recipe-lna/vllm_exl3_exl3.py.lna:963-987,1234-1236), three or more small
 * kernels per layer; here the kernel reads them directly:
 *   ids          device [m, topk], int32 (ids_dtype 0) or int64 (ids_dtype 1);
 *   weights      device [m, topk], fp16 / bf16 / fp32 (weights_dtype, EXL3_DTYPE_*);
 *   expert_map   NULL: ids are local expert ids; else device int64 [n_global]
 *                mapping a global id to this rank's local id, negative when
 *                the expert lives on another rank.
 * A slot is skipped when its id is negative, not below n_global (with a
 * map), mapped to a negative id, or (after mapping) not below n_experts --
 * exactly the slots map_topk_to_local sends to its sentinel.  Everything else
 * is exl3_moe_decode; tp_bufs non-NULL adds the fused tensor-parallel sum of
 * exl3_moe_decode_tp (tp_rank, tp_world, tp_max_rows as there; ignored when
 * tp_bufs is NULL). */
typedef struct exl3_moe_route {
    const void* ids;
    int ids_dtype;
    const void* weights;
    int weights_dtype;
    const int64_t* expert_map;
    int64_t n_global;
} exl3_moe_route;
int exl3_moe_decode_routed(const void* x, int x_dtype, void* out, int out_dtype,
                           int64_t m, int64_t hidden, int64_t inter,
                           const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                           const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                           const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh,
                           int64_t n_experts, const int32_t* k_table, int K, int kmax, int cb,
                           const exl3_moe_route* route, int64_t topk, float swiglu_limit,
                           void* scratch, int64_t scratch_bytes, int precise,
                           const int64_t* tp_bufs, int tp_rank, int tp_world, int64_t tp_max_rows,
                           void* stream);
/* Replaces lna2_moe_prepare (recipe-lna/lna2/lna_moe_ticket.cu:494-500):
 * occupancy, grid and kernel attributes for the current device, cached, so
 * that later calls can be captured in a CUDA graph. */
int exl3_moe_prepare(int kmax);
/* Replaces lna2_moe_info (recipe-lna/lna2/lna_moe_ticket.cu:502-513): fills
 * info[14] = {sms, resident CTAs/SM, warps/CTA, grid, threads, codebook count,
 * ring stages, max rows, static smem bytes, ctrl bytes, scratch bytes for
 * (max rows, topk 8, 4096, 2048), max rows, max pairs, concurrent streams}. */
int exl3_moe_info(int kmax, int64_t* info);

/* Allocation-free variant of exl3_moe_decode.  No counterpart in the
 * reference.  For callers that cannot allocate device memory: a plugin loaded
 * into a serving process whose device memory belongs to the host's own
 * caching allocator (it may not cudaMalloc a buffer of its own, and the host
 * offers it none), and latency-critical callers that cannot take
 * cudaMalloc's implicit device-wide synchronization.  Same arguments as
 * exl3_moe_decode minus the scratch: the scratch is an 8 MiB array compiled
 * into the library (EXL3_MOE_STATIC_SCRATCH_BYTES), held on every GPU that
 * loads the library until the process exits.  Geometries whose
 * exl3_moe_scratch_bytes() exceeds it are rejected with EXL3_ERR_ARG (8 MiB
 * covers m <= 16 rows at top-8, hidden 4096, intermediate 256, and m <= 4 at
 * intermediate 2048).  Each call clears the array's control region with
 * cudaMemsetAsync on `stream` (the rest is fully written before it is read),
 * then launches; the memset sits between consecutive layers, so these calls
 * do not get the programmatic launch overlap of exl3_moe_decode.  The first
 * call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current), remembers it for the
 * process, and should come before any stream capture; after
 * cudaDeviceReset the remembered address is stale and this entry point must
 * not be used again in that process.  All calls on a device share the one
 * array, which keeps the last call's contents: calls that can overlap on the
 * GPU (different streams without ordering) race and must not be issued. */
#define EXL3_MOE_STATIC_SCRATCH_BYTES (8 << 20)
int exl3_moe_decode_noalloc(const void* x, int x_dtype, void* out, int out_dtype,
                            int64_t m, int64_t hidden, int64_t inter,
                            const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                            const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                            const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh,
                            int64_t n_experts, const int32_t* k_table, int K, int kmax, int cb,
                            const int32_t* ids, const float* weights, int64_t topk,
                            float swiglu_limit, int precise, void* stream);

/* ------------------------------------------------------------------ fused TP sum
 * exl3_moe_decode with the tensor-parallel all-reduce of the layer output
 * done inside the kernel over NVLink peer memory, replacing the per-layer
 * NCCL all-reduce the reference runs after lna2_moe_decode
 * (recipe-lna/vllm_exl3_exl3.py.lna:855-871 shards the experts).  Every
 * rank holds one exchange buffer (exl3_tp_buffer_alloc, zeroed; its handle
 * is shared with exl3_tp_ipc_handle / exl3_tp_ipc_open) and passes the
 * device table `tp_bufs` [world] of all ranks' buffer addresses, its own
 * included.  The CTA that finishes a 128-column block of the output stores
 * this rank's partial rows into every rank's buffer, each fp32 value in one
 * 8-byte word with the launch's epoch beside it; the last CTA to retire waits
 * (bounded, 2 s) until every rank's values carry the epoch and writes the
 * fp32 sum over ranks in rank order, then one cast: every rank ends with the
 * same `out`.  Peer stores and loads only: no multicast, no NVLS.  The epoch
 * that tells launches apart lives in the buffer, so calls can be captured in
 * a CUDA graph.  All ranks must make the same sequence of calls with the
 * same m and routes; a rank that does not arrive sets status bit 0 on the
 * others after 2 s.  m <= tp_max_rows (the buffers' row capacity).
 * No counterpart in the reference, which calls NCCL after its kernel. */
int64_t exl3_tp_buffer_bytes(int world, int64_t max_rows, int64_t hidden);
int exl3_tp_buffer_alloc(int world, int64_t max_rows, int64_t hidden, void** out);
int exl3_tp_buffer_free(void* buffer);
/* cudaIpcMemHandle_t of a buffer (64 bytes) / mapping of a peer's buffer. */
int exl3_tp_ipc_handle(void* buffer, void* handle64);
int exl3_tp_ipc_open(const void* handle64, void** out);
int exl3_tp_ipc_close(void* mapped);
int exl3_moe_decode_tp(const void* x, int x_dtype, void* out, int out_dtype,
                       int64_t m, int64_t hidden, int64_t inter,
                       const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                       const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                       const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh,
                       int64_t n_experts, const int32_t* k_table, int K, int kmax, int cb,
                       const int32_t* ids, const float* weights, int64_t topk,
                       float swiglu_limit, void* scratch, int64_t scratch_bytes, int precise,
                       const int64_t* tp_bufs, int tp_rank, int tp_world, int64_t tp_max_rows,
                       void* stream);

/* ------------------------------------------------------------------ prefill MoE
 * The routed-expert layer of exl3_moe_decode for many rows (prefill chunks)
 * on the tcgen05 tensor cores: same arguments and semantics (gate / up / down
 * multiply the fp16-rounded decoded weights the reference returns, i.e. the
 * precise arithmetic), any m >= 1.  The route plan (the argsort / count glue
 * of the reference's prefill branch) is built on the device, and calls with
 * more than exl3_moe_prefill_chunk_tokens(n_experts) tokens (2048 at 256
 * experts, the reference's TEMP_ROWS_FUSED) are processed in chunks of that
 * many tokens, one after another on `stream`.  Bits: K1..K4 (k_table or K).
 * Replaces the fused prefill launch exllamav3_ext.exl3_moe
 * (orders/F1-ref/exl3_moe.cu:99-301) and its plugin glue
 * (recipe-lna/vllm_exl3_exl3.py.lna:1597-1704).
 * `scratch`: >= exl3_moe_prefill_scratch_bytes(m, topk, hidden, inter,
 * n_experts) bytes; nothing in it needs clearing.  One launch at a time per
 * scratch buffer.  Its status word (exl3_scratch_status(scratch, 1, ...))
 * reports the last call. */
int64_t exl3_moe_prefill_scratch_bytes(int64_t m, int64_t topk, int64_t hidden, int64_t inter, int64_t n_experts);
int64_t exl3_moe_prefill_chunk_tokens(int64_t n_experts);
int exl3_moe_prefill(const void* x, int x_dtype, void* out, int out_dtype,
                     int64_t m, int64_t hidden, int64_t inter,
                     const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                     const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                     const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh,
                     int64_t n_experts, const int32_t* k_table, int K, int kmax, int cb,
                     const int32_t* ids, const float* weights, int64_t topk,
                     float swiglu_limit, void* scratch, int64_t scratch_bytes, void* stream);
/* exl3_moe_prefill with the routing inputs of exl3_moe_decode_routed (int32 or
 * int64 ids, optional expert map, fp16 / bf16 / fp32 weights), read by the
 * device route plan directly instead of after the plugin's torch mapping and
 * casts (recipe-lna/vllm_exl3_exl3.py.lna:963-987,1617-1629). */
int exl3_moe_prefill_routed(const void* x, int x_dtype, void* out, int out_dtype,
                            int64_t m, int64_t hidden, int64_t inter,
                            const int64_t* gate_trellis, const int64_t* gate_suh, const int64_t* gate_svh,
                            const int64_t* up_trellis, const int64_t* up_suh, const int64_t* up_svh,
                            const int64_t* down_trellis, const int64_t* down_suh, const int64_t* down_svh,
                            int64_t n_experts, const int32_t* k_table, int K, int kmax, int cb,
                            const exl3_moe_route* route, int64_t topk, float swiglu_limit,
                            void* scratch, int64_t scratch_bytes, void* stream);

/* Decode-issue roof: runs the GEMV engine's decode inner loop (window
 * extraction, codebook, split-accumulator MMAs) on 32 weight tiles held in
 * shared memory, with no global traffic, on a grid of 2 CTAs x 8 decoding
 * warps per SM (the MoE kernel's occupancy), `iters` rounds of 8 k-slices per
 * warp.  `words`: device uint32 [>= 32 * 8 * K], any bits (a tile's words);
 * `out`: device float [>= exl3_decode_roof_out_floats()] (per-thread sums, so
 * the work is not optimised away).  *weights_decoded receives the number of
 * weights the launch decodes; time the launch on `stream` to get the rate.
 * Counterpart of the reference's null-decode build, which removed the decode
 * instead of the memory traffic (LNA2_NULL_DECODE,
 * recipe-lna/lna2/lna_gemv_core.cuh:31-32,170). */
int64_t exl3_decode_roof_out_floats(void);
int exl3_decode_roof(int K, int cb, int iters, const void* words, int64_t words_len, float* out, int64_t out_len,
                     int64_t* weights_decoded, void* stream);

/* Device status word of a scratch buffer (MoE or linear): bit 0 dependency
 * wait timed out, bit 1 misaligned trellis pointer, bit 2 bit width out of
 * range, bit 3 ring wait timed out, bit 4 route plan overflow.  Synchronizes
 * `stream`; not for use during graph capture.  clear != 0 resets the word.
 * No counterpart in the reference, whose kernels cannot report errors. */
int exl3_scratch_status(void* scratch, int is_moe, int clear, uint32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif
