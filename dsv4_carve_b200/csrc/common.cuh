// common.cuh -- shared device helpers for the EXL3 B200 kernels (sm_100a).
//
// mbarrier / bulk-copy wrappers (inline PTX), bounded waits, error flags, and
// the 128-point Walsh-Hadamard transform held as 4 values per lane of a warp.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace exl3 {

// ---------------------------------------------------------------- errors
// Device-side error bits, OR-ed into the scratch status word.  The kernels
// never trap: a failed check records its bit and skips the work.
enum : uint32_t {
    ERR_DEP_TIMEOUT  = 1u << 0,   // a dependency counter did not reach its target
    ERR_MISALIGNED   = 1u << 1,   // a trellis pointer is not 16-byte aligned
    ERR_BAD_K        = 1u << 2,   // per-expert bit width outside the build's range
    ERR_RING_TIMEOUT = 1u << 3,   // an mbarrier wait gave up
    ERR_PLAN         = 1u << 4,   // route plan exceeded its capacity
};

// Every spin is bounded twice: by elapsed %globaltimer time (kWaitLimitNs)
// and by an iteration cap, whichever comes first.  A wait that runs out
// records its error bit and returns false; the caller abandons its work.
constexpr uint64_t kWaitLimitNs = 2000000000ull;    // 2 s
constexpr uint32_t kSpinCap = 1u << 28;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void set_error(uint32_t* status, uint32_t bit) {
    atomicOr(status, bit);
}

__device__ __forceinline__ bool aligned16_dev(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread for up to ~20 us while the
// phase is incomplete, so a waiting warp issues almost no instructions.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 20000;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait: returns false (after recording the error) if the phase never
// completed.  Callers then abandon the CTA's remaining work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1; i < kSpinCap; ++i) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    set_error(status, ERR_RING_TIMEOUT);
    return false;
}

// Bounded wait polled by every lane of a warp (each lane gets the barrier's
// acquire ordering itself); the verdict is made warp-uniform.
__device__ __forceinline__ bool mbar_wait_lanes(uint64_t* bar, uint32_t parity, uint32_t* status) {
    bool ok = mbar_try_wait(bar, parity);
    if (!ok) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t i = 1; i < kSpinCap; ++i) {
            if (mbar_try_wait_sleep(bar, parity)) { ok = true; break; }
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && (threadIdx.x & 31) == 0) set_error(status, ERR_RING_TIMEOUT);
    return ok;
}

// Orders this thread's generic-proxy accesses to global memory with its
// async-proxy (bulk copy) accesses: used after writing data that another
// CTA's bulk copy will read, and after acquiring it before issuing the copy.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// 3-D tiled TMA load of one box into this CTA's shared memory, completion
// counted in bytes on an mbarrier; this CTA only.  The innermost coordinate
// is always 0 here (whole 16-bit tiles), so it is 16-byte aligned.
__device__ __forceinline__ void tma_load_3d(void* dst_smem, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(smem_u32(dst_smem)), "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Device-side tensor-map update: replace the global address of a tensor map
// held in shared memory (128-byte aligned), publish it to its global slot
// with the tensormap-proxy release (all 32 lanes), acquire it before use.
__device__ __forceinline__ void tmap_replace_address(void* smem_tmap, const void* gaddr) {
    asm volatile("tensormap.replace.tile.global_address.shared::cta.b1024.b64 [%0], %1;"
                 :: "r"(smem_u32(smem_tmap)), "l"(gaddr) : "memory");
}

__device__ __forceinline__ void tmap_publish(void* gmem_tmap, const void* smem_tmap) {
    asm volatile("tensormap.cp_fenceproxy.global.shared::cta.tensormap::generic.release.gpu.sync.aligned [%0], [%1], 128;"
                 :: "l"(gmem_tmap), "r"(smem_u32(smem_tmap)) : "memory");
}

__device__ __forceinline__ void tmap_acquire(const void* gmem_tmap) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" :: "l"(gmem_tmap) : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted in bytes
// on an mbarrier (plain per-CTA copy).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now / wait until the previous kernel has completed and its writes
// are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- memory
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Atomic add with release semantics at GPU scope: orders this thread's
// earlier writes (and those ordered before them by a warp or CTA barrier)
// before the increment, without a separate full fence.
__device__ __forceinline__ uint32_t atom_add_release_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Atomic add with acquire-release semantics at GPU scope: releases this
// thread's earlier writes like atom_add_release_gpu and, for the thread that
// learns from the old value that it completed a count, acquires what the
// other adders released, without a separate fence.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Add without a return value, ordered after this thread's earlier writes
// (and those a preceding warp or CTA barrier made it observe).
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Spin (bounded) until *ctr >= target.  Returns false on timeout.
__device__ __forceinline__ bool wait_counter(const uint32_t* ctr, uint32_t target, uint32_t* status) {
    if (ld_acquire_u32(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1; i < kSpinCap; ++i) {
        __nanosleep(64);
        if (ld_acquire_u32(ctr) >= target) return true;
        if ((i & 63u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    set_error(status, ERR_DEP_TIMEOUT);
    return false;
}

// ---------------------------------------------------------------- numerics
constexpr float kHadNorm = 0.088388347648318440550f;   // 1/sqrt(128)

__device__ __forceinline__ uint32_t dup_half(__half h) {
    const uint32_t b = __half_as_ushort(h);
    return b | (b << 16);
}

// 128-point natural-order (Sylvester) Walsh-Hadamard transform over a warp:
// lane l holds elements 4l..4l+3 in v[0..3].  Stages of stride 1 and 2 are in
// registers, strides 4..64 pair lane l with lane l^(stride/4).  Each output is
// the same sequence of fp32 additions as the textbook in-place butterfly with
// strides 1, 2, 4, ..., 64.
__device__ __forceinline__ void wht128_warp(float (&v)[4], int lane) {
    float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
    v[0] = a0 + a2; v[1] = a1 + a3; v[2] = a0 - a2; v[3] = a1 - a3;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = upper ? (o - v[i]) : (v[i] + o);
        }
    }
}

__device__ __forceinline__ __half load_act_half(const void* x, int dtype, int64_t i) {
    if (dtype == 0) return reinterpret_cast<const __half*>(x)[i];
    if (dtype == 1) return __float2half_rn(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]));
    return __float2half_rn(reinterpret_cast<const float*>(x)[i]);
}

__device__ __forceinline__ void store_out(void* out, int dtype, int64_t i, float v) {
    if (dtype == 0) reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
    else if (dtype == 1) reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(out)[i] = v;
}

// ---------------------------------------------------------------- routes
// Router outputs as the serving layer holds them: expert ids int32 or int64
// [m, topk], global ids when an expert map is given; routing weights fp32,
// bf16 or fp16.  The reference casts and maps them with torch before its
// kernel (recipe-lna/vllm_exl3_exl3.py.lna:963-987,1234-1236); here every
// read goes through these helpers instead.
struct RouteIn {
    const void* ids;
    const void* weights;
    const int64_t* emap;      // global id -> local id (< 0: not on this rank), or null
    int64_t n_global;         // entries of emap
    int ids64;                // 0: int32 ids, 1: int64 ids
    int w_dtype;              // 0 fp16, 1 bf16, 2 fp32
};

// Local expert of slot s, or -1 when the slot is skipped: a negative id, an
// id past the map, an id the map sends off this rank (negative), or a local
// id outside [0, E) -- the cases the reference maps to its n_local sentinel.
__device__ __forceinline__ int route_local_id(const RouteIn& r, int64_t s, int E) {
    int64_t v = r.ids64 ? reinterpret_cast<const int64_t*>(r.ids)[s] : (int64_t) reinterpret_cast<const int32_t*>(r.ids)[s];
    if (r.emap != nullptr) {
        if (v < 0 || v >= r.n_global) return -1;
        v = r.emap[v];
    }
    return (v >= 0 && v < (int64_t) E) ? (int) v : -1;
}

__device__ __forceinline__ float route_weight(const RouteIn& r, int64_t s) {
    if (r.w_dtype == 2) return reinterpret_cast<const float*>(r.weights)[s];
    if (r.w_dtype == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(r.weights)[s]);
    return __half2float(reinterpret_cast<const __half*>(r.weights)[s]);
}

}  // namespace exl3
