// f3s_ptx.cuh -- inline-PTX building blocks for sm_100a: mbarriers, TMA bulk
// tensor loads, ldmatrix, mma.sync, the global timer, and the bounded wait
// every kernel in this library uses instead of an unbounded spin.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "fused3s.h"

namespace f3s {

// Device-side error reporting.  Word 0 of `abort` is a per-launch flag that
// tells every CTA to stop; `status` keeps the first error code until the host
// reads it.
struct ErrorSink {
    int* abort;
    int* status;
};

__device__ __forceinline__ void raise_error(const ErrorSink& e, int code) {
    atomicCAS(e.status, 0, code);
    atomicExch(e.abort, 1);
}

__device__ __forceinline__ int load_volatile(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive once `dep` is available: `dep` is first stored to a scratch word in
// shared memory, and a store cannot issue before the instructions that
// produced its value (e.g. ldmatrix loads from the buffer this arrive frees)
// have written their registers.
__device__ __forceinline__ void mbar_arrive_after(uint32_t bar, uint32_t sink, uint32_t dep) {
    asm volatile(
        "st.shared.b32 [%1], %2;\n\t"
        "mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar),
        "r"(sink), "r"(dep)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete, but never forever:
// give up when another thread has raised the abort flag, or after
// `timeout_ns` of global time (then raise F3S_ERR_TIMEOUT).  Returns false on
// give-up.  The result is made warp-uniform by the caller where needed.
static __device__ __noinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, const ErrorSink e,
                                               uint64_t timeout_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (load_volatile(e.abort)) return false;
        if (global_timer_ns() - t0 > timeout_ns) {
            raise_error(e, F3S_ERR_TIMEOUT);
            return false;
        }
    }
}

// Acquire load / release store of a flag in global memory (GPU scope): the
// reader of a flag set with st_release_gpu sees every write the setter made
// before it.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Strong (relaxed, GPU scope) 16-byte load: coherent at GPU scope, never
// served from a stale copy in this SM's L1.
__device__ __forceinline__ float4 ld_relaxed_gpu_f4(const float4* p) {
    float4 v;
    asm volatile("ld.relaxed.gpu.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag == want (set by another CTA with st_release_gpu); bounded
// by the global timer and the abort flag like every wait in the library.
static __device__ __noinline__ bool flag_wait_bounded(const int* flag, int want, const ErrorSink e,
                                                      uint64_t timeout_ns) {
    if (ld_acquire_gpu(flag) == want) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (ld_acquire_gpu(flag) == want) return true;
        if (load_volatile(e.abort)) return false;
        if (global_timer_ns() - t0 > timeout_ns) {
            raise_error(e, F3S_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(256);
    }
}

// Short bounded wait that ignores the abort flag: used on the abort path to
// let this CTA's own bulk copies land before it exits.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > timeout_ns) return;
}

// -------------------------------------------------------------------- TMA --
// Tiled bulk-tensor loads global -> shared, completion counted on an
// mbarrier in bytes, carrying an L2 eviction-priority policy (createpolicy
// below).  No multicast form is used anywhere in this library.
__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ------------------------------------------------------- warp-level MMA ---
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).  A register-only
// operation (not volatile): the compiler may schedule it freely.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
        " {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D(16x8 f32) = A(16x16 f16, row) * B(16x8 f16, col), accumulator zero.
__device__ __forceinline__ void mma_16816_zero(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
    const float z = 0.f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
        " {%8, %9}, {%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of the 16-byte chunk `chunk` of 128-byte row `row` inside a
// tile written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (tile base aligned to
// 1024 bytes): the chunk index is XORed with the row index modulo 8.
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace f3s
