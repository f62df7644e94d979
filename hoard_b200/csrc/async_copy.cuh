// async_copy.cuh -- mbarriers, 1-D bulk copies (cp.async.bulk, the TMA unit's untiled form) and
// bounded waits, shared by the kernels that stage expert weights into shared memory.
//
// Every wait is bounded by %globaltimer (WAIT_NS): a wait that runs out returns false, and the
// caller records an error bit in the scratch error word and leaves its loop, so that a lost copy
// or a stalled peer never hangs the GPU.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace hoard {

constexpr unsigned long long WAIT_NS = 2000000000ull;   // 2 s bound on any device-side wait

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint: a waiting warp sleeps in hardware until the phase completes
// (or the hint elapses) instead of spinning, so it takes no issue slots from the working warps.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier; false if the bound expired.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > WAIT_NS) return false;
    }
    return true;
}
// 1-D bulk copy global -> shared, completion counted on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Per-thread asynchronous copies global -> shared (cp.async): 16 bytes through L2 only, or 4 bytes.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Named barrier `id` over `nthreads` threads (a multiple of 32): syncs a subset of the CTA's warps.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace hoard
