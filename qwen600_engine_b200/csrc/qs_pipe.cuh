// Shared-memory pipeline primitives for sm_100a kernels: mbarriers with
// bounded waits.
#pragma once
#include <stdint.h>

namespace qs {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned long long* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of `parity` to complete; false if the kernel is
// aborting (honor_abort) or `limit_ns` passed (then it raises the abort flag).
// Short limits (below 1 ms, the test hook) are checked on every poll.  The
// drains that let issued copies and MMAs finish before the CTA leaves pass
// honor_abort = false: they wait for completion, bounded only by time.
__device__ inline bool mbar_wait(unsigned long long* b, uint32_t parity, volatile int* abort,
                          unsigned long long limit_ns, bool honor_abort = true) {
    if (mbar_try(b, parity)) return true;
    const unsigned long long t0 = global_ns();
    const uint32_t mask = limit_ns < 1000000ull ? 0u : 127u;
    for (uint32_t it = 1;; it++) {
        if (mbar_try(b, parity)) return true;
        if ((it & mask) == 0) {
            if (honor_abort && *abort) return false;
            if (global_ns() - t0 > limit_ns) {
                *abort = 1;
                return false;
            }
        }
    }
}
}  // namespace qs
