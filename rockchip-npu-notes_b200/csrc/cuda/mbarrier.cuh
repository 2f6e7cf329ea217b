// mbarrier.cuh -- shared-memory mbarrier wrappers and the bounded wait used by every pipelined
// kernel of the library (the tcgen05 GEMM and the bulk-copy GEMV).
//
// A wait polls mbarrier.try_wait.parity; every 256 polls it checks the CTA's abort flag and the
// global nanosecond timer. After WAIT_LIMIT_NS without progress it raises FLAG_TIMEOUT in the
// handle's status words, sets the abort flag and returns false, so the kernel can stop issuing
// work, drain its own copies in flight (drain_phase, also bounded) and return instead of hanging.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace b2 {

constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;   // 1 s per wait; a healthy wait is microseconds

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of parity `parity` to complete. Returns false when the CTA is aborting or
// the wait exceeded WAIT_LIMIT_NS (then the timeout flag is raised and the CTA aborts).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                           unsigned *flags) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {   // the abort flag and the clock are checked every 256 polls
            if (*abort_flag) return false;
            const uint64_t t = global_ns();
            if (!t0) {
                t0 = t;
            } else if (t - t0 > WAIT_LIMIT_NS) {
                *abort_flag = 1;
                raise_flag(flags, FLAG_TIMEOUT);
                return false;
            }
        }
    }
}
// Bounded wait used only while draining after an abort (ignores the abort flag).
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > WAIT_LIMIT_NS) return;
}

}  // namespace b2
