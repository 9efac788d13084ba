// gw_async.cuh — mbarrier, bulk-copy and bounded-wait helpers shared by the
// warp-specialised kernels (gw_grouped.cu, gw_stream.cu).
#pragma once

#include <stdint.h>

namespace gw {

constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at the B200's clocks

__device__ __forceinline__ uint32_t saddr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
// True once the phase with `parity` has completed.
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void bar_arrive_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes)
                 : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tcgen05.mma operands).
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Contiguous global -> shared copy of `bytes` (multiple of 16, both ends
// 16-byte aligned), counted on `b` as it lands.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(b))
        : "memory");
}
// All threads of one role group (the 128 epilogue threads) agree on a flag.
__device__ __forceinline__ bool group_any(bool v, int id, int n) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void group_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Bounded wait; false when the CTA is winding down (this wait ran out, or
// another role's did).
static __device__ __noinline__ bool wait_slow(int* abort_flag, uint64_t* b, uint32_t parity, unsigned* status,
                                       unsigned bit, long long limit = kWaitCycles) {
    const long long t0 = clock64();
    volatile int* ab = abort_flag;
    for (uint32_t i = 1;; ++i) {
        if (bar_try(b, parity)) return true;
        if ((i & 63) == 0) {
            if (*ab) return false;
            if (clock64() - t0 > limit) {
                *ab = 1;
                if (status) atomicOr(status, bit);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool wait_on(int* abort_flag, uint64_t* b, uint32_t parity, unsigned* status,
                                        unsigned bit) {
    return bar_try(b, parity) || wait_slow(abort_flag, b, parity, status, bit);
}
// The same, waited for by lane 0 for its whole warp.
__device__ __forceinline__ bool warp_wait(int* abort_flag, uint64_t* b, uint32_t parity, unsigned* status,
                                          unsigned bit) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = wait_on(abort_flag, b, parity, status, bit);
    return __shfl_sync(0xffffffffu, ok, 0);
}

}  // namespace gw
