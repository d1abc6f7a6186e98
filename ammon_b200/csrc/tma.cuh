// TMA (cp.async.bulk.tensor) and mbarrier helpers for sm_100a kernels.
//
// Loads are plain tensor copies into the issuing CTA's own shared memory, so the same
// code is safe in multi-GPU processes. Every wait is bounded by %globaltimer.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace ab {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Arrive once and announce `bytes` of transactions for the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(phase)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Limit of every bounded wait. The runtime's flag block holds it as a u64 (nanoseconds) at
// byte 8, behind the flag word (ab_runtime_set_wait_limit; 0 = the default of 2 s). A wait
// reads it only once it has lasted kWaitFloorNs, so waits that end sooner cost no load.
constexpr uint64_t kWaitDefaultNs = 2000000000ull;
constexpr uint64_t kWaitFloorNs = 1000000ull;
__device__ __forceinline__ uint64_t wait_limit_ns(const uint32_t* flags) {
    const uint64_t v = flags ? *reinterpret_cast<const volatile uint64_t*>(flags + 2) : 0;
    return v ? v : kWaitDefaultNs;
}

// Tracks one bounded wait: expired() is true once the wait has lasted the flag block's limit
// (and at least kWaitFloorNs).
struct WaitClock {
    uint64_t t0;
    uint64_t limit = kWaitFloorNs;
    bool read = false;
    __device__ __forceinline__ WaitClock() : t0(global_timer_ns()) {}
    __device__ __forceinline__ bool expired(const uint32_t* flags) {
        const uint64_t dt = global_timer_ns() - t0;
        if (dt <= limit) return false;
        if (read) return true;
        read = true;
        limit = wait_limit_ns(flags);
        return dt > limit;
    }
};

// Waits for phase `phase` of the barrier, giving up after the flag block's limit (returns
// false).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t phase,
                                                  const uint32_t* flags) {
    if (mbar_try_wait(bar, phase)) return true;
    WaitClock clock;
    while (!mbar_try_wait(bar, phase))
        if (clock.expired(flags)) return false;
    return true;
}

// 2-D tiled tensor load into this CTA's shared memory, completing on `bar`.
// x is the innermost coordinate (elements); x * element size must be 16-byte aligned.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Byte offset within a TMA-swizzled tile (SWZ = 32, 64 or 128 byte span, tile base
// aligned to 1024 bytes): 16-byte chunk index bits [4, 4+log2(SWZ/16)) are XORed with
// address bits [7, ...), the CU_TENSOR_MAP_SWIZZLE_<SWZ>B pattern.
template <int SWZ>
__device__ __forceinline__ uint32_t swizzle_off(uint32_t off) {
    constexpr uint32_t mask = SWZ / 16 - 1;
    return off ^ (((off >> 7) & mask) << 4);
}

}  // namespace ab
