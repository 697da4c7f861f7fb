#pragma once

// Bulk asynchronous copies (the Blackwell/Hopper TMA engine's non-tensor form) from global to
// shared memory, completed through an mbarrier, and the bounded waits on them.
//
// cp.async.bulk needs 16-byte aligned source and destination addresses and a size that is a
// multiple of 16 bytes; callers check that on the host. The copies here are never multicast to
// other CTAs of a cluster, and their sources are always this GPU's own memory.
//
// Every wait is bounded: mbar_wait gives up after kSpinLimit polls (each poll already suspends
// for a hardware-chosen time), and the kernel then records a fault code in a device word that
// the host reads with spectral_device_faults(), instead of spinning forever.

#include "common.cuh"

#include <cstdint>

namespace spectral::tma {

constexpr unsigned kSpinLimit = 1u << 22;

// Fault codes, OR-ed into the fault word.
constexpr unsigned kFaultWaitTimeout = 1u;
constexpr unsigned kFaultDrainTimeout = 2u;  // the wait for an abandoned copy also gave up

__device__ __forceinline__ unsigned smem_addr(const void* p)
{
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes the initialisation visible to the async proxy (the bulk-copy engine).
__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy accesses to shared memory before later async-proxy
// writes (a bulk copy into a buffer the CTA has just finished reading).
__device__ __forceinline__ void fence_proxy_async()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// One bulk copy of `bytes` from global `src` to shared `dst`, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity)
{
    unsigned ok = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Completes `bytes` of the current phase's expected transaction count without a copy: what a
// copy that will never come would have delivered. Used to drain a phase after a wait gave up.
__device__ __forceinline__ void mbar_complete_tx(uint64_t* bar, unsigned bytes)
{
    asm volatile("mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Waits for phase `parity` of `bar` to complete; false if it did not within `limit` polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned limit = kSpinLimit)
{
    for (unsigned i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) {
            return true;
        }
    }
    return false;
}

}  // namespace spectral::tma

namespace spectral {

// The device fault word of the current device (faults.cu): kernels OR fault codes into it.
unsigned* device_fault_word();

}  // namespace spectral
