// The device fault word: a kernel whose bounded wait gave up ORs a code into it (tma.cuh) and
// returns, so a stuck copy never hangs the GPU. spectral_device_faults() reads (and optionally
// clears) it for the current device.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "launch.cuh"
#include "tma.cuh"

#include <mutex>

namespace spectral {
namespace {

__device__ unsigned g_fault_word;

std::mutex g_mutex;
unsigned* g_words[64] = {};

}  // namespace

unsigned* device_fault_word()
{
    int device = 0;
    SPECTRAL_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= 64) {
        throw InvalidArgument("device index out of range");
    }
    const std::lock_guard<std::mutex> lock(g_mutex);
    if (g_words[device] == nullptr) {
        void* p = nullptr;
        SPECTRAL_CUDA(cudaGetSymbolAddress(&p, g_fault_word));
        g_words[device] = static_cast<unsigned*>(p);
    }
    return g_words[device];
}

}  // namespace spectral

extern "C" int spectral_device_faults(unsigned* faults, int clear)
{
    using namespace spectral;
    try {
        unsigned value = 0;
        SPECTRAL_CUDA(cudaMemcpyFromSymbol(&value, g_fault_word, sizeof(value)));
        if (clear != 0 && value != 0) {
            const unsigned zero = 0;
            SPECTRAL_CUDA(cudaMemcpyToSymbol(g_fault_word, &zero, sizeof(zero)));
        }
        if (faults != nullptr) {
            *faults = value;
        }
        return SPECTRAL_OK;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
}

// --- the bounded-wait path, exercised on purpose ------------------------------------------------
//
// One CTA of 64 threads copies 1 KiB into shared memory with one bulk copy completing on an
// mbarrier, exactly as the staged row kernel does, and waits for it with the same bounded wait.
// With `missing` > 0 the barrier is armed for `missing` bytes more than the copy delivers, so its
// phase cannot complete: the wait gives up after `spin_limit` polls and records
// SPECTRAL_FAULT_WAIT_TIMEOUT, as a lost copy would make a production kernel do. The probe then
// completes the missing bytes itself, so the phase completes once the real copy has landed, and
// waits for that (bounded too, recording SPECTRAL_FAULT_DRAIN_TIMEOUT if it also gives up), so no
// copy is in flight when the CTA exits. Every thread finally writes its 16 bytes of the staged
// tile to `dst`. Nothing faults, traps or spins without a limit.

namespace spectral {
namespace {

constexpr int kProbeThreads = 64;
constexpr unsigned kProbeBytes = kProbeThreads * 16;

__global__ void __launch_bounds__(kProbeThreads)
    wait_probe_kernel(const float4* __restrict__ src, float4* __restrict__ dst, unsigned missing,
                      unsigned spin_limit, unsigned* fault)
{
    __shared__ alignas(16) float4 tile[kProbeThreads];
    __shared__ alignas(8) uint64_t bar;
    if (threadIdx.x == 0) {
        tma::mbar_init(&bar, 1);
        tma::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        tma::mbar_arrive_expect_tx(&bar, kProbeBytes + missing);
        tma::bulk_g2s(tile, src, kProbeBytes, &bar);
        if (!tma::mbar_wait(&bar, 0, spin_limit)) {
            atomicOr(fault, tma::kFaultWaitTimeout);
            tma::mbar_complete_tx(&bar, missing);
            if (!tma::mbar_wait(&bar, 0)) {
                atomicOr(fault, tma::kFaultDrainTimeout);
            }
        }
    }
    __syncthreads();
    dst[threadIdx.x] = tile[threadIdx.x];
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_probe_bounded_wait(const void* src, void* dst, unsigned missing_bytes,
                                           unsigned spin_limit, void* stream)
{
    using namespace spectral;
    try {
        if (src == nullptr || dst == nullptr) {
            throw InvalidArgument("spectral_probe_bounded_wait: src and dst must not be null");
        }
        if ((reinterpret_cast<unsigned long long>(src) & 15u) != 0
            || (reinterpret_cast<unsigned long long>(dst) & 15u) != 0) {
            throw InvalidArgument("spectral_probe_bounded_wait: src and dst must be 16-byte aligned");
        }
        if (missing_bytes % 16u != 0 || missing_bytes > (1u << 20)) {
            throw InvalidArgument("spectral_probe_bounded_wait: missing_bytes must be a multiple of 16 "
                                  "and at most 1 MiB");
        }
        if (spin_limit == 0) {
            throw InvalidArgument("spectral_probe_bounded_wait: spin_limit must be positive");
        }
        wait_probe_kernel<<<1, kProbeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const float4*>(src), static_cast<float4*>(dst), missing_bytes, spin_limit,
            device_fault_word());
        SPECTRAL_CUDA(cudaGetLastError());
        return SPECTRAL_OK;
    } catch (const InvalidArgument& e) {
        set_last_error(e.what());
        return SPECTRAL_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
}
