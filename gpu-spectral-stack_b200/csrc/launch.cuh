#pragma once

// Launch shapes: persistent grids sized to what is resident on the device at once, with the
// occupancy query and the shared-memory opt-in done once per kernel and device.

#include "common.cuh"

#include <atomic>

namespace spectral {

constexpr int kMaxDevices = 64;

inline int current_device()
{
    int device = 0;
    SPECTRAL_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kMaxDevices) {
        throw InvalidArgument("device index out of range");
    }
    return device;
}

inline int device_sm_count(int device)
{
    static std::atomic<int> cache[kMaxDevices];
    int sms = cache[device].load(std::memory_order_relaxed);
    if (sms == 0) {
        SPECTRAL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        cache[device].store(sms, std::memory_order_relaxed);
    }
    return sms;
}

// Resident CTAs per SM for `kernel`; `cache` is the caller's per-kernel cache (one slot per
// device). Opts the kernel into more than 48 KiB of dynamic shared memory when it needs it.
inline int resident_ctas(const void* kernel, int threads, std::size_t smem, std::atomic<int>* cache,
                         int device)
{
    int per_sm = cache[device].load(std::memory_order_relaxed);
    if (per_sm == 0) {
        if (smem > 48 * 1024) {
            SPECTRAL_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem)));
        }
        SPECTRAL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem));
        if (per_sm < 1) {
            throw CudaError("kernel does not fit on one SM (threads " + std::to_string(threads)
                            + ", shared memory " + std::to_string(smem) + " bytes)");
        }
        cache[device].store(per_sm, std::memory_order_relaxed);
    }
    return per_sm;
}

// Grid of persistent CTAs for `tiles` units of work: every resident slot once, or fewer.
inline unsigned persistent_grid(const void* kernel, int threads, std::size_t smem,
                                std::atomic<int>* cache, long long tiles)
{
    const int device = current_device();
    const long long slots =
        static_cast<long long>(device_sm_count(device)) * resident_ctas(kernel, threads, smem, cache, device);
    const long long grid = tiles < slots ? tiles : slots;
    return static_cast<unsigned>(grid < 1 ? 1 : grid);
}

}  // namespace spectral
