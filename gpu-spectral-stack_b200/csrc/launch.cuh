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

// Launches `kernel` with programmatic dependent launch allowed: it may be scheduled while the
// previous kernel on the stream drains, which hides the launch gap between back-to-back
// transforms. The kernel must call griddepcontrol.wait (engine.cuh: wait_for_previous_grid)
// before its first global memory access; launched after a kernel that does not trigger early,
// that wait simply lasts until the previous kernel completes.
template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, std::size_t smem,
                cudaStream_t stream, Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SPECTRAL_CUDA(cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...));
}

}  // namespace spectral
