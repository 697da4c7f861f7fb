// spectral_fft2_c2r_noalloc: the complex-to-real 2D transform for callers that cannot allocate
// device memory.
//
// spectral_fft2_c2r needs a workspace (the strided method transforms the columns out of place,
// since it may not overwrite its input). Most callers allocate it. Some cannot: a plugin whose
// host framework owns every device allocation and hands it only input and output buffers, a
// real-time loop that must never enter the CUDA allocator (cudaMalloc can synchronize the device
// and take milliseconds), or a foreign-language binding that has device pointers but no
// allocator. For them this entry point takes its workspace from a fixed array compiled into the
// library, so it calls no cudaMalloc, cudaFree or allocating library routine.
//
// The array holds kScratchValues complex values (32 MiB) on every GPU that loads the library,
// for the life of the process. Transforms whose workspace (batch * n1 * (n2/2 + 1) values) does
// not fit are rejected with SPECTRAL_INVALID_ARGUMENT. Every call on a device shares the array:
// calls whose work overlaps on that GPU (another stream, another host thread) race on it, so a
// caller must serialise them. The array keeps the last call's contents; the column pass writes
// every value it later reads, so nothing needs clearing between calls.
//
// Host code may not pass the array's symbol to a kernel: on the host it names a host-side shadow,
// not device memory. The first call on each device therefore looks up the device address with
// cudaGetSymbolAddress (with that device current) and keeps it; that first call should come
// before any stream capture.

#include "../../include/spectral_b200.h"

#include "backend.hpp"

#include <mutex>

namespace spectral {
namespace {

constexpr std::size_t kScratchValues = SPECTRAL_NOALLOC_SCRATCH_VALUES;

static __device__ __align__(256) float2 g_noalloc_scratch[kScratchValues];

std::mutex g_scratch_mutex;
float2* g_scratch_ptr[64] = {};

// The device address of this device's scratch array, looked up once per device.
float2* device_scratch()
{
    int device = 0;
    SPECTRAL_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= 64) {
        throw InvalidArgument("fft2_c2r_noalloc: device index out of range");
    }
    const std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_ptr[device] == nullptr) {
        void* p = nullptr;
        SPECTRAL_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_scratch_ptr[device] = static_cast<float2*>(p);
    }
    return g_scratch_ptr[device];
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_fft2_c2r_noalloc(const char* impl, const void* x, float* y, int n1, int n2,
                                         long long batch, void* stream)
{
    using namespace spectral;
    // The size limit is checked before any CUDA call, so an oversized request fails cleanly.
    const long long w = n2 >= 2 ? n2 / 2 + 1 : 0;
    if (n1 < 1 || n2 < 2 || batch < 1) {
        set_last_error("fft2_c2r_noalloc: need n1 >= 1, n2 >= 2 and batch >= 1");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    const long double needed = static_cast<long double>(batch) * n1 * w;
    if (needed > static_cast<long double>(kScratchValues)) {
        set_last_error("fft2_c2r_noalloc: batch * n1 * (n2/2 + 1) = "
                       + std::to_string(static_cast<unsigned long long>(needed))
                       + " complex values of workspace exceed the built-in scratch array of "
                       + std::to_string(kScratchValues)
                       + " values; use spectral_fft2_c2r with a caller workspace");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    float2* scratch = nullptr;
    try {
        scratch = device_scratch();
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
    return run_fft2_c2r_strided(impl, x, y, n1, n2, batch, scratch, kScratchValues, stream);
}
