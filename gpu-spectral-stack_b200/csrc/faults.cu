// The device fault word: a kernel whose bounded wait gave up ORs a code into it (tma.cuh) and
// returns, so a stuck copy never hangs the GPU. spectral_device_faults() reads (and optionally
// clears) it for the current device.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
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
