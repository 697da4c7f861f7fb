// The per-mode channel contraction of an FNO spectral convolution:
//   out[b, o, m] = sum_i x[b, i, m] w[i, o, m]
// over complex values, for every kept mode m. The reference plans it (docs/ROADMAP.md:71-76,
// tasks 3.3-3.6) but has no implementation; the oracle is a float64 einsum.
//
// The mode index is the fastest-varying one in all three arrays, so lane = mode: every load and
// store of a warp is 32 consecutive complex values (256 bytes). A CTA is 32 modes by 8 warps;
// warp w owns 8 output channels, and each thread accumulates a 4 (batch) x 8 (channel) block of
// one mode in registers, 32 complex multiply-adds (128 FMAs) per 12 loads. The block is sized so
// two CTAs fit per SM (an 8 x 8 block took 204 registers and left one). x is re-read by the 8
// warps of a CTA through L1, w once per batch group through L2. FP32 throughout, so the
// contraction keeps the tolerance of the transforms around it.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "launch.cuh"

#include <string>

namespace spectral {
namespace {

constexpr int kModesPerCta = 32;
constexpr int kWarps = 8;
constexpr int kBatchPerThread = 4;
constexpr int kOutPerThread = 8;

__global__ void __launch_bounds__(kModesPerCta * kWarps, 2)
    contract_kernel(const float2* __restrict__ x, const float2* __restrict__ w,
                    float2* __restrict__ out, int batch, int cin, int cout, long long modes)
{
    wait_for_previous_grid();
    allow_next_grid();
    const long long m = static_cast<long long>(blockIdx.x) * kModesPerCta + (threadIdx.x & 31);
    const int warp = threadIdx.x >> 5;
    const int b0 = blockIdx.y * kBatchPerThread;
    const int o0 = (blockIdx.z * kWarps + warp) * kOutPerThread;
    if (m >= modes || o0 >= cout) {
        return;
    }
    float2 acc[kBatchPerThread][kOutPerThread];
#pragma unroll
    for (int bb = 0; bb < kBatchPerThread; ++bb) {
#pragma unroll
        for (int oo = 0; oo < kOutPerThread; ++oo) {
            acc[bb][oo] = make_float2(0.0f, 0.0f);
        }
    }
    for (int i = 0; i < cin; ++i) {
        float2 xv[kBatchPerThread];
        float2 wv[kOutPerThread];
#pragma unroll
        for (int bb = 0; bb < kBatchPerThread; ++bb) {
            const int b = b0 + bb;
            xv[bb] = b < batch ? __ldg(x + (static_cast<long long>(b) * cin + i) * modes + m)
                               : make_float2(0.0f, 0.0f);
        }
#pragma unroll
        for (int oo = 0; oo < kOutPerThread; ++oo) {
            const int o = o0 + oo;
            wv[oo] = o < cout ? __ldg(w + (static_cast<long long>(i) * cout + o) * modes + m)
                              : make_float2(0.0f, 0.0f);
        }
#pragma unroll
        for (int bb = 0; bb < kBatchPerThread; ++bb) {
#pragma unroll
            for (int oo = 0; oo < kOutPerThread; ++oo) {
                float2& a = acc[bb][oo];
                a.x = fmaf(xv[bb].x, wv[oo].x, fmaf(-xv[bb].y, wv[oo].y, a.x));
                a.y = fmaf(xv[bb].x, wv[oo].y, fmaf(xv[bb].y, wv[oo].x, a.y));
            }
        }
    }
#pragma unroll
    for (int bb = 0; bb < kBatchPerThread; ++bb) {
        const int b = b0 + bb;
#pragma unroll
        for (int oo = 0; oo < kOutPerThread; ++oo) {
            const int o = o0 + oo;
            if (b < batch && o < cout) {
                out[(static_cast<long long>(b) * cout + o) * modes + m] = acc[bb][oo];
            }
        }
    }
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_mode_contract(const void* x, const void* w, void* out, long long batch,
                                      int cin, int cout, long long modes, void* stream)
{
    using namespace spectral;
    if (batch < 0 || cin < 1 || cout < 1 || modes < 0 || batch > (1LL << 30)) {
        set_last_error("mode_contract: need batch >= 0, cin >= 1, cout >= 1, modes >= 0");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    if (batch == 0 || modes == 0) {
        return SPECTRAL_OK;
    }
    const dim3 grid(static_cast<unsigned>((modes + kModesPerCta - 1) / kModesPerCta),
                    static_cast<unsigned>((batch + kBatchPerThread - 1) / kBatchPerThread),
                    static_cast<unsigned>((cout + kWarps * kOutPerThread - 1) / (kWarps * kOutPerThread)));
    if (grid.y > 65535 || grid.z > 65535) {
        set_last_error("mode_contract: batch or cout too large for one launch");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    try {
        launch_pdl(contract_kernel, grid, dim3(kModesPerCta * kWarps), 0, static_cast<cudaStream_t>(stream),
                   static_cast<const float2*>(x), static_cast<const float2*>(w), static_cast<float2*>(out),
                   static_cast<int>(batch), cin, cout, modes);
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
    return SPECTRAL_OK;
}
