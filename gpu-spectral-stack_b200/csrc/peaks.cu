// The FP32 arithmetic ceiling of this GPU, measured: the denominator of the roofline for kernels
// bound by FP32 issue rather than by HBM (the per-mode contraction). The reference measures the
// same ceiling with a dedicated tool (csrc/tools/peaks.cu:46-70 there); here the library carries
// the kernel so that bench.py can time it with CUDA events in the same process and run as the
// transforms it is compared with.
//
// Each thread advances kChains independent recurrences a <- a * m + c (0 < m < 1, so the values
// settle instead of overflowing), kUnroll steps per loop trip. Two forms:
//   scalar  one FFMA per step and chain (2 flops);
//   packed  one FFMA2 (Blackwell's FP32x2 fused multiply-add, __ffma2_rn) per step and chain,
//           two lanes of a float2 at once (4 flops).
// The larger of the two measured rates is the FP32 ceiling. The store at the end is guarded by
// a condition the compiler cannot fold, so the arithmetic is not dead code.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "launch.cuh"

namespace spectral {
namespace {

constexpr int kChains = 8;
constexpr int kUnroll = 16;
constexpr int kCeilingThreads = 256;

template <bool Packed>
__global__ void __launch_bounds__(kCeilingThreads) fp32_ceiling_kernel(float* sink, int iters, float m, float c)
{
    float2 a[kChains];
#pragma unroll
    for (int k = 0; k < kChains; ++k) {
        a[k] = make_float2(static_cast<float>(threadIdx.x + k), static_cast<float>(blockIdx.x + k));
    }
    const float2 m2 = make_float2(m, m);
    const float2 c2 = make_float2(c, c);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
            for (int k = 0; k < kChains; ++k) {
                if constexpr (Packed) {
                    a[k] = __ffma2_rn(a[k], m2, c2);
                } else {
                    a[k].x = fmaf(a[k].x, m, c);
                }
            }
        }
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < kChains; ++k) {
        s += Packed ? a[k].x + a[k].y : a[k].x;
    }
    if (s == -1.0f) {
        sink[0] = s;
    }
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_fp32_ceiling(float* sink, int iters, int packed, void* stream, double* flops)
{
    using namespace spectral;
    try {
        if (sink == nullptr) {
            throw InvalidArgument("spectral_fp32_ceiling: sink must not be null");
        }
        if (iters < 1) {
            throw InvalidArgument("spectral_fp32_ceiling: iters must be positive");
        }
        // One full wave: every resident slot of every SM once.
        static std::atomic<int> cache_scalar[kMaxDevices];
        static std::atomic<int> cache_packed[kMaxDevices];
        const void* kernel = packed != 0 ? reinterpret_cast<const void*>(fp32_ceiling_kernel<true>)
                                         : reinterpret_cast<const void*>(fp32_ceiling_kernel<false>);
        const int device = current_device();
        const int per_sm = resident_ctas(kernel, kCeilingThreads, 0, packed != 0 ? cache_packed : cache_scalar,
                                         device);
        const unsigned grid = static_cast<unsigned>(device_sm_count(device) * per_sm);
        const auto s = static_cast<cudaStream_t>(stream);
        if (packed != 0) {
            fp32_ceiling_kernel<true><<<grid, kCeilingThreads, 0, s>>>(sink, iters, 0.999f, 0.001f);
        } else {
            fp32_ceiling_kernel<false><<<grid, kCeilingThreads, 0, s>>>(sink, iters, 0.999f, 0.001f);
        }
        SPECTRAL_CUDA(cudaGetLastError());
        if (flops != nullptr) {
            *flops = 2.0 * (packed != 0 ? 2.0 : 1.0) * kChains * kUnroll * static_cast<double>(iters)
                     * static_cast<double>(grid) * kCeilingThreads;
        }
        return SPECTRAL_OK;
    } catch (const InvalidArgument& e) {
        set_last_error(e.what());
        return SPECTRAL_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
}
