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

// The staged contraction, for shapes that tile exactly (modes a multiple of 32, batch and cout of
// 16, 16-byte aligned arrays). A CTA computes 32 modes x 16 outputs x 16 samples: warp w takes
// outputs (w % 2) 8 .. +8 and samples (w / 2) 4 .. +4 for the 32 modes of its lanes. The inputs it
// needs, x[16 samples][i][32 modes] and w[i][16 outputs][32 modes], are runs of 32 complex values
// (256 bytes) that cp.async copies into shared memory four input channels at a time, double-
// buffered, so the loads of channels i + 4 .. i + 7 are in flight while channels i .. i + 3 are
// multiplied. Each weight is read into shared memory once per 16 samples (the direct kernel reads
// it once per 4), and no load latency sits in the multiply loop. The sum over channels runs in
// the same order with the same operations as the direct kernel.
constexpr int kStagedModes = 32;
constexpr int kStagedOut = 16;
constexpr int kStagedBatch = 16;
constexpr int kStagedIc = 4;
constexpr int kStagedStage = kStagedIc * (kStagedBatch + kStagedOut) * kStagedModes;  // float2

__device__ __forceinline__ void cp_async16(void* dst, const void* src)
{
    const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(256, 2)
    contract_staged_kernel(const float2* __restrict__ x, const float2* __restrict__ w,
                           float2* __restrict__ out, int cin, int cout, long long modes)
{
    wait_for_previous_grid();
    allow_next_grid();
    extern __shared__ float4 smem_raw[];
    float2* stages = reinterpret_cast<float2*>(smem_raw);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const long long m0 = static_cast<long long>(blockIdx.x) * kStagedModes;
    const int o_cta = blockIdx.y * kStagedOut;
    const int b_cta = blockIdx.z * kStagedBatch;
    const int ob = (warp & 1) * kOutPerThread;    // within the CTA's 16 outputs
    const int bb0 = (warp >> 1) * kBatchPerThread;  // within the CTA's 16 samples

    // Stage layout: xs[ic][16 samples][32 modes], then ws[ic][16 outputs][32 modes]. One copy is
    // 16 bytes (2 modes); a stage is kStagedStage / 2 copies, 4 per thread.
    auto issue = [&](int s, int i0) {
        float2* xs = stages + s * kStagedStage;
        float2* ws = xs + kStagedIc * kStagedBatch * kStagedModes;
        for (int e = threadIdx.x; e < kStagedStage / 2; e += blockDim.x) {
            const int mm = (e & 15) * 2;
            const int row = e >> 4;  // 0 .. ic * 32 - 1
            if (row < kStagedIc * kStagedBatch) {
                const int ic = row / kStagedBatch;
                const int b = row - ic * kStagedBatch;
                cp_async16(xs + row * kStagedModes + mm,
                           x + (static_cast<long long>(b_cta + b) * cin + i0 + ic) * modes + m0 + mm);
            } else {
                const int r = row - kStagedIc * kStagedBatch;
                const int ic = r / kStagedOut;
                const int o = r - ic * kStagedOut;
                cp_async16(ws + r * kStagedModes + mm,
                           w + (static_cast<long long>(i0 + ic) * cout + o_cta + o) * modes + m0 + mm);
            }
        }
        cp_async_commit();
    };

    float2 acc[kBatchPerThread][kOutPerThread];
#pragma unroll
    for (int bb = 0; bb < kBatchPerThread; ++bb) {
#pragma unroll
        for (int oo = 0; oo < kOutPerThread; ++oo) {
            acc[bb][oo] = make_float2(0.0f, 0.0f);
        }
    }
    const int chunks = cin / kStagedIc;
    issue(0, 0);
    for (int k = 0; k < chunks; ++k) {
        if (k + 1 < chunks) {
            issue((k + 1) & 1, (k + 1) * kStagedIc);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // chunk k is in shared memory for every thread
        const float2* xs = stages + (k & 1) * kStagedStage;
        const float2* ws = xs + kStagedIc * kStagedBatch * kStagedModes;
#pragma unroll
        for (int ic = 0; ic < kStagedIc; ++ic) {
            float2 xv[kBatchPerThread];
            float2 wv[kOutPerThread];
#pragma unroll
            for (int bb = 0; bb < kBatchPerThread; ++bb) {
                xv[bb] = xs[(ic * kStagedBatch + bb0 + bb) * kStagedModes + lane];
            }
#pragma unroll
            for (int oo = 0; oo < kOutPerThread; ++oo) {
                wv[oo] = ws[(ic * kStagedOut + ob + oo) * kStagedModes + lane];
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
        __syncthreads();  // chunk k's buffer is free for chunk k + 2
    }
#pragma unroll
    for (int bb = 0; bb < kBatchPerThread; ++bb) {
#pragma unroll
        for (int oo = 0; oo < kOutPerThread; ++oo) {
            out[(static_cast<long long>(b_cta + bb0 + bb) * cout + o_cta + ob + oo) * modes + m0 + lane] =
                acc[bb][oo];
        }
    }
}

// SPECTRAL_CONTRACT_AUTO takes the tensor-core kernel wherever it fits the shape: at the FNO
// configuration (64 x 64 channels, 512 modes, 64 samples) it measured 27.5 us against 45.6 us for
// the staged FP32 kernel, both within the FP32 tolerance.
constexpr bool kAutoTensor = true;

bool staged_fits(const void* x, const void* w, long long batch, int cin, int cout, long long modes)
{
    const auto aligned = [](const void* p) { return (reinterpret_cast<unsigned long long>(p) & 15u) == 0; };
    return modes % kStagedModes == 0 && batch % kStagedBatch == 0 && cout % kStagedOut == 0
           && cin % kStagedIc == 0 && aligned(x) && aligned(w) && modes / kStagedModes <= 0x7fffffff
           && cout / kStagedOut <= 65535 && batch / kStagedBatch <= 65535;
}

}  // namespace

// The tensor-core contraction (contract_tc.cu).
bool contract_tc_fits(const void* x, const void* w, const void* out, long long batch, int cin, int cout,
                      long long modes);
void contract_tc(const float2* x, const float2* w, float2* out, long long batch, int cin, int cout,
                 long long modes, cudaStream_t stream);

}  // namespace spectral

namespace {

int mode_contract(const void* x, const void* w, void* out, long long batch, int cin, int cout, long long modes,
                  int method, void* stream)
{
    using namespace spectral;
    if (batch < 0 || cin < 1 || cout < 1 || modes < 0 || batch > (1LL << 30)) {
        set_last_error("mode_contract: need batch >= 0, cin >= 1, cout >= 1, modes >= 0");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    if (method < SPECTRAL_CONTRACT_AUTO || method > SPECTRAL_CONTRACT_TENSOR) {
        set_last_error("mode_contract: method must be SPECTRAL_CONTRACT_AUTO, _FP32 or _TENSOR");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    if (((reinterpret_cast<unsigned long long>(x) | reinterpret_cast<unsigned long long>(w)
          | reinterpret_cast<unsigned long long>(out)) & 7u) != 0) {
        set_last_error("mode_contract: arrays must be 8-byte aligned");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    const bool tc_fits = contract_tc_fits(x, w, out, batch, cin, cout, modes);
    if (method == SPECTRAL_CONTRACT_TENSOR && !tc_fits) {
        set_last_error("mode_contract: the tensor-core method needs batch a multiple of 64, cout of 32, cin of 8 up to 256, "
                       "modes of 4 and 16-byte aligned arrays");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    if (batch == 0 || modes == 0) {
        return SPECTRAL_OK;
    }
    if (method == SPECTRAL_CONTRACT_TENSOR || (method == SPECTRAL_CONTRACT_AUTO && tc_fits && kAutoTensor)) {
        try {
            contract_tc(static_cast<const float2*>(x), static_cast<const float2*>(w), static_cast<float2*>(out),
                        batch, cin, cout, modes, static_cast<cudaStream_t>(stream));
        } catch (const std::exception& e) {
            set_last_error(e.what());
            return SPECTRAL_CUDA_ERROR;
        }
        return SPECTRAL_OK;
    }
    if (staged_fits(x, w, batch, cin, cout, modes)) {
        const dim3 sgrid(static_cast<unsigned>(modes / kStagedModes), static_cast<unsigned>(cout / kStagedOut),
                         static_cast<unsigned>(batch / kStagedBatch));
        constexpr std::size_t smem = 2 * kStagedStage * sizeof(float2);
        try {
            static std::atomic<bool> opted[kMaxDevices];
            const int device = current_device();
            if (!opted[device].load(std::memory_order_relaxed)) {
                SPECTRAL_CUDA(cudaFuncSetAttribute(contract_staged_kernel,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem)));
                opted[device].store(true, std::memory_order_relaxed);
            }
            launch_pdl(contract_staged_kernel, sgrid, dim3(256), smem, static_cast<cudaStream_t>(stream),
                       static_cast<const float2*>(x), static_cast<const float2*>(w), static_cast<float2*>(out),
                       cin, cout, modes);
        } catch (const std::exception& e) {
            set_last_error(e.what());
            return SPECTRAL_CUDA_ERROR;
        }
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

}  // namespace

extern "C" int spectral_mode_contract(const void* x, const void* w, void* out, long long batch,
                                      int cin, int cout, long long modes, void* stream)
{
    return mode_contract(x, w, out, batch, cin, cout, modes, SPECTRAL_CONTRACT_AUTO, stream);
}

extern "C" int spectral_mode_contract_method(const void* x, const void* w, void* out, long long batch,
                                             int cin, int cout, long long modes, int method, void* stream)
{
    return mode_contract(x, w, out, batch, cin, cout, modes, method, stream);
}
