#pragma once

// Shared pieces of every kernel in this library: the complex value type, complex arithmetic,
// compile-time integer helpers, and the error types the C-ABI layer turns into status codes.
//
// A complex64 value is two packed floats (re, im), the layout of c10::complex<float>, of
// numpy's complex64, and of the reference's `cf32` (csrc/common/types.hpp:7-12). Kernels use
// CUDA's `float2` for it, which is 8-byte aligned, so every complex load or store is one 64-bit
// access, and row starts are always aligned for it (the real-transform rows of n/2 + 1 values
// are 8-byte but not 16-byte aligned).

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace spectral {

enum class Direction { Forward, Inverse };

// Thrown for shapes, sizes and arguments the library does not accept. The C-ABI maps it to
// SPECTRAL_INVALID_ARGUMENT, and the torch shim turns that into std::invalid_argument
// (Python ValueError), as the reference's drivers do.
struct InvalidArgument : std::invalid_argument {
    using std::invalid_argument::invalid_argument;
};

// Thrown when a CUDA runtime call fails. Maps to SPECTRAL_CUDA_ERROR (Python RuntimeError).
struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

[[noreturn]] inline void throw_cuda(cudaError_t err, const char* call, const char* file, int line)
{
    throw CudaError(std::string("CUDA error: ") + cudaGetErrorString(err) + " (code "
                    + std::to_string(static_cast<int>(err)) + ")\n  in: " + call + "\n  at: "
                    + file + ":" + std::to_string(line));
}

#define SPECTRAL_CUDA(call)                                                                    \
    do {                                                                                       \
        const cudaError_t spectral_err_ = (call);                                              \
        if (spectral_err_ != cudaSuccess) {                                                    \
            ::spectral::throw_cuda(spectral_err_, #call, __FILE__, __LINE__);                  \
        }                                                                                      \
    } while (0)

__host__ __device__ constexpr int ilog2(int n)
{
    int r = 0;
    while ((1 << r) < n) {
        ++r;
    }
    return r;
}

__host__ __device__ constexpr bool is_pow2(long long n) { return n >= 1 && (n & (n - 1)) == 0; }

__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }

// --- complex arithmetic on float2 -------------------------------------------------------------

// Complex addition, subtraction and real scaling use Blackwell's packed FP32x2 instructions
// (FADD2 / FFMA2 / FMUL2 through CUDA's __fadd2_rn, __ffma2_rn, __fmul2_rn): one instruction
// per complex operation instead of two, with the same IEEE rounding as the scalar forms.
// a - b is fma(b, -1, a): the product is exact, so the single rounding is that of a - b.
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 csub(float2 a, float2 b)
{
    return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a);
}
// Programmatic dependent launch: a kernel launched with the programmatic-serialization
// attribute may start while the previous kernel on its stream drains; it waits here, before its
// first global access, until that kernel has completed and its writes are visible. Launched
// without the attribute, the wait returns at once.
__device__ __forceinline__ void wait_for_previous_grid()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next kernel on the stream begin launching (it still waits for this one to complete).
__device__ __forceinline__ void allow_next_grid()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float2 cscale(float2 a, float s) { return __fmul2_rn(a, make_float2(s, s)); }

// a * w for the forward transform, a * conj(w) for the inverse: twiddle tables hold the forward
// factors exp(-2 pi i m / M), and the inverse transform uses their conjugates.
template <bool Inv>
__device__ __forceinline__ float2 cmul_tw(float2 a, float2 w)
{
    if constexpr (Inv) {
        return make_float2(fmaf(a.x, w.x, a.y * w.y), fmaf(a.y, w.x, -(a.x * w.y)));
    } else {
        return make_float2(fmaf(a.x, w.x, -(a.y * w.y)), fmaf(a.y, w.x, a.x * w.y));
    }
}

// a * b, plain complex product.
__device__ __forceinline__ float2 cmul(float2 a, float2 b)
{
    return make_float2(fmaf(a.x, b.x, -(a.y * b.y)), fmaf(a.y, b.x, a.x * b.y));
}

}  // namespace spectral
