#pragma once

// The internal interface of one FFT implementation: what a registry entry (registry.cpp) calls.
// It is the B200 counterpart of the reference's function-pointer table (csrc/fft/fft.hpp:14-83,
// csrc/fft/registry.hpp:14-25): the same operations, with the size and argument checks done
// once, in the C-ABI layer, before any of these run.

#include "common.cuh"

#include <string>

namespace spectral {

struct Backend {
    // `batch` complex rows of n points (a power of two, 2 .. 4096 for the engines). keep
    // (1 .. n) prunes the frequency side: forward writes the first keep outputs per row, inverse
    // reads keep inputs per row (the rest zero). Inverse divides by n.
    void (*c2c)(const float2* x, float2* y, int n, long long batch, Direction d, int keep,
                cudaStream_t s);
    // `batch` real rows of n points to rows of keep (1 .. n/2 + 1) values. `work` (batch n/2
    // complex values) is used only by implementations without a fused real kernel.
    void (*r2c)(const float* x, float2* y, int n, long long batch, int keep, float2* work,
                cudaStream_t s);
    // Rows of keep (1 .. n/2 + 1) values, the rest zero, to real rows of n points, divided by n.
    void (*c2r)(const float2* x, float* y, int n, long long batch, int keep, float2* work,
                cudaStream_t s);
    // Columns: `slabs` row-major arrays of n rows by `cols` columns, each column one n-point
    // transform, in place when x == y (unpruned only). m1_in > 0: arrays of x hold only the
    // 2 m1_in rows of frequencies 0 .. m1_in-1 and n-m1_in .. n-1 (the rest zero); m1_out > 0:
    // arrays of y keep only those 2 m1_out rows. Inverse divides by n. nullptr when the
    // implementation has no column kernel.
    void (*columns)(const float2* x, float2* y, int n, int cols, long long slabs, int m1_in,
                    int m1_out, Direction d, cudaStream_t s);
    // The pruned 2D real transforms in one kernel per direction, with the intermediate on chip
    // (pruned2d.cuh), for the shapes `pruned2d_supported` accepts; nullptr when there are none.
    bool (*pruned2d_supported)(int n1, int n2, int m1, int m2);
    void (*rfft2_modes)(const float* x, float2* modes, int n1, int n2, int m1, int m2,
                        long long fields, cudaStream_t s);
    void (*irfft2_modes)(const float2* modes, float* y, int n1, int n2, int m1, int m2,
                         long long fields, cudaStream_t s);
};

// The register engine in its four registry variants (variant_*.cu) and the simple reference-
// style implementation behind the name "naive" (naive.cu).
extern const Backend kEngineR2;
extern const Backend kEngineR4;
extern const Backend kEngineR8;
extern const Backend kEngineR8Table;
extern const Backend kNaive;

// Records the calling thread's error message for spectral_last_error() (capi.cu).
void set_last_error(const std::string& message);

// The strided-column complex-to-real 2D transform with a caller-given workspace of
// `work_values` complex values, checked and run as spectral_fft2_c2r does (capi.cu); returns a
// status code.
int run_fft2_c2r_strided(const char* impl, const void* x, float* y, int n1, int n2,
                         long long batch, float2* work, std::size_t work_values, void* stream);

// The pruned 2D real transforms of 128 x 128 fields with their row stage on the tensor cores
// (pruned_tc.cu): fit when n1 = n2 = 128, m2 <= 16, the real array (x forward, y inverse) is
// 16-byte aligned and fields * 128 rows address with 32-bit coordinates. Same mode layout as
// Backend::rfft2_modes / irfft2_modes.
bool pruned_tc_fits(const void* real, int n1, int n2, int m1, int m2, long long fields);
void pruned_tc_forward(const float* x, float2* modes, int m1, int m2, long long fields, cudaStream_t stream);
// The inverse: the columns by the FFT engine, the real rows as a GEMM on the tensor cores.
void pruned_tc_inverse(const float2* modes, float* y, int m1, int m2, long long fields, cudaStream_t stream);

}  // namespace spectral
