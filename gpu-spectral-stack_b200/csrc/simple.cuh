#pragma once

// Simple grid-stride kernels: the whole of the "naive" implementation (a textbook radix-2
// transform), and the helpers every implementation may use: a tiled batched transpose, the
// gather and scatter of pruned modes, the separate real-transform combine and prepare passes,
// and y = alpha x.

#include "common.cuh"

namespace spectral::simple {

// y = alpha x over n complex values (the reference's scale_c2c, csrc/ops/scale.cu:17-27).
void scale(const float2* x, float2* y, std::size_t n, float alpha, cudaStream_t s);

// y = the transpose of x for `batch` row-major arrays of rows x cols, back to back.
void transpose(const float2* x, float2* y, int rows, int cols, long long batch, cudaStream_t s);

// The modes of `batch` arrays of n1 x w values (m1 = 0: all n1 rows; else rows 0 .. m1-1 and
// n1-m1 .. n1-1), columns 0 .. m2-1: gather copies them out of `full`, scatter zeroes `full`
// and writes them into it.
void gather_modes(const float2* full, float2* modes, int n1, int w, int m1, int m2, long long batch,
                  cudaStream_t s);
void scatter_modes(const float2* modes, float2* full, int n1, int w, int m1, int m2,
                   long long batch, cudaStream_t s);

// The real-transform steps as separate passes: y rows of `keep` values from z = DFT_m of each
// packed row (m per row); z rows of m values prepared from x rows of `keep` values.
void r2c_post(const float2* z, float2* y, int m, long long batch, int keep, cudaStream_t s);
void c2r_pre(const float2* x, float2* z, int m, long long batch, int keep, cudaStream_t s);

// Radix-2 complex transform, out of place: a bit-reversal gather, then log2 n in-place
// butterfly stages, then 1/n for the inverse. Any power-of-two n (the "naive" implementation).
void radix2_c2c(const float2* x, float2* y, int n, long long batch, Direction d, cudaStream_t s);

}  // namespace spectral::simple
