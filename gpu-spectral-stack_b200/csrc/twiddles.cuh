#pragma once

// Correctly rounded twiddle tables for the "_table" variants, built in double precision on the
// host and kept in device memory for the life of the process.
//
// The tables live in one statically sized __device__ pool (twiddles.cu): no cudaMalloc is ever
// made for them. Each table is built and uploaded on first use on each device, under a mutex,
// with a synchronous copy, so the first call that needs a table on a device must not be inside a
// CUDA graph capture (the same first-use behaviour as the reference's twiddle_table(),
// twiddles.cu:17-46 there).

#include "common.cuh"

namespace spectral::twiddles {

// The pass tables of plan (n, e) in the engine's layout (engine.cuh): plan_tw_entries(n, e)
// entries; entry r L + k of pass s is W_{L R}^(k r) = exp(-2 pi i k r / (L R)).
const float2* pass_table(int n, int e, bool small_last = false);

// W_{2n}^k = exp(-pi i k / n) for k = 0 .. n: n + 1 entries (real-transform combine).
const float2* half_turn(int n);

// The same two tables computed on the GPU with sincospif, the formula the kernels use when they
// fill their shared-memory tables themselves (engine.cuh: computed_pass_twiddle,
// computed_half_turn). Kernels that read their tables from global memory use these for the
// computed-twiddle variants. Built by a kernel on first use per device, then synchronised.
const float2* pass_table_computed(int n, int e, bool small_last = false);
const float2* half_turn_computed(int n);

// W_total^j = exp(-2 pi i j / total) for j = 0 .. count-1 (the four-step inter-pass factors are
// products of two such tables).
const float2* turn(long long total, int count);

// The row-DFT operand of the tensor-core pruned forward (pruned_tc.cu): the first m (<= 16)
// outputs of n-point real rows as 64 rows of n TF32 values, cos(2 pi k j / n) and
// -sin(2 pi k j / n) for k = 0 .. 15 (zero for k >= m), each split into a hi part (the value
// rounded to TF32) and a lo part (the rest, rounded to TF32): rows 0-15 cos hi, 16-31 -sin hi,
// 32-47 cos lo, 48-63 -sin lo. Stored in the tensor core's canonical K-major layout without
// swizzle: value (row b, j) at float (j / 4) 256 + (b / 8) 32 + (b % 8) 4 + j % 4, i.e. core
// matrices of 8 rows x 16 bytes, 128 bytes apart along the rows and 1 KiB apart along j.
// 64 n floats, returned as float2 storage.
constexpr int kTf32DftOutputs = 16;
const float2* tf32_dft_rows(int n, int m);

// The row operand of the tensor-core pruned inverse (pruned_tc.cu): for output position j of an
// n-point real row (n <= 256), 32 TF32 values cos(2 pi k j / n) (k = 0 .. 15), then
// sin(2 pi k j / n) (k = 0 .. 15); rows 0 .. n-1 hold the hi parts, rows n .. 2n-1 the lo parts.
// Canonical K-major layout without swizzle: value (row b, kk) at float
// (kk / 4) (2n / 8) 32 + (b / 8) 32 + (b % 8) 4 + kk % 4. 64 n floats, returned as float2 storage.
const float2* tf32_idft_rows(int n);

}  // namespace spectral::twiddles
