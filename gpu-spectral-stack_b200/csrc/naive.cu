// The implementation behind the registry name "naive" (entry 0, and the default `impl` of every
// torch operator schema): a textbook radix-2 transform, one launch per stage, plus separate
// real-transform passes that need a workspace. It exists so the name keeps working as in the
// reference (csrc/fft/naive.cu, csrc/fft/real.cu:184-216); it is meant to be obviously correct,
// not fast. It has neither a column kernel nor in-kernel pruning, so the 2D transforms use the
// transpose method and the pruned ones gather from (or scatter into) full transforms.

#include "backend.hpp"
#include "simple.cuh"

namespace spectral {
namespace {

void c2c(const float2* x, float2* y, int n, long long batch, Direction d, int /*keep == n*/,
         cudaStream_t s)
{
    simple::radix2_c2c(x, y, n, batch, d, s);
}

void r2c(const float* x, float2* y, int n, long long batch, int keep, float2* work, cudaStream_t s)
{
    const int m = n / 2;
    simple::radix2_c2c(reinterpret_cast<const float2*>(x), work, m, batch, Direction::Forward, s);
    simple::r2c_post(work, y, m, batch, keep, s);
}

void c2r(const float2* x, float* y, int n, long long batch, int keep, float2* work, cudaStream_t s)
{
    const int m = n / 2;
    simple::c2r_pre(x, work, m, batch, keep, s);
    simple::radix2_c2c(work, reinterpret_cast<float2*>(y), m, batch, Direction::Inverse, s);
}

}  // namespace

const Backend kNaive = {&c2c, &r2c, &c2r, nullptr, nullptr, nullptr, nullptr};

}  // namespace spectral
