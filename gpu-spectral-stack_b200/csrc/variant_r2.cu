// The register engine with radix-2 DFT building blocks and twiddles computed on chip with sincospif,
// behind the registry name "stockham_r2". One translation unit per variant, so the
// variants compile in parallel.

#include "backend.hpp"
#include "fields.cuh"
#include "pruned2d.cuh"

namespace spectral {
namespace {

using Rows = engine::RowEngine<2, false>;
using Cols = engine::ColumnEngine<2, false>;
using Fused = engine::Pruned2dEngine<2, false>;
using Whole = engine::FieldsEngine<2, false>;

void rfft2_fields(const float* x, float2* y, float2* scratch, int n1, int n2, long long fields,
                  cudaStream_t s)
{
    Whole::run<true>(reinterpret_cast<const float2*>(x), y, scratch, n1, n2, fields, s);
}

void irfft2_fields(const float2* y, float* x, float2* scratch, int n1, int n2, long long fields,
                   cudaStream_t s)
{
    Whole::run<false>(y, reinterpret_cast<float2*>(x), scratch, n1, n2, fields, s);
}

void c2c(const float2* x, float2* y, int n, long long batch, Direction d, int keep, cudaStream_t s)
{
    if (n <= engine::kMaxRowN) {
        Rows::c2c(x, y, n, batch, d, keep, s);
    } else {
        Cols::fourstep(x, y, n, batch, d, s);
    }
}

}  // namespace

const Backend kEngineR2 = {&c2c, &Rows::r2c, &Rows::c2r, &Cols::columns, &Fused::supported,
                      &Fused::forward, &Fused::inverse,
                      &Whole::supported, &rfft2_fields, &irfft2_fields};

}  // namespace spectral
