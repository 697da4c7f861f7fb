// The register engine with radix-8 DFT building blocks and correctly rounded twiddle tables copied from the host,
// behind the registry name "stockham_r8_table". One translation unit per variant, so the
// variants compile in parallel.

#include "backend.hpp"
#include "fields.cuh"
#include "pruned2d.cuh"

namespace spectral {
namespace {

using Rows = engine::RowEngine<8, true>;
using Cols = engine::ColumnEngine<8, true>;
using Fused = engine::Pruned2dEngine<8, true>;
using Whole = engine::FieldsEngine<8, true>;

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

const Backend kEngineR8Table = {&c2c, &Rows::r2c, &Rows::c2r, &Cols::columns, &Fused::supported,
                      &Fused::forward, &Fused::inverse,
                      &Whole::supported, &rfft2_fields, &irfft2_fields};

}  // namespace spectral
