// The register engine with radix-8 DFT building blocks and twiddles computed on chip with sincospif,
// behind the registry name "stockham_r8". One translation unit per variant, so the
// variants compile in parallel.

#include "backend.hpp"
#include "pruned2d.cuh"

namespace spectral {
namespace {

using Rows = engine::RowEngine<8, false>;
using Cols = engine::ColumnEngine<8, false>;
using Fused = engine::Pruned2dEngine<8, false>;

void c2c(const float2* x, float2* y, int n, long long batch, Direction d, int keep, cudaStream_t s)
{
    if (n <= engine::kMaxRowN) {
        Rows::c2c(x, y, n, batch, d, keep, s);
    } else {
        Cols::fourstep(x, y, n, batch, d, s);
    }
}

}  // namespace

const Backend kEngineR8 = {&c2c, &Rows::r2c, &Rows::c2r, &Cols::columns, &Fused::supported,
                      &Fused::forward, &Fused::inverse};

}  // namespace spectral
