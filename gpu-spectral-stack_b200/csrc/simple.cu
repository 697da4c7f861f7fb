// Simple grid-stride kernels (see simple.cuh).

#include "simple.cuh"

#include "engine.cuh"
#include "launch.cuh"

#include <algorithm>

namespace spectral::simple {
namespace {

constexpr int kBlock = 256;

unsigned grid_for(long long threads)
{
    const int device = current_device();
    const long long cap = static_cast<long long>(device_sm_count(device)) * 16;
    const long long blocks = (threads + kBlock - 1) / kBlock;
    return static_cast<unsigned>(std::max(1LL, std::min(blocks, cap)));
}

__global__ void scale_kernel(const float2* __restrict__ x, float2* __restrict__ y, std::size_t n,
                             float alpha)
{
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
        const float2 v = x[i];
        y[i] = make_float2(alpha * v.x, alpha * v.y);
    }
}

// The same for 16-byte aligned arrays: two complex values per 16-byte access, four accesses in
// flight per thread before its stores. x and y may be the same array (each value is read and then
// written by the same thread), so the loads are ordinary ones, not the read-only path.
__device__ __forceinline__ float4 scale4(float4 v, float alpha)
{
    const float2 lo = __fmul2_rn(make_float2(v.x, v.y), make_float2(alpha, alpha));
    const float2 hi = __fmul2_rn(make_float2(v.z, v.w), make_float2(alpha, alpha));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__global__ void scale_pairs_kernel(const float4* x, float4* y, std::size_t pairs, float alpha)
{
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < pairs; i += 4 * stride) {
        const float4 a = x[i];
        const float4 b = x[i + stride];
        const float4 c = x[i + 2 * stride];
        const float4 d = x[i + 3 * stride];
        y[i] = scale4(a, alpha);
        y[i + stride] = scale4(b, alpha);
        y[i + 2 * stride] = scale4(c, alpha);
        y[i + 3 * stride] = scale4(d, alpha);
    }
    for (; i < pairs; i += stride) {
        y[i] = scale4(x[i], alpha);
    }
}

// 64 x 64 tiles through shared memory, one extra column so that a warp's column reads of the
// tile spread over the banks. A CTA of 32 x 8 threads moves a tile with 16 loads per thread, all
// issued before the first store, and walks the tiles of the batch with a grid stride. Reads and
// writes are runs of 32 consecutive values (256 bytes) per warp.
constexpr int kTile = 64;
constexpr int kTileRows = 8;

__global__ void __launch_bounds__(32 * kTileRows)
    transpose_kernel(const float2* __restrict__ x, float2* __restrict__ y, int rows, int cols, long long batch)
{
    wait_for_previous_grid();
    allow_next_grid();
    __shared__ float2 tile[kTile][kTile + 1];
    const long long size = static_cast<long long>(rows) * cols;
    const int tiles_x = (cols + kTile - 1) / kTile;
    const int tiles_y = (rows + kTile - 1) / kTile;
    const long long per = static_cast<long long>(tiles_x) * tiles_y;
    const int tx = threadIdx.x;
    const int ty = threadIdx.y;
    for (long long g = blockIdx.x; g < per * batch; g += gridDim.x) {
        const long long b = g / per;
        const int t = static_cast<int>(g - b * per);
        const int r0 = (t / tiles_x) * kTile;
        const int c0 = (t - (t / tiles_x) * tiles_x) * kTile;
        const float2* xs = x + b * size;
        float2* ys = y + b * size;
        float2 v[2][kTile / kTileRows];
#pragma unroll
        for (int k = 0; k < kTile / kTileRows; ++k) {
            const int r = r0 + ty + k * kTileRows;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int c = c0 + tx + 32 * h;
                v[h][k] = (r < rows && c < cols) ? xs[static_cast<long long>(r) * cols + c] : make_float2(0.0f, 0.0f);
            }
        }
#pragma unroll
        for (int k = 0; k < kTile / kTileRows; ++k) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                tile[ty + k * kTileRows][tx + 32 * h] = v[h][k];
            }
        }
        __syncthreads();
        // Output row c0 + j holds input column c0 + j; its values are the tile's column j.
#pragma unroll
        for (int k = 0; k < kTile / kTileRows; ++k) {
            const int j = ty + k * kTileRows;
            const int c_out = c0 + j;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r_out = r0 + tx + 32 * h;
                if (c_out < cols && r_out < rows) {
                    ys[static_cast<long long>(c_out) * rows + r_out] = tile[tx + 32 * h][j];
                }
            }
        }
        __syncthreads();
    }
}

// Index in `full` (arrays of n1 x w) of mode e of `modes` (arrays of rows x m2).
__device__ __forceinline__ long long full_index(long long e, int n1, int w, int m1, int m2)
{
    const int rows = m1 > 0 ? 2 * m1 : n1;
    const long long per = static_cast<long long>(rows) * m2;
    const long long b = e / per;
    const int rem = static_cast<int>(e - b * per);
    const int r = rem / m2;
    const int c = rem - r * m2;
    const int row = (m1 > 0 && r >= m1) ? r + (n1 - rows) : r;
    return (b * n1 + row) * static_cast<long long>(w) + c;
}

__global__ void gather_kernel(const float2* __restrict__ full, float2* __restrict__ modes, int n1,
                              int w, int m1, int m2, long long total)
{
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += stride) {
        modes[e] = full[full_index(e, n1, w, m1, m2)];
    }
}

__global__ void scatter_kernel(const float2* __restrict__ modes, float2* __restrict__ full, int n1,
                               int w, int m1, int m2, long long total)
{
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += stride) {
        full[full_index(e, n1, w, m1, m2)] = modes[e];
    }
}

// W_{2m}^k, rounded once from double precision.
__device__ __forceinline__ float2 half_turn(int k, int m)
{
    double sn = 0.0;
    double cs = 1.0;
    sincospi(static_cast<double>(k) / static_cast<double>(m), &sn, &cs);
    return make_float2(static_cast<float>(cs), static_cast<float>(-sn));
}

__global__ void r2c_post_kernel(const float2* __restrict__ z, float2* __restrict__ y, int m,
                                int keep, long long total)
{
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += stride) {
        const long long t = e / keep;
        const int k = static_cast<int>(e - t * keep);
        const float2* row = z + t * m;
        y[e] = engine::r2c_combine(row[k & (m - 1)], row[(m - k) & (m - 1)], half_turn(k, m));
    }
}

__global__ void c2r_pre_kernel(const float2* __restrict__ x, float2* __restrict__ z, int m,
                               int keep, long long total)
{
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const float2 zero = make_float2(0.0f, 0.0f);
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += stride) {
        const long long t = e / m;
        const int k = static_cast<int>(e - t * m);
        const float2* row = x + t * keep;
        float2 xk = k < keep ? row[k] : zero;
        float2 xmk = m - k < keep ? row[m - k] : zero;
        if (k == 0) {
            xk.y = 0.0f;
            xmk.y = 0.0f;
        }
        z[e] = engine::c2r_prepare(xk, xmk, half_turn(k, m));
    }
}

// y[base + i] = x[base + bitreverse(i)] within each transform of 2^log2n values.
__global__ void bit_reverse_kernel(const float2* __restrict__ x, float2* __restrict__ y,
                                   long long total, int log2n)
{
    const long long mask = (1LL << log2n) - 1;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += stride) {
        const long long base = e & ~mask;
        const unsigned i = static_cast<unsigned>(e & mask);
        const unsigned r = log2n == 0 ? 0u : (__brev(i) >> (32 - log2n));
        y[e] = x[base + r];
    }
}

// One in-place decimation-in-time stage: blocks of 2h from blocks of h, twiddle W_{2h}^k rounded
// once from double precision.
__global__ void radix2_stage_kernel(float2* y, long long butterflies, int log2h, bool inverse)
{
    const long long h = 1LL << log2h;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
         b < butterflies; b += stride) {
        const long long k = b & (h - 1);
        const long long i0 = ((b >> log2h) << (log2h + 1)) | k;
        const long long i1 = i0 + h;
        double sn = 0.0;
        double cs = 1.0;
        sincospi(static_cast<double>(k) / static_cast<double>(h), &sn, &cs);
        const float2 w = make_float2(static_cast<float>(cs), static_cast<float>(inverse ? sn : -sn));
        const float2 u = y[i0];
        const float2 v = cmul(y[i1], w);
        y[i0] = cadd(u, v);
        y[i1] = csub(u, v);
    }
}

}  // namespace

void scale(const float2* x, float2* y, std::size_t n, float alpha, cudaStream_t s)
{
    if (n == 0) {
        return;
    }
    const auto a16 = [](const void* p) { return (reinterpret_cast<unsigned long long>(p) & 15u) == 0; };
    if (a16(x) && a16(y) && n >= 2) {
        const std::size_t pairs = n / 2;
        const int device = current_device();
        const unsigned grid = static_cast<unsigned>(
            std::max<long long>(1, std::min<long long>(static_cast<long long>((pairs + kBlock - 1) / kBlock),
                                                       static_cast<long long>(device_sm_count(device)) * 8)));
        scale_pairs_kernel<<<grid, kBlock, 0, s>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y),
                                                   pairs, alpha);
        SPECTRAL_CUDA(cudaGetLastError());
        if (n % 2 != 0) {
            scale_kernel<<<1, 32, 0, s>>>(x + n - 1, y + n - 1, 1, alpha);
            SPECTRAL_CUDA(cudaGetLastError());
        }
        return;
    }
    scale_kernel<<<grid_for(static_cast<long long>(n)), kBlock, 0, s>>>(x, y, n, alpha);
    SPECTRAL_CUDA(cudaGetLastError());
}

void transpose(const float2* x, float2* y, int rows, int cols, long long batch, cudaStream_t s)
{
    if (batch <= 0 || rows <= 0 || cols <= 0) {
        return;
    }
    const dim3 block(32, kTileRows);
    const long long tiles = static_cast<long long>((cols + kTile - 1) / kTile) * ((rows + kTile - 1) / kTile) * batch;
    const long long cap = static_cast<long long>(device_sm_count(current_device())) * 6;  // resident: 6 CTAs of 33 KB per SM
    const dim3 grid(static_cast<unsigned>(std::min(tiles, cap)));
    launch_pdl(transpose_kernel, grid, block, 0, s, x, y, rows, cols, batch);
}

void gather_modes(const float2* full, float2* modes, int n1, int w, int m1, int m2, long long batch,
                  cudaStream_t s)
{
    const long long total = batch * (m1 > 0 ? 2 * m1 : n1) * static_cast<long long>(m2);
    if (total == 0) {
        return;
    }
    gather_kernel<<<grid_for(total), kBlock, 0, s>>>(full, modes, n1, w, m1, m2, total);
    SPECTRAL_CUDA(cudaGetLastError());
}

void scatter_modes(const float2* modes, float2* full, int n1, int w, int m1, int m2,
                   long long batch, cudaStream_t s)
{
    SPECTRAL_CUDA(cudaMemsetAsync(full, 0,
                                  static_cast<std::size_t>(batch) * n1 * w * sizeof(float2), s));
    const long long total = batch * (m1 > 0 ? 2 * m1 : n1) * static_cast<long long>(m2);
    if (total == 0) {
        return;
    }
    scatter_kernel<<<grid_for(total), kBlock, 0, s>>>(modes, full, n1, w, m1, m2, total);
    SPECTRAL_CUDA(cudaGetLastError());
}

void r2c_post(const float2* z, float2* y, int m, long long batch, int keep, cudaStream_t s)
{
    const long long total = batch * keep;
    r2c_post_kernel<<<grid_for(total), kBlock, 0, s>>>(z, y, m, keep, total);
    SPECTRAL_CUDA(cudaGetLastError());
}

void c2r_pre(const float2* x, float2* z, int m, long long batch, int keep, cudaStream_t s)
{
    const long long total = batch * m;
    c2r_pre_kernel<<<grid_for(total), kBlock, 0, s>>>(x, z, m, keep, total);
    SPECTRAL_CUDA(cudaGetLastError());
}

void radix2_c2c(const float2* x, float2* y, int n, long long batch, Direction d, cudaStream_t s)
{
    const long long total = static_cast<long long>(n) * batch;
    const int log2n = ilog2(n);
    bit_reverse_kernel<<<grid_for(total), kBlock, 0, s>>>(x, y, total, log2n);
    SPECTRAL_CUDA(cudaGetLastError());
    for (int st = 0; st < log2n; ++st) {
        radix2_stage_kernel<<<grid_for(total / 2), kBlock, 0, s>>>(y, total / 2, st,
                                                                   d == Direction::Inverse);
        SPECTRAL_CUDA(cudaGetLastError());
    }
    if (d == Direction::Inverse) {
        scale(y, y, static_cast<std::size_t>(total), 1.0f / static_cast<float>(n), s);
    }
}

}  // namespace spectral::simple
