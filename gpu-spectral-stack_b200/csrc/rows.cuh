#pragma once

// Row transforms (contiguous rows) of one engine variant: the plan per size, and the launchers
// that the per-variant translation units (variant_*.cu) instantiate.
//
// A variant is (B, Table): B = 2, 4 or 8 is the DFT building block (dft.cuh), Table says
// whether the twiddle tables are copied from the correctly rounded host tables (true) or
// computed on chip (false).

#include "engine.cuh"
#include "launch.cuh"
#include "twiddles.cuh"

namespace spectral::engine {

// Points per thread for a transform of n points. Large E means few passes and few shared-memory
// exchanges, but more registers: 32 points keep one transform of up to 1024 points inside one
// warp with a single exchange; beyond that 16 points keep register use low enough for several
// CTAs per SM while three passes cover 4096 points.
__host__ __device__ constexpr int default_e(int n)
{
    return n <= 16 ? n : n <= 64 ? 8 : n <= 256 ? 16 : n <= 1024 ? 32 : n <= 8192 ? 16 : 32;
}

// Threads per CTA (the CTA holds THREADS / P transforms). Measured on B200 at 2^24 points per
// call: for 1024 and 2048 points, 128-thread CTAs (4 and 1 transforms) leave more CTAs per SM
// than 256-thread ones, whose twiddle tables and buffers fill shared memory; that beats larger
// CTAs by 7-10 %.
__host__ __device__ constexpr int default_threads(int n)
{
    return (n == 1024 || n == 2048) ? 128 : kMinThreads;
}

template <int N>
using PlanFor = Plan<N, default_e(N), false, default_threads(N)>;

// The inverse complex transform of 1024 points measured fastest with 256-thread CTAs (51 us
// against 56 us with 128 threads at 2^24 points), unlike the forward one.
__host__ __device__ constexpr int inverse_threads(int n) { return n == 1024 ? 256 : default_threads(n); }

template <int N>
using PlanForInv = Plan<N, default_e(N), false, inverse_threads(N)>;

// The plan with the small radix last, for the mirror-paired real-to-complex rows.
template <int N>
using PlanR2c = Plan<N, default_e(N), true, default_threads(N)>;

// Complex rows: the bulk-copy prefetch pays where a transform spans several warps; for 1024
// points (one warp per transform, 4 CTAs of 4 transforms per SM) direct loads measured 10 %
// faster than the staged kernel, whose second buffer halves the CTAs that fit.
__host__ __device__ constexpr bool stage_c2c(int n) { return n >= 2048; }

template <class PL, bool Inv, int B, bool Table, class Io>
void launch_rows(const Io& io, long long batch, cudaStream_t stream, const float2* extra_table)
{
    if (batch <= 0) {
        return;
    }
    auto kernel = row_kernel<PL, Inv, B, Table, Io>;
    constexpr std::size_t smem = row_smem_bytes<PL, Io>();
    static std::atomic<int> cache[kMaxDevices];
    const float2* tw = Table ? twiddles::pass_table(PL::N, PL::E, PL::SmallLast) : nullptr;
    const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel), PL::THREADS, smem,
                                          cache, (batch + PL::G - 1) / PL::G);
    kernel<<<grid, PL::THREADS, smem, stream>>>(io, batch, tw, extra_table);
    SPECTRAL_CUDA(cudaGetLastError());
}

// The staged kernel (bulk-copy prefetch, engine.cuh) for sizes where it pays, when the input
// satisfies cp.async.bulk's rules: a 16-byte aligned source and whole 16-byte tiles.
constexpr int kMinStagedN = 64;

inline bool aligned16(const void* p) { return (reinterpret_cast<unsigned long long>(p) & 15u) == 0; }

template <class PL, bool Inv, int B, bool Table, class Io>
void launch_rows_staged(const Io& io, long long batch, cudaStream_t stream, const float2* extra_table)
{
    if (batch <= 0) {
        return;
    }
    auto kernel = staged_row_kernel<PL, Inv, B, Table, Io>;
    constexpr std::size_t smem = staged_smem_bytes<PL, Io>();
    static_assert(smem <= 227 * 1024, "staged tile does not fit in shared memory");
    static std::atomic<int> cache[kMaxDevices];
    const float2* tw = Table ? twiddles::pass_table(PL::N, PL::E, PL::SmallLast) : nullptr;
    const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel), PL::THREADS, smem,
                                          cache, (batch + PL::G - 1) / PL::G);
    kernel<<<grid, PL::THREADS, smem, stream>>>(io, batch, tw, extra_table, device_fault_word());
    SPECTRAL_CUDA(cudaGetLastError());
}

// Calls f(std::integral_constant<int, n>) for a power of two n in [Lo, Hi], else throws.
template <int Lo, int Hi, class F>
void dispatch_pow2(int n, F&& f)
{
    if constexpr (Lo <= Hi) {
        if (n == Lo) {
            f(std::integral_constant<int, Lo>{});
            return;
        }
        dispatch_pow2<Lo * 2, Hi>(n, static_cast<F&&>(f));
    } else {
        throw InvalidArgument("unsupported transform size " + std::to_string(n));
    }
}

constexpr int kMaxRowN = 4096;  // largest row transform held by one CTA

template <int B, bool Table>
struct RowEngine {
    // `batch` complex rows of n points (2 <= n <= 4096). keep (1 .. n) prunes the frequency side:
    // a forward transform writes only the first keep outputs per row, an inverse one reads only
    // the first keep inputs per row (the rest are zero). The inverse divides by n.
    static void c2c(const float2* x, float2* y, int n, long long batch, Direction d, int keep,
                    cudaStream_t s)
    {
        dispatch_pow2<2, kMaxRowN>(n, [&](auto n_) {
            constexpr int N = decltype(n_)::value;
            using PL = PlanFor<N>;
            const bool staged = stage_c2c(N) && aligned16(x);
            if (d == Direction::Forward) {
                const C2cIo io{x, y, N, keep, 1.0f};
                if constexpr (stage_c2c(N)) {
                    if (staged) {
                        launch_rows_staged<PL, false, B, Table>(io, batch, s, nullptr);
                        return;
                    }
                }
                launch_rows<PL, false, B, Table>(io, batch, s, nullptr);
            } else {
                using PI = PlanForInv<N>;
                const C2cIo io{x, y, keep, N, 1.0f / N};
                if constexpr (stage_c2c(N)) {
                    if (staged && keep == N) {
                        launch_rows_staged<PI, true, B, Table>(io, batch, s, nullptr);
                        return;
                    }
                }
                launch_rows<PI, true, B, Table>(io, batch, s, nullptr);
            }
        });
    }

    // `batch` real rows of n points (2 <= n <= 8192) to rows of `keep` (1 .. n/2 + 1) outputs.
    // Where the plan with the small radix last leaves two butterflies per thread in the last
    // pass, the combine runs in registers on mirror pairs (R2cPairIo).
    static void r2c(const float* x, float2* y, int n, long long batch, int keep, float2* /*work*/,
                    cudaStream_t s)
    {
        dispatch_pow2<1, kMaxRowN>(n / 2, [&](auto m_) {
            constexpr int M = decltype(m_)::value;
            const float2* w = Table ? twiddles::half_turn(M) : nullptr;
            const auto* xz = reinterpret_cast<const float2*>(x);
            using PP = PlanR2c<M>;
            if constexpr (M >= 32 && PP::kPairLast) {
                const R2cPairIo io{xz, y, keep};
                if constexpr (M >= kMinStagedN) {
                    if (aligned16(x)) {
                        launch_rows_staged<PP, false, B, Table>(io, batch, s, w);
                        return;
                    }
                }
                launch_rows<PP, false, B, Table>(io, batch, s, w);
            } else {
                using PL = PlanFor<M>;
                const R2cIo io{xz, y, keep};
                if constexpr (M >= kMinStagedN) {
                    if (aligned16(x)) {
                        launch_rows_staged<PL, false, B, Table>(io, batch, s, w);
                        return;
                    }
                }
                launch_rows<PL, false, B, Table>(io, batch, s, w);
            }
        });
    }

    // Rows of `keep` (1 .. n/2 + 1) complex inputs, the rest zero, to real rows of n points,
    // divided by n. Where the first pass has two butterflies per thread, the prepare step runs
    // in registers on mirror pairs (C2rPairIo).
    static void c2r(const float2* x, float* y, int n, long long batch, int keep, float2* /*work*/,
                    cudaStream_t s)
    {
        dispatch_pow2<1, kMaxRowN>(n / 2, [&](auto m_) {
            constexpr int M = decltype(m_)::value;
            using PL = PlanFor<M>;
            const float2* w = Table ? twiddles::half_turn(M) : nullptr;
            auto* yz = reinterpret_cast<float2*>(y);
            // The staged copy of a tile is rounded to 16 bytes; with batch * keep even and x
            // aligned the rounding never reaches past the end of x.
            const bool staged = M >= kMinStagedN && aligned16(x) && (batch * keep) % 2 == 0;
            if constexpr (M >= 32 && PL::kPairFirst) {
                const C2rPairIo io{x, yz, keep, 1.0f / M};
                if constexpr (M >= kMinStagedN) {
                    if (staged) {
                        launch_rows_staged<PL, true, B, Table>(io, batch, s, w);
                        return;
                    }
                }
                launch_rows<PL, true, B, Table>(io, batch, s, w);
            } else {
                const C2rIo io{x, yz, keep, 1.0f / M};
                if constexpr (M >= kMinStagedN) {
                    if (staged) {
                        launch_rows_staged<PL, true, B, Table>(io, batch, s, w);
                        return;
                    }
                }
                launch_rows<PL, true, B, Table>(io, batch, s, w);
            }
        });
    }
};

}  // namespace spectral::engine
