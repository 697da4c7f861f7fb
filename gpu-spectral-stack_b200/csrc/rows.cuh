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

// Threads per CTA for the column and fused 2D kernels' plans (PlanFor); row kernels use
// row_choice below.
__host__ __device__ constexpr int default_threads(int n)
{
    return (n == 1024 || n == 2048) ? 128 : kMinThreads;
}

template <int N>
using PlanFor = Plan<N, default_e(N), false, default_threads(N)>;

// --- row kernel choices ------------------------------------------------------------------------
//
// Per transform kind and size (n complex points per transform; M = n / 2 for the real kinds):
// threads per CTA, the CTAs per SM the register budget must allow, whether the twiddle tables
// are copied into shared memory per CTA or read from global memory (one L1-resident copy per SM),
// whether the input is prefetched with bulk copies (the staged kernel), and whether the grid is
// persistent (every resident slot once, walking the batch) or one CTA per tile of transforms
// (no per-CTA set-up left once the tables are in global memory, and the hardware scheduler
// balances the last wave: 1024-point complex transforms 47.3 -> 44.5 us), and whether the next
// tile's input is loaded while this one computes (4096-point real forward 30.9 -> 28.8 us,
// 256-point real 29.6 -> 29.0 us inverse; elsewhere it measured slower; the 256-point real
// forward, once its twiddles were derived, runs best as one CTA per tile with a budget of 5 CTAs
// per SM: 30.7 us persistent with the prefetch, 27.3 us). Each entry is the
// best of a sweep on B200 at 2^24 points per call. The pattern: reading the twiddles from global
// memory halves the shared memory of the real-transform kernels and lets the compiler hoist the
// twiddle loads past the exchanges' barriers (1024 real points: 38.9 -> 30.0 us; 4096: 39.1 ->
// 31.2 us; its inverse 41.6 -> 29.0 us), while the complex transforms up to 1024 points, whose
// tables are small, gain little or nothing from it. The bulk-copy prefetch pays only for complex
// transforms of 2048 and 4096 points, which span eight warps.

enum class RowKind { C2c, R2c, C2r };

struct RowChoice {
    int threads;
    int min_blocks;
    bool smem_twiddles;
    bool staged;
    bool persistent;
    bool prefetch;  // load the next tile while computing this one (plain-load inputs only)
};

__host__ __device__ constexpr RowChoice row_choice(RowKind k, int n)
{
    if (k == RowKind::C2c) {
        return n <= 64   ? RowChoice{kMinThreads, 1, true, false, true}
             : n == 128  ? RowChoice{128, 4, false, false, true}
             : n <= 1024 ? RowChoice{128, 4, false, false, false}
             : n == 2048 ? RowChoice{kMinThreads, 1, false, true, true}
                         : RowChoice{kMinThreads, 2, true, true, true};
    }
    const bool r2c = k == RowKind::R2c;
    return n <= 8      ? RowChoice{kMinThreads, 1, !r2c, false, !r2c}
         : n == 16     ? RowChoice{kMinThreads, 1, !r2c, false, false}
         : n == 32     ? RowChoice{kMinThreads, 1, true, false, true}
         : n == 64     ? RowChoice{kMinThreads, 1, false, false, true}
         : n == 128    ? (r2c ? RowChoice{128, 5, false, false, false, false} : RowChoice{128, 4, false, false, true, true})
         : n == 512    ? RowChoice{128, r2c ? 3 : 4, r2c, false, true}
         : n <= 1024   ? RowChoice{128, 4, false, false, true}
         : n == 2048   ? RowChoice{128, r2c ? 5 : 6, false, false, r2c, r2c}
                       : RowChoice{kMinThreads, 2, false, false, true};
}

// Grid of a row launch: persistent (resident slots) or one CTA per tile. Either way the kernel
// walks the batch with a grid stride, and the shared-memory opt-in is made once.
inline unsigned row_grid(const void* kernel, int threads, std::size_t smem, std::atomic<int>* cache,
                         long long tiles, bool persistent)
{
    if (persistent) {
        return persistent_grid(kernel, threads, smem, cache, tiles);
    }
    resident_ctas(kernel, threads, smem, cache, current_device());
    constexpr long long kMaxGrid = 1LL << 30;
    return static_cast<unsigned>(tiles < 1 ? 1 : tiles < kMaxGrid ? tiles : kMaxGrid);
}

template <RowKind K, int N, bool SmallLast = false>
using RowPlan = Plan<N, default_e(N), SmallLast, row_choice(K, N).threads, row_choice(K, N).min_blocks>;

// The twiddle tables a row kernel reads: the correctly rounded host tables (Table), else the
// on-chip computed ones, in global memory when the kernel does not fill its own shared copy.
template <class PL, bool Table, bool SmemTw>
const float2* row_pass_table()
{
    if constexpr (Table) {
        return twiddles::pass_table(PL::N, PL::E, PL::SmallLast);
    } else if constexpr (SmemTw) {
        return nullptr;
    } else {
        return twiddles::pass_table_computed(PL::N, PL::E, PL::SmallLast);
    }
}

template <int M, bool Table, bool SmemTw>
const float2* row_half_turn()
{
    if constexpr (Table) {
        return twiddles::half_turn(M);
    } else if constexpr (SmemTw) {
        return nullptr;
    } else {
        return twiddles::half_turn_computed(M);
    }
}

template <class PL, bool Inv, int B, bool Table, bool SmemTw, bool Persistent = true,
          bool Prefetch = false, class Io>
void launch_rows(const Io& io, long long batch, cudaStream_t stream, const float2* extra_table)
{
    if (batch <= 0) {
        return;
    }
    auto kernel = row_kernel<PL, Inv, B, Table, Io, !SmemTw, Prefetch>;
    constexpr std::size_t smem = row_smem_bytes<PL, Io, !SmemTw>();
    static std::atomic<int> cache[kMaxDevices];
    const float2* tw = row_pass_table<PL, Table, SmemTw>();
    const unsigned grid = row_grid(reinterpret_cast<const void*>(kernel), PL::THREADS, smem, cache,
                                   (batch + PL::G - 1) / PL::G, Persistent);
    launch_pdl(kernel, grid, static_cast<unsigned>(PL::THREADS), smem, stream, io, batch, tw, extra_table);
}

// The staged kernel (bulk-copy prefetch, engine.cuh), when the input satisfies cp.async.bulk's
// rules: a 16-byte aligned source and whole 16-byte tiles.
inline bool aligned16(const void* p) { return (reinterpret_cast<unsigned long long>(p) & 15u) == 0; }

template <class PL, bool Inv, int B, bool Table, bool SmemTw, class Io>
void launch_rows_staged(const Io& io, long long batch, cudaStream_t stream, const float2* extra_table)
{
    if (batch <= 0) {
        return;
    }
    auto kernel = staged_row_kernel<PL, Inv, B, Table, Io, !SmemTw>;
    constexpr std::size_t smem = staged_smem_bytes<PL, Io, !SmemTw>();
    static_assert(smem <= 227 * 1024, "staged tile does not fit in shared memory");
    static std::atomic<int> cache[kMaxDevices];
    const float2* tw = row_pass_table<PL, Table, SmemTw>();
    const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel), PL::THREADS, smem,
                                          cache, (batch + PL::G - 1) / PL::G);
    launch_pdl(kernel, grid, static_cast<unsigned>(PL::THREADS), smem, stream, io, batch, tw, extra_table, device_fault_word());
}

// How much of their twiddles the computed-twiddle variants' real-row kernels derive instead of
// loading (engine.cuh: run_passes' Derive).
constexpr int kDeriveLevel = 1;

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
            constexpr RowChoice rc = row_choice(RowKind::C2c, N);
            using PL = RowPlan<RowKind::C2c, N>;
            const bool inv = d == Direction::Inverse;
            const C2cIo io = inv ? C2cIo{x, y, keep, N, 1.0f / N} : C2cIo{x, y, N, keep, 1.0f};
            // Staged tiles are whole unpruned input rows.
            const bool staged = rc.staged && aligned16(x) && (!inv || keep == N);
            if constexpr (rc.staged && N >= 64) {
                if (staged) {
                    if (inv) {
                        launch_rows_staged<PL, true, B, Table, rc.smem_twiddles>(io, batch, s, nullptr);
                    } else {
                        launch_rows_staged<PL, false, B, Table, rc.smem_twiddles>(io, batch, s, nullptr);
                    }
                    return;
                }
            }
            if (inv) {
                launch_rows<PL, true, B, Table, rc.smem_twiddles, rc.persistent>(io, batch, s, nullptr);
            } else {
                launch_rows<PL, false, B, Table, rc.smem_twiddles, rc.persistent>(io, batch, s, nullptr);
            }
        });
    }

    // `batch` real rows of n points (2 <= n <= 8192) to rows of `keep` (1 .. n/2 + 1) outputs.
    // Where the plan with the small radix last leaves two butterflies per thread in the last
    // pass, the combine runs in registers on mirror pairs (R2cPairIoT); the computed-twiddle
    // variants derive the mirror and combine twiddles from constants, the table variant reads them.
    static void r2c(const float* x, float2* y, int n, long long batch, int keep, float2* /*work*/,
                    cudaStream_t s)
    {
        dispatch_pow2<1, kMaxRowN>(n / 2, [&](auto m_) {
            constexpr int M = decltype(m_)::value;
            constexpr RowChoice rc = row_choice(RowKind::R2c, M);
            const float2* w = row_half_turn<M, Table, rc.smem_twiddles>();
            const auto* xz = reinterpret_cast<const float2*>(x);
            using PP = RowPlan<RowKind::R2c, M, true>;
            if constexpr (M >= 32 && PP::kPairLast) {
                launch_rows<PP, false, B, Table, rc.smem_twiddles, rc.persistent, rc.prefetch>(R2cPairIoT<Table ? 0 : kDeriveLevel>{xz, y, keep}, batch, s, w);
            } else {
                using PL = RowPlan<RowKind::R2c, M>;
                launch_rows<PL, false, B, Table, rc.smem_twiddles, rc.persistent, rc.prefetch>(R2cIo{xz, y, keep}, batch, s, w);
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
            constexpr RowChoice rc = row_choice(RowKind::C2r, M);
            using PL = RowPlan<RowKind::C2r, M>;
            const float2* w = row_half_turn<M, Table, rc.smem_twiddles>();
            auto* yz = reinterpret_cast<float2*>(y);
            if constexpr (M >= 32 && PL::kPairFirst) {
                launch_rows<PL, true, B, Table, rc.smem_twiddles, rc.persistent, rc.prefetch>(C2rPairIoT<Table ? 0 : kDeriveLevel>{x, yz, keep, 1.0f / M}, batch, s, w);
            } else {
                launch_rows<PL, true, B, Table, rc.smem_twiddles, rc.persistent>(C2rIo{x, yz, keep, 1.0f / M}, batch, s, w);
            }
        });
    }
};

}  // namespace spectral::engine
