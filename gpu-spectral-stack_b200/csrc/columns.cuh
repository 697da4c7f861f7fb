#pragma once

// Column transforms: the transform runs down a column of a row-major array, so its elements are
// a row length apart. The reference's StridedIo (stockham.cuh:359-410) gives each block T
// neighbouring columns with T = 256 / (threads per column), which is 1-8 columns at the sizes
// that matter, so each warp reads runs of 8-64 bytes (20 sectors per request at 1024 points,
// docs/PROFILING.md:164-179).
//
// Here a CTA takes C = 16 neighbouring columns (fewer only where 16 would not fit in 1024
// threads) and maps thread (t, c) to threadIdx = t C + c: for every row it touches, a warp reads
// or writes C consecutive columns, runs of 128 bytes, straight from global memory into
// registers. The engine's exchanges use the column-interleaved layout (position p of column c at
// p C + c), in which those same C threads touch C consecutive words: no bank conflicts at any
// pass. Columns are numbered across arrays (column f is column f mod cols of array f / cols), so
// a tile may straddle two arrays and no CTA idles on a ragged last tile of each array.

#include "rows.cuh"

namespace spectral::engine {

template <class PL>
__host__ __device__ constexpr int columns_per_cta()
{
    return cmin(16, cmax(1, 1024 / PL::P));
}

// Where a column thread is: column f = f0 + c of `transforms`, thread t of its P; `tile` is the
// CTA's exchange tile (C (N + 1) entries), free for staging after the last pass.
struct ColumnCtx {
    long long f;
    long long f0;
    long long transforms;
    int c;
    int t;
    bool active;
    float2* tile;
};

// Prefetch: the next tile's loads are issued before this tile's passes (the Io's load must not
// read what another tile stores: true of column tiles, which are disjoint sets of columns).
template <class PL, int C, bool Inv, int B, bool Table, class Io, bool TwGlobal = false, bool Prefetch = false>
__global__ void __launch_bounds__(C * PL::P, PL::MIN_BLOCKS)
    column_kernel(const Io io, long long transforms, const float2* __restrict__ tw_table)
{
    wait_for_previous_grid();
    allow_next_grid();
    extern __shared__ float4 smem_raw[];
    // TwGlobal: the pass tables are read where they lie in global memory (L1-resident).
    float2* tw_s = reinterpret_cast<float2*>(smem_raw);
    float2* tile = tw_s + (TwGlobal ? 0 : ((PL::TW + 1) & ~1));
    const float2* tw = TwGlobal ? tw_table : tw_s;

    if constexpr (!TwGlobal) {
        fill_pass_twiddles<PL, Table>(tw_s, tw_table);
    }
    __syncthreads();

    const int c = threadIdx.x % C;
    const int t = threadIdx.x / C;
    auto context = [&](long long f0) {
        ColumnCtx ctx;
        ctx.f0 = f0;
        ctx.f = f0 + c;
        ctx.active = ctx.f < transforms;
        ctx.transforms = transforms;
        ctx.c = c;
        ctx.t = t;
        ctx.tile = tile;
        return ctx;
    };
    const long long stride = static_cast<long long>(gridDim.x) * C;
    if constexpr (Prefetch) {
        float2 next[PL::E];
        io.template load<PL>(next, context(static_cast<long long>(blockIdx.x) * C));
        for (long long f0 = static_cast<long long>(blockIdx.x) * C; f0 < transforms; f0 += stride) {
            const ColumnCtx ctx = context(f0);
            float2 v[PL::E];
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = next[i];
            }
            io.template load<PL>(next, context(f0 + stride));  // inactive past the end: zeros
            run_passes<PL, Inv, B, C, true>(v, t, tile + c, tw);
            io.template store<PL, C, Inv>(v, ctx);
        }
    } else {
        for (long long f0 = static_cast<long long>(blockIdx.x) * C; f0 < transforms; f0 += stride) {
            const ColumnCtx ctx = context(f0);
            float2 v[PL::E];
            io.template load<PL>(v, ctx);
            run_passes<PL, Inv, B, C, true>(v, t, tile + c, tw);
            io.template store<PL, C, Inv>(v, ctx);
        }
    }
}

template <class PL, int C, bool TwGlobal = false>
constexpr std::size_t column_smem_bytes()
{
    return sizeof(float2)
           * ((TwGlobal ? 0 : static_cast<std::size_t>((PL::TW + 1) & ~1))
              + static_cast<std::size_t>(C) * (PL::N + 1));
}

// Io policies whose load may run one tile ahead (kPrefetch = true): their loads never read what
// another tile's store writes. The prefetch pays for 64- to 512-point columns (measured on B200,
// 2^24 points per call: 256 points 29.2 -> 27.2 µs, 512 points 37.1 -> 29.8 µs, 128 points
// 26.9 -> 25.6 µs, 64 points 29.7 -> 27.1 µs); elsewhere it is untested and off.
template <class Io, class = void>
struct column_prefetch : std::false_type {};
template <class Io>
struct column_prefetch<Io, std::void_t<decltype(Io::kPrefetch)>> : std::bool_constant<Io::kPrefetch> {};

template <class PL, bool Inv, int B, bool Table, class Io>
void launch_columns(const Io& io, long long transforms, cudaStream_t stream)
{
    if (transforms <= 0) {
        return;
    }
    constexpr int C = columns_per_cta<PL>();
    constexpr bool Prefetch = column_prefetch<Io>::value && PL::N >= 64 && PL::N <= 512;
    auto kernel = column_kernel<PL, C, Inv, B, Table, Io, false, Prefetch>;
    constexpr std::size_t smem = column_smem_bytes<PL, C>();
    static std::atomic<int> cache[kMaxDevices];
    const float2* tw = Table ? twiddles::pass_table(PL::N, PL::E) : nullptr;
    const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel), C * PL::P, smem,
                                          cache, (transforms + C - 1) / C);
    launch_pdl(kernel, grid, static_cast<unsigned>(C * PL::P), smem, stream, io, transforms, tw);
}

// Where frequency `pos` of an N-point column is stored when only the 2 m1 lowest frequencies
// are (0 .. m1-1 in rows 0 .. m1-1, then N-m1 .. N-1 in rows m1 .. 2 m1-1), or -1 when it is not;
// m1 = 0 stores every row. The layout of the reference's pruned columns (stockham.cuh:387-407)
// and of spectral.reference.rfft2_truncate.
__device__ __forceinline__ int mode_row(int pos, int n, int m1)
{
    if (m1 == 0) {
        return pos;
    }
    return pos < m1 ? pos : (pos >= n - m1 ? pos - (n - 2 * m1) : -1);
}

// Columns of `slabs` row-major arrays of N rows by `cols` columns, pruned as Backend::columns
// describes. In place or out of place: a tile's columns are its own, so its loads may run one
// tile ahead.
struct StridedIo {
    static constexpr bool kPrefetch = true;
    const float2* x;
    float2* y;
    int cols;
    int m1_in;
    int m1_out;
    float scale;

    // Array and column of column f: one division per tile, in 32 bits where f allows.
    __device__ __forceinline__ void locate(long long f, long long& slab, int& col) const
    {
        if (f < (1LL << 31)) {
            const unsigned q = static_cast<unsigned>(f) / static_cast<unsigned>(cols);
            slab = q;
            col = static_cast<int>(static_cast<unsigned>(f) - q * static_cast<unsigned>(cols));
        } else {
            slab = f / cols;
            col = static_cast<int>(f - slab * cols);
        }
    }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        const float2 zero = make_float2(0.0f, 0.0f);
        if (!c.active) {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = zero;
            }
            return;
        }
        long long slab = 0;
        int col = 0;
        locate(c.f, slab, col);
        const int rows = m1_in > 0 ? 2 * m1_in : PL::N;
        const float2* base = x + slab * rows * cols + col;
        // Plain loads: the column transforms may run in place (x == y).
        if (m1_in == 0) {
            const float2* p = base + static_cast<long long>(c.t) * cols;
            const long long step = static_cast<long long>(PL::P) * cols;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = *p;
                p += step;
            }
        } else {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                const int row = mode_row(c.t + i * PL::P, PL::N, m1_in);
                v[i] = row >= 0 ? base[static_cast<long long>(row) * cols] : zero;
            }
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
            return;
        }
        long long slab = 0;
        int col = 0;
        locate(c.f, slab, col);
        const int rows = m1_out > 0 ? 2 * m1_out : PL::N;
        float2* base = y + slab * rows * cols + col;
        if (m1_out == 0) {
            float2* p = base + static_cast<long long>(c.t) * cols;
            const long long step = static_cast<long long>(PL::P) * cols;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                *p = Inv ? cscale(v[i], scale) : v[i];
                p += step;
            }
        } else {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                const int row = mode_row(c.t + i * PL::P, PL::N, m1_out);
                if (row >= 0) {
                    base[static_cast<long long>(row) * cols] = Inv ? cscale(v[i], scale) : v[i];
                }
            }
        }
    }
};

// Pass 1 of a complex transform of n = N1 N2 points (the four-step algorithm, Bailey 1990; the
// reference's fourstep.cuh:3-26). Transform b is viewed as N1 rows by N2 columns; column n2
// (f = b N2 + n2) is an N1-point transform whose output k1 is multiplied by W_n^(k1 n2) and
// stored at y[b n + n2 N1 + k1]: transposed, so that pass 2 is a plain column transform of the
// N2 x N1 view, in place, whose output k2 of column k1 lands at k1 + N1 k2, the natural order.
// Two passes over global memory and no workspace, where the reference makes three (columns, a
// twiddled row pass into a workspace, and a transpose) and allocates the workspace per call.
// The transposed store goes through the tile as [column][k1] with a stride of N1 + 1, so the
// staging writes and the global writes (runs of N1 values) are both conflict-free and coalesced.
struct FourStepIo {
    const float2* x;
    float2* y;
    int n2log;    // log2 of the columns of the first view (= the second pass's length)
    long long n;  // points per transform
    float scale;  // 1 / N1 for the inverse

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = make_float2(0.0f, 0.0f);
            }
            return;
        }
        const long long b = c.f >> n2log;
        const int col = static_cast<int>(c.f & ((1LL << n2log) - 1));
        const float2* p = x + b * n + col + (static_cast<long long>(c.t) << n2log);
        const long long step = static_cast<long long>(PL::P) << n2log;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = *p;
            p += step;
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        constexpr int N1 = PL::N;
        const int col = static_cast<int>(c.f & ((1LL << n2log) - 1));
        const float step = 2.0f / static_cast<float>(n);  // a power of two: exact
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k1 = c.t + i * PL::P;
            // k1 col < n <= 2^24 is exact in float, so 2 k1 col / n is too. (Two table loads and
            // a complex multiply measured slower here than the arithmetic.)
            float sn = 0.0f;
            float cs = 1.0f;
            sincospif(static_cast<float>(k1 * col) * step, &sn, &cs);
            const float2 r = cmul_tw<Inv>(v[i], make_float2(cs, -sn));
            c.tile[c.c * (N1 + 1) + k1] = Inv ? cscale(r, scale) : r;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < C * N1; e += C * PL::P) {
            const int cc = e / N1;
            const int k1 = e - cc * N1;
            const long long f = c.f0 + cc;
            if (f < c.transforms) {
                const long long bb = f >> n2log;
                const long long cl = f & ((1LL << n2log) - 1);
                y[bb * n + cl * N1 + k1] = c.tile[cc * (N1 + 1) + k1];
            }
        }
        __syncthreads();
    }
};

// Strided column plans with the CTAs per SM that the register budget must allow, from sweeps
// on B200. Without the prefetch, 256-point columns of 256 fields x 129 took 32.3 us at the
// compiler's own budget (two CTAs per SM) and 29.7 us at three; with it (32 more registers),
// 27.2 us at two, while three spill. 512-point columns: 38.8 us at two CTAs per SM without the
// prefetch, 29.8 us at one with it.
__host__ __device__ constexpr int column_min_blocks(int n) { return n == 256 ? 2 : 1; }

template <int N>
using ColumnPlan = Plan<N, default_e(N), false, default_threads(N), column_min_blocks(N)>;

template <int B, bool Table>
struct ColumnEngine {
    static void columns(const float2* x, float2* y, int n, int cols, long long slabs, int m1_in,
                        int m1_out, Direction d, cudaStream_t s)
    {
        dispatch_pow2<2, kMaxRowN>(n, [&](auto n_) {
            constexpr int N = decltype(n_)::value;
            using PL = ColumnPlan<N>;
            const long long transforms = slabs * cols;
            if (d == Direction::Forward) {
                launch_columns<PL, false, B, Table>(StridedIo{x, y, cols, m1_in, m1_out, 1.0f},
                                                    transforms, s);
            } else {
                launch_columns<PL, true, B, Table>(
                    StridedIo{x, y, cols, m1_in, m1_out, 1.0f / N}, transforms, s);
            }
        });
    }

    // Complex transforms of 4096 < n <= 2^24 points: pass 1 (FourStepIo) from x into y, then
    // pass 2, plain columns in place on y. n1 = 2^floor(log2 n / 2) <= n2 = n / n1 <= 4096.
    static void fourstep(const float2* x, float2* y, int n, long long batch, Direction d,
                         cudaStream_t s)
    {
        const int n1 = 1 << (ilog2(n) / 2);
        const int n2 = n / n1;
        dispatch_pow2<2, kMaxRowN>(n1, [&](auto n1_) {
            constexpr int N1 = decltype(n1_)::value;
            using PL = PlanFor<N1>;
            const int n2log = ilog2(n2);
            if (d == Direction::Forward) {
                launch_columns<PL, false, B, Table>(FourStepIo{x, y, n2log, n, 1.0f}, batch * n2, s);
            } else {
                launch_columns<PL, true, B, Table>(FourStepIo{x, y, n2log, n, 1.0f / N1}, batch * n2, s);
            }
        });
        columns(y, y, n2, n1, batch, 0, 0, d, s);
    }
};

}  // namespace spectral::engine
