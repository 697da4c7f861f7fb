// The large single-field 2D complex FFT, slab-decomposed by rows over R ranks (one per GPU).
// The reference has no counterpart: its fft2 stops at 4096 points per side
// (csrc/fft/fft2d.cu:65-75) and it has no multi-GPU code.
//
// An n x n field; rank r holds rows [r n/R, (r+1) n/R) ("rows" of them), w = n / R.
//
//   forward   1. spectral_slab_rows: n-point row transforms of the local rows, each stored into R
//               contiguous chunks, chunk s = columns [s w, (s+1) w) of every local row: the
//               send buffer of an all-to-all, [s][row][c].
//             2. all-to-all (the caller's NCCL; spectral.distributed uses torch.distributed):
//               rank s receives [r][row][c] from every r, which is exactly the n x w row-major
//               matrix of the field's columns [s w, (s+1) w).
//             3. spectral_slab_columns: n-point transforms down those w columns, natural order.
//   inverse   the same steps backwards: columns on the column slab (its row blocks are the send
//             chunks), the all-to-all, then row transforms whose input is gathered from the R
//             received chunks.
//
// Rows of up to 16384 points are transformed on chip in one pass; their larger twiddle tables
// are read from the correctly rounded table in global memory (L2-resident) instead of being
// copied to shared memory, which then holds only the transform. Columns longer than 4096 points
// use two column-tile passes (four-step, n = n1 n2): the first in place with the inter-pass
// twiddles, the second into the output in natural order. Every global access is a run of at
// least 16 consecutive complex values.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "columns.cuh"
#include "simple.cuh"

#include <climits>
#include <type_traits>

namespace spectral {
namespace {

using namespace engine;

constexpr int kMaxSlabN = 16384;

template <int N>
using SlabPlan = Plan<N, (N <= 4096 ? default_e(N) : N == 8192 ? 16 : 32), false,
                      (N <= 4096 ? default_threads(N) : kMinThreads)>;

// Rows of a slab: contiguous rows on the natural side, R chunks of w columns on the chunked side
// (element (row, k) at chunk k / w, offset row * w + k % w). Forward reads natural and writes
// chunked; inverse reads chunked and writes natural.
template <bool Inv>
struct SlabRowIo {
    static constexpr bool kPeer = false;
    const float2* x;
    float2* y;
    long long rows;  // rows per rank
    int wlog;        // log2 of the columns per chunk
    float scale;

    __device__ __forceinline__ long long chunked(long long row, int k) const
    {
        const int s = k >> wlog;
        return ((static_cast<long long>(s) * rows + row) << wlog) + (k & ((1 << wlog) - 1));
    }

    // Where chunks are whole multiples of the plan's P threads (w >= P), element t + i P of a
    // row lies in chunk (i P) >> wlog at offset t + ((i P) & (w - 1)): one base address per row,
    // a chunk stride and compile-time offsets instead of the index arithmetic per element.
    template <class PL>
    __device__ __forceinline__ long long chunked_fast(int i) const
    {
        const int off = i * PL::P;
        return static_cast<long long>(off >> wlog) * (rows << wlog) + (off & ((1 << wlog) - 1));
    }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], long long row, int t) const
    {
        if (Inv && (1 << wlog) >= PL::P) {
            const float2* b = x + (row << wlog) + t;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = b[chunked_fast<PL>(i)];
            }
            return;
        }
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = t + i * PL::P;
            v[i] = Inv ? x[chunked(row, k)] : x[row * PL::N + k];
        }
    }

    template <class PL>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], long long row, int t) const
    {
        if (!Inv && (1 << wlog) >= PL::P) {
            float2* b = y + (row << wlog) + t;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                b[chunked_fast<PL>(i)] = v[i];
            }
            return;
        }
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = t + i * PL::P;
            if constexpr (Inv) {
                y[row * PL::N + k] = cscale(v[i], scale);
            } else {
                y[chunked(row, k)] = v[i];
            }
        }
    }
};

// Rows of a slab exchanged through peer memory instead of an all-to-all: the chunked side lives
// on the ranks themselves. peer[s] is rank s's n x w column-slab buffer mapped into this GPU's
// address space (CUDA IPC over NVLink); this rank's rows are rows rank * rows .. of every one.
// Forward: the row transforms store chunk s of each row straight into peer[s] (plain stores over
// NVLink, coalesced in runs of at least 32 values). Inverse: the row transforms load chunk s of
// each row from peer[s]. The caller orders the ranks around the launch (a collective between the
// row and column kernels).
constexpr int kMaxPeerRanks = 8;

struct PeerSlabs {
    float2* p[kMaxPeerRanks];
};

template <bool Inv>
struct SlabPeerRowIo {
    static constexpr bool kPeer = true;
    const float2* x;  // forward: the rank's rows
    float2* y;        // inverse: the rank's rows
    PeerSlabs peer;
    long long rows;   // rows per rank
    int rank;
    int wlog;         // log2 of the columns per chunk
    float scale;

    __device__ __forceinline__ long long at(long long row, int k) const
    {
        return ((static_cast<long long>(rank) * rows + row) << wlog) + (k & ((1 << wlog) - 1));
    }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], long long row, int t) const
    {
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = t + i * PL::P;
            v[i] = Inv ? peer.p[k >> wlog][at(row, k)] : x[row * PL::N + k];
        }
    }

    template <class PL>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], long long row, int t) const
    {
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = t + i * PL::P;
            if constexpr (Inv) {
                y[row * PL::N + k] = cscale(v[i], scale);
            } else {
                peer.p[k >> wlog][at(row, k)] = v[i];
            }
        }
    }
};

template <class PL, bool Inv, class Io>
__global__ void __launch_bounds__(PL::THREADS)
    slab_row_kernel(const Io io, const float2* __restrict__ tw)
{
    wait_for_previous_grid();
    allow_next_grid();
    extern __shared__ float4 smem_raw[];
    float2* bufs = reinterpret_cast<float2*>(smem_raw);
    const int g = threadIdx.x / PL::P;
    const int t = threadIdx.x - g * PL::P;
    float2* buf = bufs + g * PL::BUF;
    for (long long r0 = static_cast<long long>(blockIdx.x) * PL::G; r0 < io.rows;
         r0 += static_cast<long long>(gridDim.x) * PL::G) {
        const long long row = r0 + g;
        const bool active = row < io.rows;
        float2 v[PL::E];
        if (active) {
            io.template load<PL>(v, row, t);
        } else {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = make_float2(0.0f, 0.0f);
            }
        }
        run_passes<PL, Inv, 8>(v, t, buf, tw);  // twiddles straight from the global table
        if (active) {
            io.template store<PL>(v, row, t);
        }
    }
    if constexpr (Io::kPeer && !Inv) {
        __threadfence_system();  // stores into peers' memory are complete before the kernel ends
    }
}

template <bool Inv, class MakeIo>
void slab_rows(int n, long long rows, cudaStream_t s, MakeIo&& make_io)
{
    dispatch_pow2<2, kMaxSlabN>(n, [&](auto n_) {
        constexpr int N = decltype(n_)::value;
        using PL = SlabPlan<N>;
        const auto io = make_io(static_cast<float>(Inv ? 1.0 / N : 1.0));
        auto kernel = slab_row_kernel<PL, Inv, std::decay_t<decltype(io)>>;
        constexpr std::size_t smem = sizeof(float2) * static_cast<std::size_t>(PL::G) * PL::BUF;
        static std::atomic<int> cache[kMaxDevices];
        const float2* tw = twiddles::pass_table(PL::N, PL::E);
        const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel), PL::THREADS,
                                              smem, cache, (rows + PL::G - 1) / PL::G);
        launch_pdl(kernel, grid, static_cast<unsigned>(PL::THREADS), smem, s, io, tw);
    });
}

// Pass 1 of an n = n1 n2 column transform over an n x w row-major matrix (four-step, Bailey):
// transform f = n2 w + c is column c at rows p n2 + n2 (an n1-point transform); its output k1 is
// multiplied by W_n^(k1 n2) and stored in place, at row k1 n2 + n2.
// (Loading the next tile ahead, as the strided columns do, made the one-rank 16384^2 step slower
// here: 3.00 -> 3.07 ms.)
struct SlabColumnPass1Io {
    float2* x;
    int w;
    int n2;
    int n;
    float scale;  // 1 / n1 for the inverse
    int wlog;     // log2 w

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
        const float2* b = x + c.f;  // column c of row n2 is element n2 w + c = f
        const long long stride = static_cast<long long>(n2) * w;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = b[(c.t + i * PL::P) * stride];
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
            return;
        }
        const int q = static_cast<int>(c.f >> wlog);
        float2* b = x + c.f;
        const long long stride = static_cast<long long>(n2) * w;
        const float step = 2.0f / static_cast<float>(n);  // exact: n is a power of two
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k1 = c.t + i * PL::P;
            float sn = 0.0f;
            float cs = 1.0f;
            sincospif(static_cast<float>(k1 * q) * step, &sn, &cs);  // k1 q < n <= 2^14: exact
            const float2 r = cmul_tw<Inv>(v[i], make_float2(cs, -sn));
            b[k1 * stride] = Inv ? cscale(r, scale) : r;
        }
    }
};

// Pass 2: transform f = k1 w + c is column c at rows k1 n2 + p (an n2-point transform); its output
// k2 is X[k1 + n1 k2], stored into y at that row.
struct SlabColumnPass2Io {
    const float2* x;
    float2* y;
    int w;
    int n1;
    int n2;
    float scale;  // 1 / n2 for the inverse

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
        const long long k1 = c.f / w;
        const long long col = c.f - k1 * w;
        const float2* b = x + (k1 * n2) * w + col;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = b[static_cast<long long>(c.t + i * PL::P) * w];
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
            return;
        }
        const long long k1 = c.f / w;
        const long long col = c.f - k1 * w;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const long long k2 = c.t + i * PL::P;
            y[(k1 + static_cast<long long>(n1) * k2) * w + col] = Inv ? cscale(v[i], scale) : v[i];
        }
    }
};

// The first stage of a 1D transform of n = n1 n2 points distributed over ranks (the four-step
// algorithm, Bailey 1990): an (n1, width) row-major slab holds columns j2 = col0 .. col0+width-1
// of the n1 x n2 view x[j1 n2 + j2]. Column c is an n1-point transform over j1; its output k1 is
// multiplied by W_n^(k1 j2) (its conjugate for the inverse) and stored back at row k1 of y.
struct SlabTwiddleColumnIo {
    const float2* x;
    float2* y;
    int width;
    long long col0;
    long long n;
    float scale;  // 1 / n1 for the inverse

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        const float2* b = x + (c.active ? c.f : 0);
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = c.active ? b[static_cast<long long>(c.t + i * PL::P) * width] : make_float2(0.0f, 0.0f);
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
            return;
        }
        const long long j2 = col0 + c.f;
        const float step = 2.0f / static_cast<float>(n);  // exact: n is a power of two
        float2* b = y + c.f;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const long long k1 = c.t + i * PL::P;
            float sn = 0.0f;
            float cs = 1.0f;
            sincospif(static_cast<float>(k1 * j2) * step, &sn, &cs);  // k1 j2 < n <= 2^24: exact
            const float2 r = cmul_tw<Inv>(v[i], make_float2(cs, -sn));
            b[k1 * width] = Inv ? cscale(r, scale) : r;
        }
    }
};

template <bool Inv>
void slab_columns(float2* x, float2* y, int n, int w, cudaStream_t s)
{
    if (n <= kMaxRowN) {
        kEngineR8.columns(x, y, n, w, 1, 0, 0, Inv ? Direction::Inverse : Direction::Forward, s);
        return;
    }
    const int n1 = 1 << (ilog2(n) / 2);
    const int n2 = n / n1;
    dispatch_pow2<2, kMaxRowN>(n1, [&](auto n1_) {
        constexpr int N1 = decltype(n1_)::value;
        launch_columns<PlanFor<N1>, Inv, 8, false>(
            SlabColumnPass1Io{x, w, n2, n, Inv ? 1.0f / N1 : 1.0f, ilog2(w)},
            static_cast<long long>(n2) * w, s);
    });
    dispatch_pow2<2, kMaxRowN>(n2, [&](auto n2_) {
        constexpr int N2 = decltype(n2_)::value;
        launch_columns<PlanFor<N2>, Inv, 8, false>(
            SlabColumnPass2Io{x, y, w, n1, n2, Inv ? 1.0f / N2 : 1.0f},
            static_cast<long long>(n1) * w, s);
    });
}

// Block relayout between the column-slab side and the natural (row) side of the exchange: for
// every rank r, the h x w block at src[r] (row stride src_stride) is copied to dst[r] (row stride
// dst_stride). With the blocks' pointers chosen by the caller this is each of the four steps a
// natural-layout transform needs (square blocks, h = w, for the 2D slab):
//   forward, received blocks -> rows:  src[r] = recv + r w^2 (w),  dst[r] = out + r w (n)
//   inverse, rows -> send blocks:      src[r] = x + r w (n),       dst[r] = send + r w^2 (w)
//   and the same with src[r] in another rank's memory (peer loads over NVLink, plain loads).
// One thread moves two complex values (16 bytes) where w is even, so every warp reads and
// writes runs of 512 bytes.
constexpr int kMaxRelayoutRanks = 16;

struct BlockTable {
    const float2* src[kMaxRelayoutRanks];
    float2* dst[kMaxRelayoutRanks];
};

template <bool Pairs>
__global__ void __launch_bounds__(256) slab_relayout_kernel(const BlockTable t, int w, long long src_stride,
                                                            long long dst_stride, long long per_rank)
// per_rank = h * (vectors per block row); the row count itself is implied.
{
    wait_for_previous_grid();
    allow_next_grid();
    constexpr int V = Pairs ? 2 : 1;
    const int cols = w / V;  // vectors per block row
    const int r = blockIdx.y;
    const float2* src = t.src[r];
    float2* dst = t.dst[r];
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < per_rank;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long k = e / cols;
        const int c = static_cast<int>(e - k * cols) * V;
        if constexpr (Pairs) {
            const float4 v = *reinterpret_cast<const float4*>(src + k * src_stride + c);
            *reinterpret_cast<float4*>(dst + k * dst_stride + c) = v;
        } else {
            dst[k * dst_stride + c] = src[k * src_stride + c];
        }
    }
}

// True when the byte ranges [a, a + an) and [b, b + bn) share a byte.
bool overlap(const void* a, unsigned long long an, const void* b, unsigned long long bn)
{
    const auto pa = reinterpret_cast<unsigned long long>(a);
    const auto pb = reinterpret_cast<unsigned long long>(b);
    return an > 0 && bn > 0 && pa < pb + bn && pb < pa + an;
}

void check_aligned(const void* p)
{
    if ((reinterpret_cast<unsigned long long>(p) & 7u) != 0) {
        throw InvalidArgument("fft2_slab: arrays must be 8-byte aligned");
    }
}

void check_slab(int n, int ranks)
{
    if (!is_pow2(n) || n < 2 || n > kMaxSlabN) {
        throw InvalidArgument("fft2_slab: n must be a power of two from 2 to "
                              + std::to_string(kMaxSlabN) + ", got " + std::to_string(n));
    }
    if (ranks < 1 || !is_pow2(ranks) || ranks > n) {
        throw InvalidArgument("fft2_slab: the ranks (" + std::to_string(ranks)
                              + ") must be a power of two dividing n = " + std::to_string(n));
    }
}

template <class F>
int slab_guarded(F&& f)
{
    try {
        f();
        return SPECTRAL_OK;
    } catch (const InvalidArgument& e) {
        set_last_error(e.what());
        return SPECTRAL_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_slab_rows(const void* x, void* y, int n, long long rows, int ranks,
                                  int inverse, void* stream)
{
    using namespace spectral;
    return slab_guarded([&] {
        check_slab(n, ranks);
        check_aligned(x);
        check_aligned(y);
        if (rows < 1 || rows > INT_MAX) {
            throw InvalidArgument("fft2_slab: rows must be from 1 to INT_MAX");
        }
        // A CTA stores its row's chunks where other rows' inputs lie (ranks > 1), so any overlap
        // of x and y races between CTAs: out of place only.
        const unsigned long long bytes = 8ULL * static_cast<unsigned long long>(rows) * static_cast<unsigned>(n);
        if (overlap(x, bytes, y, bytes)) {
            throw InvalidArgument("fft2_slab: the row stage is out of place (x and y must not overlap)");
        }
        const auto* xs = static_cast<const float2*>(x);
        auto* ys = static_cast<float2*>(y);
        const auto s = static_cast<cudaStream_t>(stream);
        const int wlog = ilog2(n / ranks);
        if (inverse) {
            slab_rows<true>(n, rows, s, [&](float sc) { return SlabRowIo<true>{xs, ys, rows, wlog, sc}; });
        } else {
            slab_rows<false>(n, rows, s, [&](float sc) { return SlabRowIo<false>{xs, ys, rows, wlog, sc}; });
        }
    });
}

extern "C" int spectral_slab_rows_peer(const void* x, void* y, void* const* peers, int n,
                                       long long rows, int rank, int ranks, int inverse,
                                       void* stream)
{
    using namespace spectral;
    return slab_guarded([&] {
        check_slab(n, ranks);
        if (ranks > kMaxPeerRanks) {
            throw InvalidArgument("fft2_slab: the peer exchange takes at most "
                                  + std::to_string(kMaxPeerRanks) + " ranks, got " + std::to_string(ranks));
        }
        if (rank < 0 || rank >= ranks) {
            throw InvalidArgument("fft2_slab: rank " + std::to_string(rank) + " outside 0 .. "
                                  + std::to_string(ranks - 1));
        }
        if (rows < 1 || rows * ranks != n) {
            throw InvalidArgument("fft2_slab: rows * ranks must equal n");
        }
        if (peers == nullptr) {
            throw InvalidArgument("fft2_slab: peers must list one buffer per rank");
        }
        check_aligned(x);
        check_aligned(y);
        PeerSlabs ps = {};
        for (int q = 0; q < ranks; ++q) {
            if (peers[q] == nullptr) {
                throw InvalidArgument("fft2_slab: peer buffer " + std::to_string(q) + " is null");
            }
            ps.p[q] = static_cast<float2*>(peers[q]);
        }
        const auto s = static_cast<cudaStream_t>(stream);
        const int wlog = ilog2(n / ranks);
        if (inverse) {
            auto* ys = static_cast<float2*>(y);
            slab_rows<true>(n, rows, s, [&](float sc) {
                return SlabPeerRowIo<true>{nullptr, ys, ps, rows, rank, wlog, sc};
            });
        } else {
            const auto* xs = static_cast<const float2*>(x);
            slab_rows<false>(n, rows, s, [&](float sc) {
                return SlabPeerRowIo<false>{xs, nullptr, ps, rows, rank, wlog, sc};
            });
        }
    });
}

extern "C" int spectral_slab_twiddle_columns(const void* x, void* y, int n1, int width, long long col0,
                                             long long n, int inverse, void* stream)
{
    using namespace spectral;
    return slab_guarded([&] {
        if (!is_pow2(n1) || n1 < 2 || n1 > kMaxRowN) {
            throw InvalidArgument("slab_twiddle_columns: n1 must be a power of two from 2 to "
                                  + std::to_string(kMaxRowN) + ", got " + std::to_string(n1));
        }
        if (!is_pow2(n) || n % n1 != 0 || n > (1LL << 24)) {
            throw InvalidArgument("slab_twiddle_columns: n must be a power of two multiple of n1, at most 2^24");
        }
        if (width < 1 || col0 < 0 || col0 + width > n / n1) {
            throw InvalidArgument("slab_twiddle_columns: the slab's columns must lie in 0 .. n/n1 - 1");
        }
        const unsigned long long bytes = 8ULL * n1 * width;
        if (overlap(x, bytes, y, bytes)) {
            throw InvalidArgument("slab_twiddle_columns: x and y must not overlap");
        }
        check_aligned(x);
        check_aligned(y);
        const auto s = static_cast<cudaStream_t>(stream);
        dispatch_pow2<2, kMaxRowN>(n1, [&](auto n1_) {
            constexpr int N1 = decltype(n1_)::value;
            const SlabTwiddleColumnIo io{static_cast<const float2*>(x), static_cast<float2*>(y), width, col0, n,
                                         1.0f / N1};
            if (inverse) {
                launch_columns<ColumnPlan<N1>, true, 8, false>(io, width, s);
            } else {
                launch_columns<ColumnPlan<N1>, false, 8, false>(io, width, s);
            }
        });
    });
}

extern "C" int spectral_transpose(const void* x, void* y, int rows, int cols, long long batch, void* stream)
{
    using namespace spectral;
    return slab_guarded([&] {
        if (rows < 1 || cols < 1 || batch < 0) {
            throw InvalidArgument("transpose: need rows, cols >= 1 and batch >= 0");
        }
        const unsigned long long bytes = 8ULL * rows * cols * static_cast<unsigned long long>(batch);
        if (x == y || overlap(x, bytes, y, bytes)) {
            throw InvalidArgument("transpose: x and y must not overlap");
        }
        check_aligned(x);
        check_aligned(y);
        if (batch > 0) {
            simple::transpose(static_cast<const float2*>(x), static_cast<float2*>(y), rows, cols, batch,
                              static_cast<cudaStream_t>(stream));
        }
    });
}

extern "C" int spectral_slab_relayout(const void* const* src, void* const* dst, int ranks, int h, int w,
                                      long long src_stride, long long dst_stride, void* stream)
{
    using namespace spectral;
    return slab_guarded([&] {
        if (ranks < 1 || ranks > kMaxRelayoutRanks) {
            throw InvalidArgument("slab_relayout: ranks must be from 1 to " + std::to_string(kMaxRelayoutRanks));
        }
        if (h < 1 || w < 1 || src_stride < w || dst_stride < w) {
            throw InvalidArgument("slab_relayout: need h, w >= 1 and row strides of at least w");
        }
        if (src == nullptr || dst == nullptr) {
            throw InvalidArgument("slab_relayout: src and dst must list one block per rank");
        }
        BlockTable t = {};
        bool pairs = w % 2 == 0 && src_stride % 2 == 0 && dst_stride % 2 == 0;
        for (int r = 0; r < ranks; ++r) {
            if (src[r] == nullptr || dst[r] == nullptr) {
                throw InvalidArgument("slab_relayout: block " + std::to_string(r) + " is null");
            }
            check_aligned(src[r]);
            check_aligned(dst[r]);
            pairs = pairs && (reinterpret_cast<unsigned long long>(src[r]) & 15u) == 0
                    && (reinterpret_cast<unsigned long long>(dst[r]) & 15u) == 0;
            t.src[r] = static_cast<const float2*>(src[r]);
            t.dst[r] = static_cast<float2*>(dst[r]);
        }
        // Threads of different CTAs copy different blocks: a source block that shares memory
        // with any destination block races, so every pair is refused (at most 16 x 16).
        const unsigned long long src_bytes = 8ULL * (static_cast<unsigned long long>(h - 1) * src_stride + w);
        const unsigned long long dst_bytes = 8ULL * (static_cast<unsigned long long>(h - 1) * dst_stride + w);
        for (int r = 0; r < ranks; ++r) {
            for (int q = 0; q < ranks; ++q) {
                if (overlap(src[r], src_bytes, dst[q], dst_bytes)) {
                    throw InvalidArgument("slab_relayout: source block " + std::to_string(r)
                                          + " overlaps destination block " + std::to_string(q));
                }
            }
        }
        const long long per_rank = static_cast<long long>(h) * (pairs ? w / 2 : w);
        const long long blocks_x = (per_rank + 255) / 256;
        const dim3 grid(static_cast<unsigned>(blocks_x < 4096 ? blocks_x : 4096), static_cast<unsigned>(ranks));
        const auto s = static_cast<cudaStream_t>(stream);
        if (pairs) {
            launch_pdl(slab_relayout_kernel<true>, grid, dim3(256), 0, s, t, w, src_stride, dst_stride, per_rank);
        } else {
            launch_pdl(slab_relayout_kernel<false>, grid, dim3(256), 0, s, t, w, src_stride, dst_stride, per_rank);
        }
    });
}

extern "C" int spectral_slab_columns(void* x, void* y, int n, int width, int inverse, void* stream)
{
    using namespace spectral;
    return slab_guarded([&] {
        check_slab(n, 1);
        check_aligned(x);
        check_aligned(y);
        if (width < 1) {
            throw InvalidArgument("fft2_slab: width must be at least 1");
        }
        // For n > 4096 the first pass writes x and the second reads x and writes y: any overlap
        // of the two, not only x == y, would corrupt the result.
        const unsigned long long bytes = 8ULL * static_cast<unsigned>(n) * static_cast<unsigned>(width);
        if (overlap(x, bytes, y, bytes)) {
            throw InvalidArgument("fft2_slab: columns are transformed out of place (x and y must not overlap)");
        }
        auto* xs = static_cast<float2*>(x);
        auto* ys = static_cast<float2*>(y);
        const auto s = static_cast<cudaStream_t>(stream);
        if (inverse) {
            slab_columns<true>(xs, ys, n, width, s);
        } else {
            slab_columns<false>(xs, ys, n, width, s);
        }
    });
}
