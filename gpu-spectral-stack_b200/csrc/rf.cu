// Radio-signal consumers of the row engine, fused into one kernel each: the windowed spectrum of
// back-to-back frames, and FIR filtering by overlap-save. The reference's python/spectral/rf.py
// (spectrum, rf.py:91-100; fir, rf.py:115-156) frames and multiplies in PyTorch around its FFT
// calls: a padded copy, a windowed copy, and for the filter the forward transform, a product with
// the filter's spectrum and the inverse transform as separate passes over global memory. Here:
//
//   spectrum  the frame load applies the zero padding of the last frame and the window: one pass,
//             signal in, spectrum out;
//   fir       per block of nfft samples (overlapping by len(taps) - 1): load with the zero history
//             and padding, forward transform, product with the taps' spectrum, inverse transform,
//             all in registers; the store keeps the nfft - len(taps) + 1 exact outputs. One pass,
//             signal in (plus the overlap), filtered signal out.
//
// Both are Io policies of the row kernel (engine.cuh), with the pass twiddles read from global
// memory, where the filter's inverse transform finds them too.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "rows.cuh"

#include <string>
#include <type_traits>

namespace spectral {
namespace {

using namespace engine;

// Frame f of row r covers x[r n + f N ..], zero beyond n; times window[k] (nullptr: all ones).
struct WindowIo {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = false;
    const float2* x;
    float2* y;
    const float* window;
    long long n;       // samples per row
    long long frames;  // frames per row

    template <class PL>
    __host__ __device__ static constexpr int extra() { return 0; }
    template <class PL, bool Table>
    __device__ static void prologue(float2*, const float2*) {}

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        const long long r = c.tf / frames;
        const long long start = (c.tf - r * frames) * PL::N;
        const float2* row = x + r * n;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = c.t + i * PL::P;
            const long long p = start + k;
            float2 s = (c.active && p < n) ? __ldg(row + p) : make_float2(0.0f, 0.0f);
            if (window != nullptr) {
                const float w = __ldg(window + k);
                s = make_float2(s.x * w, s.y * w);
            }
            v[i] = s;
        }
    }

    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        if (!c.active) {
            return;
        }
        float2* out = y + c.tf * PL::N + c.t;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            out[i * PL::P] = v[i];
        }
    }
};

// Block b of row r transforms signal samples b L - (m - 1) .. b L - (m - 1) + N - 1 of the row
// (zero before 0 and from n on), L = N - m + 1. Its outputs m - 1 .. N - 1 are y[r n + b L ..].
template <int B>
struct OverlapSaveIo {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = false;
    const float2* x;
    float2* y;
    const float2* h;   // spectrum of the zero-padded taps, N values
    const float2* tw;  // the plan's pass tables in global memory (for the inverse transform)
    long long n;       // samples per row
    long long blocks;  // blocks per row
    int m;             // taps

    template <class PL>
    __host__ __device__ static constexpr int extra() { return 0; }
    template <class PL, bool Table>
    __device__ static void prologue(float2*, const float2*) {}

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        const long long r = c.tf / blocks;
        const long long start = (c.tf - r * blocks) * (PL::N - m + 1) - (m - 1);
        const float2* row = x + r * n;
        if (c.active && start >= 0 && start + PL::N <= n) {
            // Interior block (every block but the first and the last of a row): no bounds.
            const float2* p = row + start + c.t;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = __ldg(p + i * PL::P);
            }
            return;
        }
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const long long p = start + c.t + i * PL::P;
            v[i] = (c.active && p >= 0 && p < n) ? __ldg(row + p) : make_float2(0.0f, 0.0f);
        }
    }

    // Called after the forward passes (natural order: v[i] = X[t + i P]): the product with the
    // taps' spectrum, the inverse passes in the same registers and exchange slot, and the store
    // of the exact outputs.
    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = cmul(v[i], __ldg(h + c.t + i * PL::P));
        }
        run_passes<PL, true, B>(v, c.t, c.buf, tw);
        if (!c.active) {
            return;
        }
        const long long r = c.tf / blocks;
        const long long b = c.tf - r * blocks;
        const int L = PL::N - m + 1;
        constexpr float kScale = 1.0f / PL::N;
        // Output k >= m - 1 of the block is sample b L + k - (m - 1) of the row.
        float2* out = y + r * n + b * L;
        if (b * L + L <= n) {  // every output of the block lies inside the row
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                const int k = c.t + i * PL::P;
                if (k >= m - 1) {
                    out[k - (m - 1)] = cscale(v[i], kScale);
                }
            }
            return;
        }
        const int last = static_cast<int>(n - b * L) + (m - 1);  // outputs k < last lie in the row
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = c.t + i * PL::P;
            if (k >= m - 1 && k < last) {
                out[k - (m - 1)] = cscale(v[i], kScale);
            }
        }
    }
};

void need(bool ok, const std::string& message)
{
    if (!ok) {
        throw InvalidArgument(message);
    }
}

// True when the byte ranges [a, a + an) and [b, b + bn) share a byte.
bool overlap(const void* a, unsigned long long an, const void* b, unsigned long long bn)
{
    const auto pa = reinterpret_cast<unsigned long long>(a);
    const auto pb = reinterpret_cast<unsigned long long>(b);
    return an > 0 && bn > 0 && pa < pb + bn && pb < pa + an;
}

void need_aligned(const void* p, const char* who)
{
    need((reinterpret_cast<unsigned long long>(p) & 7u) == 0, std::string(who) + ": arrays must be 8-byte aligned");
}

// Calls f(std::integral_constant<int, B>, std::bool_constant<Table>) for the engine variant
// behind an implementation name (the registry's stockham names); throws for the others, which
// have no fused kernel (the Python layer composes them from their transforms instead).
template <class F>
void with_variant(const char* impl, const char* who, F&& f)
{
    const std::string name = impl == nullptr ? "" : impl;
    if (name == "stockham_r2") {
        f(std::integral_constant<int, 2>{}, std::false_type{});
    } else if (name == "stockham_r4") {
        f(std::integral_constant<int, 4>{}, std::false_type{});
    } else if (name == "stockham_r8") {
        f(std::integral_constant<int, 8>{}, std::false_type{});
    } else if (name == "stockham_r8_table") {
        f(std::integral_constant<int, 8>{}, std::true_type{});
    } else {
        throw InvalidArgument(std::string(who) + ": no fused kernel for implementation '" + name
                              + "' (the stockham implementations have one)");
    }
}

template <int B, bool Table>
void spectrum(const float2* x, const float* window, float2* y, long long n, int nfft, long long rows,
              cudaStream_t s)
{
    const long long frames = n <= 0 ? 1 : (n + nfft - 1) / nfft;
    dispatch_pow2<2, kMaxRowN>(nfft, [&](auto n_) {
        constexpr int N = decltype(n_)::value;
        constexpr RowChoice rc = row_choice(RowKind::C2c, N);
        using PL = RowPlan<RowKind::C2c, N>;
        launch_rows<PL, false, B, Table, false, rc.persistent>(WindowIo{x, y, window, n, frames},
                                                               rows * frames, s, nullptr);
    });
}

template <int B, bool Table>
void fir(const float2* x, const float2* h, float2* y, long long n, int nfft, int m, long long rows,
         cudaStream_t s)
{
    const long long blocks = (n + (nfft - m)) / (nfft - m + 1);  // ceil(n / (nfft - m + 1)), n >= 1
    dispatch_pow2<2, kMaxRowN>(nfft, [&](auto n_) {
        constexpr int N = decltype(n_)::value;
        constexpr RowChoice rc = row_choice(RowKind::C2c, N);
        using PL = RowPlan<RowKind::C2c, N>;
        const float2* tw = row_pass_table<PL, Table, false>();
        launch_rows<PL, false, B, Table, false, rc.persistent>(
            OverlapSaveIo<B>{x, y, h, tw, n, blocks, m}, rows * blocks, s, nullptr);
    });
}

template <class F>
int rf_guarded(F&& f)
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

void check_common(const char* who, long long n, int nfft, long long rows)
{
    need(nfft >= 2 && nfft <= kMaxRowN && (nfft & (nfft - 1)) == 0,
         std::string(who) + ": nfft must be a power of two from 2 to " + std::to_string(kMaxRowN)
             + ", got " + std::to_string(nfft));
    need(n >= 0 && rows >= 0, std::string(who) + ": n and rows must not be negative");
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_spectrum(const char* impl, const void* x, const float* window, void* y, long long n,
                                 int nfft, long long rows, void* stream)
{
    using namespace spectral;
    return rf_guarded([&] {
        check_common("spectrum", n, nfft, rows);
        // Frames are read and written by different CTAs: the output may not share memory with
        // the signal.
        const unsigned long long frames = n <= 0 ? 1 : (n + nfft - 1) / nfft;
        need(!overlap(x, 8ULL * rows * n, y, 8ULL * rows * frames * nfft), "spectrum: x and y must not overlap");
        need_aligned(x, "spectrum");
        need_aligned(y, "spectrum");
        with_variant(impl, "spectrum", [&](auto b_, auto table_) {
            if (rows == 0) {
                return;
            }
            spectrum<decltype(b_)::value, decltype(table_)::value>(
                static_cast<const float2*>(x), window, static_cast<float2*>(y), n, nfft, rows,
                static_cast<cudaStream_t>(stream));
        });
    });
}

extern "C" int spectral_fir(const char* impl, const void* x, const void* taps_spectrum, void* y, long long n,
                            int nfft, int taps, long long rows, void* stream)
{
    using namespace spectral;
    return rf_guarded([&] {
        check_common("fir", n, nfft, rows);
        need(taps >= 1 && taps <= nfft, "fir: nfft must be a power of two of at least len(taps) = "
                                            + std::to_string(taps) + ", got " + std::to_string(nfft));
        // A block reads m - 1 samples that the previous block writes: no overlap at all.
        need(!overlap(x, 8ULL * rows * n, y, 8ULL * rows * n), "fir: x and y must not overlap");
        need_aligned(x, "fir");
        need_aligned(y, "fir");
        need_aligned(taps_spectrum, "fir");
        with_variant(impl, "fir", [&](auto b_, auto table_) {
            if (rows == 0 || n == 0) {
                return;
            }
            fir<decltype(b_)::value, decltype(table_)::value>(
                static_cast<const float2*>(x), static_cast<const float2*>(taps_spectrum),
                static_cast<float2*>(y), n, nfft, taps, rows, static_cast<cudaStream_t>(stream));
        });
    });
}
