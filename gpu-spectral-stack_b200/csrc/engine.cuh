#pragma once

// The register-resident FFT engine shared by every transform in this library.
//
// A transform of N points is held by P = N / E threads, E points each, always in registers. It
// runs in PASSES = ceil(log2 N / log2 E) passes; pass s is a radix-R_s Stockham step done as an
// in-register R_s-point DFT (dft.cuh), so the only shared-memory traffic is one exchange
// between consecutive passes: N = 1024 with E = 32 is two passes and one exchange, against the
// reference's four shared-memory stages with two barriers each (stockham.cuh:177-209, 442-449).
// With P <= 32 a transform lives inside one warp and its exchanges need only __syncwarp.
//
// Layout invariant: before pass 0 and after the last pass, thread t of a transform holds the
// element at position t + i P in v[i], i = 0 .. E-1. Consecutive threads therefore touch
// consecutive elements for every i: the global loads and stores of contiguous rows are
// coalesced with no staging, and the output comes out in natural order.
//
// Pass s has radix R = radix(s) and sub-transform length L = span(s) (the product of the
// earlier radices). Butterfly j = t + b P (b < E / R) reads positions j + r N / R, which are
// v[b + r E / R]; multiplies input r by W_{L R}^(k r), k = j mod L; runs the R-point DFT; and
// writes output r to position (j - k) R + k + r L. The small radix (if log2 E does not divide
// log2 N) goes first, where no twiddles are needed.
//
// Exchange layout: position p is stored at pad(p) = p + L * floor(p / W) when L < 16, else at
// p; W = L R, or 16 where L R < 16 and a transform has at least 16 threads. For the strided
// writes of the early passes this puts the 16 threads of a half-warp on 16 different 8-byte bank
// pairs; the reads of the next pass (consecutive positions) stay conflict-free because, with
// W >= 16, a half-warp's 16 consecutive positions are never split by a pad entry (with W = 8, as
// for a radix-8 first pass, they would straddle one and wrap onto a bank already in use). Where
// a transform has fewer than 16 threads, W = L R keeps each transform's writes spread so that
// the transforms sharing a half-warp (slots P apart in banks) do not collide. One exchange is
// permuted instead of padded: the one after a mirror first pass of radix below 16 (see pass).
// The reference's stage store has 4.5 M bank conflicts per 2^24 points
// (docs/PROFILING.md:129-136).
//
// Twiddles: one table per pass after the first, in shared memory or read from global memory
// (rows.cuh chooses per size): entry r L + k of pass s holds W_{L R}^(k r) = exp(-2 pi i k r /
// (L R)). Consecutive threads read consecutive entries, so the reads are conflict-free. A
// shared-memory table is filled once per (persistent) CTA, computed on chip with sincospif (the
// "computed" variants) or copied from a correctly rounded table built in double precision on the
// host (the "_table" variant, twiddles.cu); a global-memory table is one of those two, built once
// per device.

#include "common.cuh"
#include "dft.cuh"
#include "tma.cuh"

#include <type_traits>

namespace spectral::engine {

constexpr int kMinThreads = 256;

// The pass structure of an (N, E) plan as plain functions, so host code (the twiddle tables in
// twiddles.cu, the launchers) evaluates exactly what the kernels compile in. When log2 E does
// not divide log2 N one pass has a smaller radix: the first (where it needs no twiddles) or, with
// `small_last`, the last (which leaves two butterflies per thread there, for mirror pairing).
__host__ __device__ constexpr int plan_passes(int n, int e)
{
    if (n <= 1) {
        return 0;
    }
    const int ln = ilog2(n);
    const int le = ilog2(e);
    return ln / le + (ln % le != 0 ? 1 : 0);
}
__host__ __device__ constexpr int plan_radix(int n, int e, int s, bool small_last = false)
{
    if (e <= 1) {
        return 1;
    }
    const int rem = ilog2(n) % ilog2(e);
    const int small_pass = small_last ? plan_passes(n, e) - 1 : 0;
    return (rem != 0 && s == small_pass) ? (1 << rem) : e;
}
__host__ __device__ constexpr int plan_span(int n, int e, int s, bool small_last = false)
{
    int l = 1;
    for (int i = 0; i < s; ++i) {
        l *= plan_radix(n, e, i, small_last);
    }
    return l;
}
__host__ __device__ constexpr int plan_tw_offset(int n, int e, int s, bool small_last = false)
{
    int o = 0;
    for (int i = 1; i < s; ++i) {
        o += plan_radix(n, e, i, small_last) * plan_span(n, e, i, small_last);
    }
    return o;
}
__host__ __device__ constexpr int plan_tw_entries(int n, int e, bool small_last = false)
{
    return plan_tw_offset(n, e, plan_passes(n, e), small_last);
}

template <int N_, int E_, bool SmallLast_ = false, int MinThreads_ = kMinThreads, int MinBlocks_ = 1>
struct Plan {
    static constexpr int N = N_;
    static constexpr int MIN_BLOCKS = MinBlocks_;  // CTAs per SM the register budget must allow
    static constexpr int E = E_;
    static constexpr bool SmallLast = SmallLast_;
    static_assert(is_pow2(N) && is_pow2(E) && E <= N && E <= 32 && (N == 1 || E >= 2), "bad plan");
    static constexpr int P = N / E;  // threads per transform
    static constexpr int PASSES = plan_passes(N, E);
    static constexpr int THREADS = cmax(MinThreads_, P);  // a CTA holds G = THREADS / P transforms
    static constexpr int G = THREADS / P;  // transforms per CTA

    __host__ __device__ static constexpr int radix(int s) { return plan_radix(N, E, s, SmallLast); }
    __host__ __device__ static constexpr int span(int s) { return plan_span(N, E, s, SmallLast); }
    __host__ __device__ static constexpr int tw_offset(int s) { return plan_tw_offset(N, E, s, SmallLast); }
    static constexpr int TW = plan_tw_entries(N, E, SmallLast);  // entries of all the pass tables
    // Two butterflies per thread in the first / last pass: mirror pairing is possible there.
    static constexpr bool kPairFirst = PASSES >= 1 && E / plan_radix(N, E, 0, SmallLast) == 2;
    static constexpr bool kPairLast = PASSES >= 1 && E / plan_radix(N, E, PASSES - 1, SmallLast) == 2;

    // Storage index of position p in the exchange that follows pass s.
    // Positions per pad entry after pass s (see the exchange layout above).
    __host__ __device__ static constexpr int pad_group(int s)
    {
        return (P >= 16 && span(s) * radix(s) < 16) ? 16 : span(s) * radix(s);
    }
    __host__ __device__ static constexpr int pad(int p, int s)
    {
        return span(s) < 16 ? p + span(s) * (p / pad_group(s)) : p;
    }
    // Slot length. The exchange accesses of one transform's P threads touch 2 P consecutive
    // banks (8-byte values); when P < 16, 32 / P transforms share a warp, and a slot length of
    // P (mod 16) places transform g's accesses at bank 2 P g (mod 32): the transforms of each
    // half-warp take disjoint banks. P = 1 makes it odd, which also lets 16 consecutive slots'
    // same position (the [slot][position] staging reads) fall on distinct banks.
    __host__ __device__ static constexpr int buffer_entries()
    {
        int b = N + 1;
        for (int s = 0; s + 1 < PASSES; ++s) {
            b = cmax(b, pad(N - 1, s) + 1);
        }
        if (P < 16) {
            return b + ((P - b % 16) % 16 + 16) % 16;
        }
        return b | 1;
    }
    static constexpr int BUF = buffer_entries();  // per-transform slot in shared memory
};

// Barrier over the P threads of one transform.
template <int P>
__device__ __forceinline__ void group_sync()
{
    if constexpr (P > 32) {
        __syncthreads();
    } else if constexpr (P > 1) {
        __syncwarp();
    }
}

// Entry idx of a pass table computed on chip: W_{L R}^(k r) for idx = r L + k, by sincospif of
// 2 (k r mod L R) / (L R), a dyadic fraction with at most 15 bits and so exact in float.
__device__ __forceinline__ float2 computed_pass_twiddle(int idx, int L, int R)
{
    const int LR = L * R;
    const int r = idx / L;
    const int k = idx - r * L;
    const float a = 2.0f * static_cast<float>((k * r) & (LR - 1)) / static_cast<float>(LR);
    float sn = 0.0f;
    float cs = 1.0f;
    sincospif(a, &sn, &cs);
    return make_float2(cs, -sn);
}

// W_{2n}^k computed on chip (k / n is exact in float for the sizes used).
__device__ __forceinline__ float2 computed_half_turn(int k, int n)
{
    float sn = 0.0f;
    float cs = 1.0f;
    sincospif(static_cast<float>(k) / static_cast<float>(n), &sn, &cs);
    return make_float2(cs, -sn);
}

// W_M^J = exp(-2 pi i J / M) as a compile-time constant (dft.cuh's cs2pi, rounded once to float).
template <int J, int M>
__device__ __forceinline__ float2 wconst()
{
    constexpr dft::CosSin w = dft::cs2pi(J, M);
    return make_float2(static_cast<float>(w.c), -static_cast<float>(w.s));
}

// Fills the pass tables: computed on chip (Table == false) or copied from `table`.
template <class PL, bool Table>
__device__ __forceinline__ void fill_pass_twiddles(float2* tw, const float2* __restrict__ table)
{
    for (int e = threadIdx.x; e < PL::TW; e += blockDim.x) {
        if constexpr (Table) {
            tw[e] = table[e];
        } else {
            int s = 1;
            while (s + 1 < PL::PASSES && e >= PL::tw_offset(s + 1)) {
                ++s;
            }
            tw[e] = computed_pass_twiddle(e - PL::tw_offset(s), PL::span(s), PL::radix(s));
        }
    }
}

// The barrier around an exchange. CtaSync 0: the transform's own threads (group_sync); 1: the
// whole CTA; otherwise the named barrier CtaSync >> 10 (1 .. 15) over CtaSync & 1023 threads, for
// warp-specialized kernels in which only one group of warps runs the passes.
template <int P, int CtaSync>
__device__ __forceinline__ void exchange_sync()
{
    if constexpr (CtaSync == 1) {
        __syncthreads();
    } else if constexpr (CtaSync > 1) {
        static_assert((CtaSync >> 10) >= 1 && (CtaSync >> 10) <= 15 && (CtaSync & 1023) % 32 == 0,
                      "named barrier: id 1 .. 15, whole warps");
        asm volatile("bar.sync %0, %1;" ::"n"(CtaSync >> 10), "n"(CtaSync & 1023) : "memory");
    } else {
        group_sync<P>();
    }
}

// The butterflies a thread runs in a pass with Q butterflies per thread. Plain: j = t + b P, so
// thread t holds positions t + i P, i = b + r Q. Mirror (Q == 2): butterfly t and its mirror
// 2P - t (thread 0: butterflies 0 and P), which hold each other's positions N - k: the real
// transforms' combine and prepare steps then pair X[k] with X[N - k] in registers.
template <bool Mirror, int P>
__device__ __forceinline__ int butterfly(int t, int b)
{
    if constexpr (Mirror) {
        return b == 0 ? t : (t == 0 ? P : 2 * P - t);
    } else {
        return t + b * P;
    }
}

// One pass of the engine (see the top of this file), with the register layout of the next pass.
//
// Exchange addressing. Rows (Stride == 0): each transform owns a padded slot; position
// p = (j - k) R + k + r L, k = j mod L, is stored at (j - k) (R + 1) + k + r L when L < 16 (this
// is p + L floor(p / (L R)): one gap of L after every L R positions) and at p otherwise.
// Columns (Stride == C): C transforms interleaved, position p of column c at p C + c (the
// caller offsets `buf` by c). Either way a thread's write indices are one runtime base per
// butterfly plus compile-time offsets, and for the plain layout L divides P, so k = t mod L
// and one set of twiddles serves all Q butterflies.
template <class PL, int S, bool Inv, int B, int Stride, int CtaSync, bool Mirror, bool MirrorNext,
          int Derive = 0>
__device__ __forceinline__ void pass(float2 (&v)[PL::E], int t, float2* buf, const float2* tw)
{
    constexpr int E = PL::E;
    constexpr int P = PL::P;
    constexpr int R = PL::radix(S);
    constexpr int L = PL::span(S);
    constexpr int Q = E / R;  // butterflies per thread
    constexpr bool kLast = S == PL::PASSES - 1;
    constexpr int kTw = PL::tw_offset(S);
    constexpr int W = PL::pad_group(S);  // positions per pad entry (a multiple of L R)
    // A mirror first pass of radix R < 16 (the inverse real rows): butterfly 1 of thread t is
    // j = 2 P - t, so a half-warp's 16 butterflies start at an odd j, and with one pad entry per
    // 16 positions its first and last write share a bank pair (a 2-way conflict on every write).
    // This exchange instead permutes each aligned block of 16 positions: position q is stored at
    // q ^ ((q / 16) mod R), which gives any 16 consecutive butterflies distinct bank pairs for
    // each r and keeps a half-warp's 16 consecutive reads inside one block.
    constexpr bool kSwizzle = Stride == 0 && Mirror && !kLast && S == 0 && L == 1 && W == 16 && R < 16;
    constexpr bool kPad = Stride == 0 && L < 16 && !kSwizzle;
    static_assert(!Mirror || Q == 2, "mirror pairing needs two butterflies per thread");
    static_assert(Mirror || kLast || P % L == 0, "the plain exchange layout needs L to divide P");

    // One twiddle set serves every butterfly when k = t mod L is the same for all of them (L
    // divides P); otherwise each butterfly has its own.
    constexpr bool kShared = !Mirror && P % L == 0;
    constexpr int kSets = (S > 0) ? (kShared ? 1 : Q) : 1;
    float2 wt[kSets][R];
    // Radix-16 passes whose twiddles are derived (Derive >= 3, or >= 2 where the table spans 32
    // or more entries per r, i.e. 256-byte loads per warp).
    constexpr bool kDerive16 = !Mirror && kShared && R == 16 && (Derive >= 3 || (Derive >= 2 && L >= 32));
    if constexpr (S > 0 && kDerive16) {
        // W^(k r) for r = r0 + 4 r1: the table's r in {1, 2, 3} and {4, 8, 12}, and one complex
        // product W^(k r0) W^(4 k r1) for each of the other nine (at most two roundings).
        const int k = t & (L - 1);
        dft::static_for<1, 4>([&](auto r_) {
            constexpr int r = decltype(r_)::value;
            wt[0][r] = tw[kTw + r * L + k];
            wt[0][4 * r] = tw[kTw + 4 * r * L + k];
        });
        dft::static_for<1, 4>([&](auto r1_) {
            constexpr int r1 = decltype(r1_)::value;
            dft::static_for<1, 4>([&](auto r0_) {
                constexpr int r0 = decltype(r0_)::value;
                wt[0][r0 + 4 * r1] = cmul(wt[0][r0], wt[0][4 * r1]);
            });
        });
    } else if constexpr (S > 0 && Mirror && Derive >= 1) {
        // Mirror pairs (L = 2P): butterfly 0 is t and reads W_{LR}^(t r) from the table;
        // butterfly 1 is L - t, whose twiddles W_{LR}^((L - t) r) = W_R^r conj(W_{LR}^(t r)) follow
        // with compile-time constants; for t = 0 it is P = L / 2, with twiddles W_{2R}^r.
        static_assert(L == 2 * P, "mirror pairs take positions L - t");
        const int k0 = t & (L - 1);
        dft::static_for<1, R>([&](auto r_) {
            constexpr int r = decltype(r_)::value;
            const float2 w0 = tw[kTw + r * L + k0];
            wt[0][r] = w0;
            const float2 mirror = dft::mul_w<r, R, false>(make_float2(w0.x, -w0.y));
            wt[1][r] = t == 0 ? wconst<r, 2 * R>() : mirror;
        });
    } else if constexpr (S > 0) {
#pragma unroll
        for (int b = 0; b < kSets; ++b) {
            const int k = butterfly<Mirror, P>(t, b) & (L - 1);
#pragma unroll
            for (int r = 1; r < R; ++r) {
                wt[b][r] = tw[kTw + r * L + k];
            }
        }
    }

#pragma unroll
    for (int b = 0; b < Q; ++b) {
        const int j = butterfly<Mirror, P>(t, b);
        const int k = j & (L - 1);
        float2 u[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            u[r] = v[b + r * Q];
            if constexpr (S > 0) {
                if (r > 0) {
                    u[r] = cmul_tw<Inv>(u[r], wt[kShared ? 0 : b][r]);
                }
            }
        }
        dft::Dft<R, B, Inv>::run(u);
        if constexpr (kLast) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                v[b + r * Q] = u[r];
            }
        } else {
            // The R outputs span L R consecutive positions inside one group of W.
            const int pos0 = (j - k) * R + k;
            const int base = kPad ? pos0 + L * (pos0 / W) : pos0;
            const int key = kSwizzle ? (pos0 >> 4) & (R - 1) : 0;  // pos0 = R j: low bits free
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int idx = kSwizzle ? base + (r ^ key) : base + r * L;
                buf[Stride == 0 ? idx : idx * Stride] = u[r];
            }
        }
    }

    if constexpr (!kLast) {
        exchange_sync<P, CtaSync>();
        constexpr int R2 = PL::radix(S + 1);
        constexpr int Q2 = E / R2;
        constexpr int NB2 = PL::N / R2;  // butterflies of the next pass: positions j + r NB2
        if constexpr (MirrorNext) {
#pragma unroll
            for (int b = 0; b < Q2; ++b) {
                const int j = butterfly<true, P>(t, b);
#pragma unroll
                for (int r = 0; r < R2; ++r) {
                    const int q = j + r * NB2;
                    const int idx = kSwizzle ? q ^ ((q >> 4) & (R - 1)) : kPad ? q + L * (q / W) : q;
                    v[b + r * Q2] = buf[Stride == 0 ? idx : idx * Stride];
                }
            }
        } else if constexpr (kSwizzle && (P / 16) % R == 0) {
            // (t + i P) / 16 = t / 16 + i P / 16 with i P / 16 a multiple of R: one key for all i.
            const int base = t ^ ((t >> 4) & (R - 1));
#pragma unroll
            for (int i = 0; i < E; ++i) {
                v[i] = buf[base + i * P];
            }
        } else if constexpr (kSwizzle) {
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const int q = t + i * P;
                v[i] = buf[q ^ ((q >> 4) & (R - 1))];
            }
        } else if constexpr (kPad && P % W == 0) {
            // pad(t + i P) = t + L floor(t / W) + i (P + L P / W), since W divides P.
            const int base = t + L * (t / W);
#pragma unroll
            for (int i = 0; i < E; ++i) {
                v[i] = buf[base + i * (P + L * P / W)];
            }
        } else if constexpr (kPad) {
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const int q = t + i * P;
                v[i] = buf[q + L * (q / W)];
            }
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const int q = t + i * P;
                v[i] = buf[Stride == 0 ? q : q * Stride];
            }
        }
        exchange_sync<P, CtaSync>();
    }
}

// All passes. MirrorFirst / MirrorLast select the mirror layout of the first / last pass: the
// registers before the first pass (the load) or after the last pass (the store) then hold
// butterfly-mirror pairs instead of positions t + i P.
// Derive: 1, the mirror pass takes half its twiddles from the other half and constants (pass
// above) instead of the table; 2 and 3, radix-16 passes also form 9 of their 15 twiddles from
// the other 6 (see pass). For the computed-twiddle variants, whose tables are not correctly
// rounded either.
template <class PL, bool Inv, int B, int Stride = 0, int CtaSync = 0, bool MirrorFirst = false,
          bool MirrorLast = false, int Derive = 0>
__device__ __forceinline__ void run_passes(float2 (&v)[PL::E], int t, float2* buf, const float2* tw)
{
    dft::static_for<0, PL::PASSES>([&](auto s_) {
        constexpr int S = decltype(s_)::value;
        constexpr bool kMirror = (S == 0 && MirrorFirst) || (S == PL::PASSES - 1 && MirrorLast);
        constexpr bool kMirrorNext = S + 1 == PL::PASSES - 1 && MirrorLast;
        pass<PL, S, Inv, B, Stride, CtaSync, kMirror, kMirrorNext, Derive>(v, t, buf, tw);
    });
}

// --- the row kernel ----------------------------------------------------------------------------
//
// Transforms whose elements are contiguous (rows). A CTA holds G transforms side by side and
// walks the batch with a grid stride (persistent CTAs: the twiddle tables are filled once per
// CTA). What a transform reads and writes is the Io policy:
//
//   template <class PL> static constexpr int extra()     extra shared-memory table entries
//   template <class PL, bool Table> void prologue(float2* extra, const float2* extra_table)
//   template <class PL> void load(float2 (&v)[E], const RowCtx&) const
//   template <class PL, bool Inv> void store(float2 (&v)[E], const RowCtx&) const
//
// Loads and stores may stage through shared memory and use __syncthreads(): every thread of a
// CTA runs the same number of iterations, inactive slots included.

// Io policies that split their load into raw global loads (fetch) and arithmetic on them
// (finish) declare kSplitLoad = true.
template <class Io, class = void>
struct split_load : std::false_type {};
template <class Io>
struct split_load<Io, std::void_t<decltype(Io::kSplitLoad)>> : std::bool_constant<Io::kSplitLoad> {};

// Io policies that derive part of their twiddles (kDerive > 0; the level run_passes takes).
template <class Io, class = void>
struct derive_twiddles : std::integral_constant<int, 0> {};
template <class Io>
struct derive_twiddles<Io, std::void_t<decltype(Io::kDerive)>> : std::integral_constant<int, Io::kDerive> {};

struct RowCtx {
    long long tf;        // this slot's transform (valid only when `active`)
    long long tf0;       // the CTA's first transform in this iteration
    int count;           // active slots in this iteration
    int g;               // slot within the CTA
    int t;               // thread within the transform
    bool active;
    float2* buf;         // the slot's exchange buffer
    float2* bufs;        // every slot's buffer (G * BUF entries)
    const float2* extra; // the Io's shared-memory table
};

template <class PL, bool Inv, int B, bool Table, class Io, bool TwGlobal = false, bool Prefetch = false>
__global__ void __launch_bounds__(PL::THREADS, PL::MIN_BLOCKS)
    row_kernel(const Io io, long long batch, const float2* __restrict__ tw_table,
               const float2* __restrict__ extra_table)
{
    wait_for_previous_grid();
    allow_next_grid();
    extern __shared__ float4 smem_raw[];
    // TwGlobal: the tables are read where they lie in global memory (one L1-resident copy per SM
    // instead of one shared-memory copy per CTA, so more CTAs fit).
    float2* tw_s = reinterpret_cast<float2*>(smem_raw);
    float2* extra_s = tw_s + (TwGlobal ? 0 : PL::TW);
    float2* bufs = extra_s + (TwGlobal ? 0 : Io::template extra<PL>());
    const float2* tw = TwGlobal ? tw_table : tw_s;
    const float2* extra = TwGlobal ? extra_table : extra_s;

    if constexpr (!TwGlobal) {
        fill_pass_twiddles<PL, Table>(tw_s, tw_table);
        Io::template prologue<PL, Table>(extra_s, extra_table);
    }
    __syncthreads();

    const int g = threadIdx.x / PL::P;
    const int t = threadIdx.x - g * PL::P;
    auto context = [&](long long tf0) {
        RowCtx c;
        c.tf0 = tf0;
        c.count = static_cast<int>(batch - tf0 < PL::G ? batch - tf0 : PL::G);
        c.g = g;
        c.t = t;
        c.tf = tf0 + g;
        c.active = g < c.count;
        c.buf = bufs + g * PL::BUF;
        c.bufs = bufs;
        c.extra = extra;
        return c;
    };
    const long long stride = static_cast<long long>(gridDim.x) * PL::G;
    if constexpr (Prefetch && split_load<Io>::value) {
        // The next tile's raw loads are issued before this tile's passes; the Io's arithmetic on
        // them (finish) waits for the next iteration.
        long long tf0 = static_cast<long long>(blockIdx.x) * PL::G;
        if (tf0 >= batch) {
            return;
        }
        RowCtx c = context(tf0);
        float2 raw[PL::E + 1];
        io.template fetch<PL>(raw, c);
        for (;;) {
            const long long next = tf0 + stride;
            const bool more = next < batch;
            float2 v[PL::E];
            io.template finish<PL>(v, raw, c);
            const RowCtx cn = context(more ? next : tf0);
            if (more) {
                io.template fetch<PL>(raw, cn);
            }
            run_passes<PL, Inv, B, 0, false, Io::kMirrorFirst, Io::kMirrorLast, derive_twiddles<Io>::value>(v, t, c.buf, tw);
            io.template store<PL, Inv>(v, c);
            if (!more) {
                break;
            }
            c = cn;
            tf0 = next;
        }
    } else if constexpr (Prefetch) {
        // The next tile's loads are issued before this tile's passes, so they are in flight
        // while it computes (for Io policies whose load is plain global loads).
        long long tf0 = static_cast<long long>(blockIdx.x) * PL::G;
        if (tf0 >= batch) {
            return;
        }
        RowCtx c = context(tf0);
        float2 v[PL::E];
        io.template load<PL>(v, c);
        for (;;) {
            const long long next = tf0 + stride;
            const bool more = next < batch;
            RowCtx cn = context(more ? next : tf0);
            float2 vn[PL::E];
            if (more) {
                io.template load<PL>(vn, cn);
            }
            run_passes<PL, Inv, B, 0, false, Io::kMirrorFirst, Io::kMirrorLast, derive_twiddles<Io>::value>(v, t, c.buf, tw);
            io.template store<PL, Inv>(v, c);
            if (!more) {
                break;
            }
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = vn[i];
            }
            c = cn;
            tf0 = next;
        }
    } else {
        for (long long tf0 = static_cast<long long>(blockIdx.x) * PL::G; tf0 < batch; tf0 += stride) {
            const RowCtx c = context(tf0);
            float2 v[PL::E];
            io.template load<PL>(v, c);
            run_passes<PL, Inv, B, 0, false, Io::kMirrorFirst, Io::kMirrorLast, derive_twiddles<Io>::value>(v, t, c.buf, tw);
            io.template store<PL, Inv>(v, c);
        }
    }
}

// --- the staged row kernel --------------------------------------------------------------------
//
// The same transforms as row_kernel, with the input of each tile of G transforms brought into
// shared memory by one bulk copy (cp.async.bulk, the TMA engine) while the CTA computes the
// previous tile: two stage buffers, each with an mbarrier that the copy completes. A CTA therefore
// always has its next 16-64 KiB in flight, whatever its occupancy, which is what keeps a
// persistent FFT kernel at HBM speed: without it every CTA alternates between waiting for its
// loads and computing, and the SM's memory pipe idles while all its CTAs compute.
//
// Once a tile's threads have read their inputs out of a stage buffer, the same buffer serves as
// the tile's exchange buffer (the padded per-transform slots of row_kernel), so staging costs no
// shared memory beyond the second buffer. Per tile: a CTA barrier before reissuing the buffer
// the previous tile used, one after the inputs are read, and the exchanges' own barriers.
//
// Io additionally provides
//   template <class PL> static constexpr int stage_entries()   >= G * BUF and the tile's input
//   bool stage_src(tf0, count, src&, bytes&, shift&) const    the bulk copy of a tile's input
//   template <class PL> void load_staged(v, ctx, tile) const  inputs from the staged tile

template <class PL, class Io>
__host__ __device__ constexpr int stage_entries()
{
    return (cmax(PL::G * PL::BUF, Io::template staged_input_entries<PL>()) + 1) & ~1;
}

template <class PL, bool Inv, int B, bool Table, class Io, bool TwGlobal = false>
__global__ void __launch_bounds__(PL::THREADS, PL::MIN_BLOCKS)
    staged_row_kernel(const Io io, long long batch, const float2* __restrict__ tw_table,
                      const float2* __restrict__ extra_table, unsigned* fault)
{
    wait_for_previous_grid();
    allow_next_grid();
    extern __shared__ float4 smem_raw[];
    constexpr int kExtra = TwGlobal ? 0 : (Io::template extra<PL>() + 1) & ~1;
    constexpr int kTw = TwGlobal ? 0 : (PL::TW + 1) & ~1;
    constexpr int kStage = stage_entries<PL, Io>();
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);  // two mbarriers, 16 bytes
    float2* tw_s = reinterpret_cast<float2*>(smem_raw + 1);
    float2* extra_s = tw_s + kTw;
    float2* stages = extra_s + kExtra;  // 16-byte aligned: every region above is an even count
    const float2* tw = TwGlobal ? tw_table : tw_s;
    const float2* extra = TwGlobal ? extra_table : extra_s;

    if constexpr (!TwGlobal) {
        fill_pass_twiddles<PL, Table>(tw_s, tw_table);
        Io::template prologue<PL, Table>(extra_s, extra_table);
    }
    if (threadIdx.x == 0) {
        tma::mbar_init(&bars[0], 1);
        tma::mbar_init(&bars[1], 1);
        tma::fence_mbar_init();
    }
    __syncthreads();

    const long long stride = static_cast<long long>(gridDim.x) * PL::G;
    const long long first = static_cast<long long>(blockIdx.x) * PL::G;
    auto issue = [&](int s, long long tf0) {
        const int count = static_cast<int>(batch - tf0 < PL::G ? batch - tf0 : PL::G);
        const float2* src = nullptr;
        unsigned bytes = 0;
        int shift = 0;
        io.template stage_src<PL>(tf0, count, src, bytes, shift);
        tma::mbar_arrive_expect_tx(&bars[s], bytes);
        tma::bulk_g2s(stages + s * kStage, src, bytes, &bars[s]);
    };
    if (threadIdx.x == 0 && first < batch) {
        issue(0, first);
    }

    const int g = threadIdx.x / PL::P;
    const int t = threadIdx.x - g * PL::P;
    int j = 0;
    for (long long tf0 = first; tf0 < batch; tf0 += stride, ++j) {
        const int s = j & 1;
        // The other buffer's previous tile is finished with: every thread orders its generic
        // accesses to it (the exchanges) before the bulk copy that refills it.
        tma::fence_proxy_async();
        __syncthreads();
        if (threadIdx.x == 0 && tf0 + stride < batch) {
            issue(s ^ 1, tf0 + stride);
        }
        const bool ok = tma::mbar_wait(&bars[s], static_cast<unsigned>(j >> 1) & 1u);
        if (__syncthreads_or(!ok)) {
            // A copy never completed: record it, let the copy this CTA issued last drain (also
            // bounded) so nothing lands in shared memory after the CTA is gone, and stop.
            if (threadIdx.x == 0) {
                atomicOr(fault, tma::kFaultWaitTimeout);
                if (tf0 + stride < batch
                    && !tma::mbar_wait(&bars[s ^ 1], static_cast<unsigned>((j + 1) >> 1) & 1u)) {
                    atomicOr(fault, tma::kFaultDrainTimeout);
                }
            }
            return;
        }
        float2* stage = stages + s * kStage;
        RowCtx c;
        c.tf0 = tf0;
        c.count = static_cast<int>(batch - tf0 < PL::G ? batch - tf0 : PL::G);
        c.g = g;
        c.t = t;
        c.tf = tf0 + g;
        c.active = g < c.count;
        c.buf = stage + g * PL::BUF;
        c.bufs = stage;
        c.extra = extra;

        float2 v[PL::E];
        {
            const float2* src = nullptr;
            unsigned bytes = 0;
            int shift = 0;
            io.template stage_src<PL>(tf0, c.count, src, bytes, shift);
            io.template load_staged<PL>(v, c, stage + shift);
        }
        __syncthreads();  // every input read before the exchanges reuse the buffer
        run_passes<PL, Inv, B, 0, false, Io::kMirrorFirst, Io::kMirrorLast, derive_twiddles<Io>::value>(v, t, c.buf, tw);
        io.template store<PL, Inv>(v, c);
    }
}

template <class PL, class Io, bool TwGlobal = false>
constexpr std::size_t staged_smem_bytes()
{
    return 16
           + sizeof(float2)
                 * ((TwGlobal ? 0 : static_cast<std::size_t>((PL::TW + 1) & ~1)
                                        + ((Io::template extra<PL>() + 1) & ~1))
                    + 2 * static_cast<std::size_t>(stage_entries<PL, Io>()));
}

template <class PL, class Io, bool TwGlobal = false>
constexpr std::size_t row_smem_bytes()
{
    return sizeof(float2)
           * ((TwGlobal ? 0 : static_cast<std::size_t>(PL::TW) + Io::template extra<PL>())
              + static_cast<std::size_t>(PL::G) * PL::BUF);
}

// --- Io policies for rows ----------------------------------------------------------------------

// Complex rows. Unpruned: rows of N in and out. Pruned (the reference's PrunedFns::c2c,
// fft.hpp:62-78): input rows hold only the first keep_in values (the rest are zero), output rows
// only the first keep_out values. `scale` multiplies every output (1/N for the inverse).
struct C2cIo {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = false;
    const float2* x;
    float2* y;
    int keep_in;
    int keep_out;
    float scale;

    template <class PL>
    __host__ __device__ static constexpr int extra() { return 0; }
    template <class PL, bool Table>
    __device__ static void prologue(float2*, const float2*) {}

    // Staged (unpruned input only): a tile is count * N contiguous values.
    template <class PL>
    __host__ __device__ static constexpr int staged_input_entries() { return PL::G * PL::N; }
    template <class PL>
    __device__ __forceinline__ void stage_src(long long tf0, int count, const float2*& src,
                                              unsigned& bytes, int& shift) const
    {
        src = x + tf0 * PL::N;
        bytes = static_cast<unsigned>(count) * static_cast<unsigned>(PL::N) * 8u;
        shift = 0;
    }
    template <class PL>
    __device__ __forceinline__ void load_staged(float2 (&v)[PL::E], const RowCtx& c,
                                                const float2* tile) const
    {
        const float2* row = tile + c.g * PL::N + c.t;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = c.active ? row[i * PL::P] : make_float2(0.0f, 0.0f);
        }
    }

    // One thread per transform (P = 1, N <= 16): each warp's 32 transforms are 32 N contiguous
    // values, loaded and stored coalesced and transposed through the warp's own slots (odd
    // length: both the [slot][position] writes and reads are conflict-free). Every lane takes
    // part, active or not.
    template <class PL>
    __device__ __forceinline__ void load_warp_transposed(float2 (&v)[PL::E], const RowCtx& c) const
    {
        constexpr int N = PL::N;
        const int lane = c.g & 31;
        const int g0 = c.g - lane;
        const int live = c.count - g0;  // transforms of this warp that exist (may be <= 0 or > 32)
        const float2* src = x + (c.tf0 + g0) * N;
        float2* slots = c.bufs + g0 * PL::BUF;
        __syncwarp();  // every lane is done with its slot from the previous tile (the Io's store)
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int e = i * 32 + lane;
            const int g = e / N;
            if (g < live) {
                slots[g * PL::BUF + (e - g * N)] = __ldg(src + e);
            }
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < N; ++i) {
            v[i] = c.active ? slots[lane * PL::BUF + i] : make_float2(0.0f, 0.0f);
        }
    }

    template <class PL, bool Inv>
    __device__ __forceinline__ void store_warp_transposed(float2 (&v)[PL::E], const RowCtx& c) const
    {
        constexpr int N = PL::N;
        const int lane = c.g & 31;
        const int g0 = c.g - lane;
        const int live = c.count - g0;
        float2* dst = y + (c.tf0 + g0) * N;
        float2* slots = c.bufs + g0 * PL::BUF;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            slots[lane * PL::BUF + i] = Inv ? cscale(v[i], scale) : v[i];
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int e = i * 32 + lane;
            const int g = e / N;
            if (g < live) {
                dst[e] = slots[g * PL::BUF + (e - g * N)];
            }
        }
        __syncwarp();  // the slots are read before the next tile's load refills them
    }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        if constexpr (PL::P == 1 && PL::N > 1) {
            if (keep_in == PL::N) {
                load_warp_transposed<PL>(v, c);
                return;
            }
        }
        if (!c.active) {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = make_float2(0.0f, 0.0f);
            }
            return;
        }
        if (keep_in == PL::N) {
            const float2* row = x + c.tf * PL::N + c.t;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = __ldg(row + i * PL::P);
            }
        } else {
            const float2* row = x + c.tf * keep_in;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                const int pos = c.t + i * PL::P;
                v[i] = pos < keep_in ? __ldg(row + pos) : make_float2(0.0f, 0.0f);
            }
        }
    }

    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        if constexpr (PL::P == 1 && PL::N > 1) {
            if (keep_out == PL::N) {
                store_warp_transposed<PL, Inv>(v, c);
                return;
            }
        }
        if (!c.active) {
            return;
        }
        if (keep_out == PL::N) {
            float2* row = y + c.tf * PL::N + c.t;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                row[i * PL::P] = Inv ? cscale(v[i], scale) : v[i];
            }
        } else {
            float2* row = y + c.tf * keep_out;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                const int pos = c.t + i * PL::P;
                if (pos < keep_out) {
                    row[pos] = Inv ? cscale(v[i], scale) : v[i];
                }
            }
        }
    }
};

// Fills extra[k] = W_{2N}^k = exp(-pi i k / N), k = 0 .. N: the twiddles of the real-transform
// combine and prepare steps for n = 2N real points.
template <class PL, bool Table>
__device__ __forceinline__ void fill_half_turn(float2* w, const float2* __restrict__ table)
{
    for (int k = threadIdx.x; k <= PL::N; k += blockDim.x) {
        if constexpr (Table) {
            w[k] = table[k];
        } else {
            w[k] = computed_half_turn(k, PL::N);
        }
    }
}

// X[k] of the 2N-point real transform from zk = Z[k mod N], zmk = Z[(N - k) mod N] of the
// N-point transform of the packed input and w = W_{2N}^k (the standard packing identity, as in
// the reference's real.cuh:31-42):
//   E = (Z[k] + conj Z[N-k]) / 2,  O = (Z[k] - conj Z[N-k]) / (2i),  X[k] = E + w O.
__device__ __forceinline__ float2 r2c_combine(float2 zk, float2 zmk, float2 w)
{
    const float ex = 0.5f * (zk.x + zmk.x);
    const float ey = 0.5f * (zk.y - zmk.y);
    const float ox = 0.5f * (zk.y + zmk.y);   // O = -i D with D = (Z[k] - conj Z[N-k]) / 2
    const float oy = -0.5f * (zk.x - zmk.x);
    return make_float2(ex + fmaf(w.x, ox, -(w.y * oy)), ey + fmaf(w.x, oy, w.y * ox));
}

// Z[k] = E + i O from xk = X[k], xmk = X[N - k] and w = W_{2N}^k, the inverse of the combine
// (real.cuh:46-61 in the reference): E = (X[k] + conj X[N-k]) / 2,
// O = (X[k] - conj X[N-k]) conj(w) / 2. At k = 0 the imaginary parts of X[0] and X[N] are
// dropped, as numpy and torch do.
__device__ __forceinline__ float2 c2r_prepare(float2 xk, float2 xmk, float2 w)
{
    const float ex = 0.5f * (xk.x + xmk.x);
    const float ey = 0.5f * (xk.y - xmk.y);
    const float dx = 0.5f * (xk.x - xmk.x);
    const float dy = 0.5f * (xk.y + xmk.y);
    const float ox = fmaf(dx, w.x, dy * w.y);   // D conj(w), w = (c, -s)
    const float oy = fmaf(dy, w.x, -(dx * w.y));
    return make_float2(ex - oy, ey + ox);
}

// Real input rows (the reference's R2cIo, stockham.cuh:273-307): rows of 2N floats read as N
// complex values (the memory layout is the same), an N-point forward transform, then the
// combine into the first `keep` (<= N + 1) outputs per row, staged through the slot buffer so
// each output can read Z[k] and Z[N - k].
struct R2cIo {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = false;
    const float2* x;  // rows of N packed complex values
    float2* y;        // rows of `keep` complex outputs
    int keep;

    template <class PL>
    __host__ __device__ static constexpr int extra() { return PL::N + 1; }
    template <class PL, bool Table>
    __device__ static void prologue(float2* w, const float2* table) { fill_half_turn<PL, Table>(w, table); }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        C2cIo{x, nullptr, PL::N, PL::N, 1.0f}.template load<PL>(v, c);
    }

    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        constexpr int N = PL::N;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            c.buf[c.t + i * PL::P] = v[i];
        }
        group_sync<PL::P>();
        if (c.active) {
            float2* row = y + c.tf * keep;
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                const int k = c.t + i * PL::P;
                if (k < keep) {
                    row[k] = r2c_combine(c.buf[k], c.buf[(N - k) & (N - 1)], c.extra[k]);
                }
            }
            if (c.t == 0 && N < keep) {
                row[N] = r2c_combine(c.buf[0], c.buf[0], c.extra[N]);
            }
        }
        group_sync<PL::P>();
    }
};

// Real output rows (the reference's C2rIo, stockham.cuh:314-340): rows of `keep` (<= N + 1)
// complex inputs, the rest zero; the load prepares Z[k] from X[k] and X[N - k] (an ascending and
// a descending run, both coalesced), an N-point inverse transform, and the store writes z / N as
// 2N reals.
struct C2rIo {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = false;
    const float2* x;  // rows of `keep` complex inputs
    float2* y;        // rows of N complex values = 2N reals
    int keep;
    float scale;      // 1 / N

    template <class PL>
    __host__ __device__ static constexpr int extra() { return PL::N + 1; }
    template <class PL, bool Table>
    __device__ static void prologue(float2* w, const float2* table) { fill_half_turn<PL, Table>(w, table); }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        constexpr int N = PL::N;
        const float2 zero = make_float2(0.0f, 0.0f);
        if (!c.active) {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = zero;
            }
            return;
        }
        const float2* row = x + c.tf * keep;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = c.t + i * PL::P;
            float2 xk = k < keep ? __ldg(row + k) : zero;
            float2 xmk = N - k < keep ? __ldg(row + (N - k)) : zero;
            if (k == 0) {
                xk.y = 0.0f;
                xmk.y = 0.0f;
            }
            v[i] = c2r_prepare(xk, xmk, c.extra[k]);
        }
    }

    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        if (!c.active) {
            return;
        }
        float2* row = y + c.tf * PL::N + c.t;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            row[i * PL::P] = cscale(v[i], scale);
        }
    }
};

// --- mirror-paired real transforms -------------------------------------------------------------
//
// For plans with two butterflies per thread in the last pass (real-to-complex) or the first pass
// (complex-to-real), the engine can give each thread butterfly t together with its mirror 2P - t
// (run_passes' MirrorLast / MirrorFirst), whose positions are exactly the N - k of the first's. The
// real-transform step, which pairs Z[k] with Z[N - k] (or X[k] with X[N - k]), then happens in
// registers: no staging of the spectrum in shared memory, no barrier, every input read once, and
// one twiddle and one complex product for each pair of outputs:
//   forward  X[k] = E + W^k O,   X[N - k] = conj(E - W^k O)
//   inverse  Z[k] = E + i O,     Z[N - k] = conj(E - i O),   O = D conj(W^k)
// with E, O (forward) and E, D (inverse) as in r2c_combine / c2r_prepare.

// Writes X[k] and X[N - k] (only those below `keep`) from zk = Z[k], zmk = Z[N - k], w = W_{2N}^k.
__device__ __forceinline__ void r2c_pair(float2* row, int n, int k, int keep, float2 zk, float2 zmk,
                                         float2 w)
{
    const float ex = 0.5f * (zk.x + zmk.x);
    const float ey = 0.5f * (zk.y - zmk.y);
    const float ox = 0.5f * (zk.y + zmk.y);
    const float oy = -0.5f * (zk.x - zmk.x);
    const float wx = fmaf(w.x, ox, -(w.y * oy));
    const float wy = fmaf(w.x, oy, w.y * ox);
    if (k < keep) {
        row[k] = make_float2(ex + wx, ey + wy);
    }
    if (n - k != k && n - k < keep) {
        row[n - k] = make_float2(ex - wx, wy - ey);
    }
}

// Z[k] and Z[N - k] from xa = X[k], xb = X[N - k], w = W_{2N}^k, times 2 `half` (half = 1/2 gives
// the prepare step itself; the inverse's 1 / N folded in gives half = 1 / (2N), a power of two, so
// the results are the same bits as scaling the outputs afterwards).
__device__ __forceinline__ void c2r_pair(int k, float2 xa, float2 xb, float2 w, float2& zk, float2& zmk,
                                         float half = 0.5f)
{
    if (k == 0) {
        xa.y = 0.0f;
        xb.y = 0.0f;
    }
    const float ex = half * (xa.x + xb.x);
    const float ey = half * (xa.y - xb.y);
    const float dx = half * (xa.x - xb.x);
    const float dy = half * (xa.y + xb.y);
    const float ox = fmaf(dx, w.x, dy * w.y);
    const float oy = fmaf(dy, w.x, -(dx * w.y));
    zk = make_float2(ex - oy, ey + ox);
    zmk = make_float2(ex + oy, ox - ey);
}

// Real input rows with the combine in registers (plans with SmallLast and kPairLast). Derive: the
// combine's twiddles W_{2N}^(t + r NB) = W_{2N}^t W_{2R}^r come from one table entry and
// constants (thread 0's are all constants), and the last pass derives its mirror twiddles.
template <int Derive>
struct R2cPairIoT {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = true;
    static constexpr int kDerive = Derive;
    const float2* x;
    float2* y;
    int keep;

    template <class PL>
    __host__ __device__ static constexpr int extra() { return PL::N + 1; }
    template <class PL, bool Table>
    __device__ static void prologue(float2* w, const float2* table) { fill_half_turn<PL, Table>(w, table); }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        C2cIo{x, nullptr, PL::N, PL::N, 1.0f}.template load<PL>(v, c);
    }
    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        static_assert(PL::kPairLast, "needs two butterflies per thread in the last pass");
        if (!c.active) {
            return;
        }
        constexpr int N = PL::N;
        constexpr int P = PL::P;
        constexpr int R = PL::radix(PL::PASSES - 1);
        constexpr int NB = N / R;  // = 2P: positions of butterfly j are j + r NB
        float2* row = y + c.tf * keep;
        const int t = c.t;
        if constexpr (Derive >= 1) {
            static_assert(NB == 2 * P, "half-turn twiddles W_{2N}^(t + r NB) = W_{2N}^t W_{2R}^r");
            if (t != 0) {
                const float2 base = c.extra[t];
                dft::static_for<0, R>([&](auto r_) {
                    constexpr int r = decltype(r_)::value;
                    const float2 w = r == 0 ? base : dft::mul_w<r, 2 * R, false>(base);
                    r2c_pair(row, N, t + r * NB, keep, v[2 * r], v[1 + 2 * (R - 1 - r)], w);
                });
            } else {
                r2c_pair(row, N, 0, keep, v[0], v[0], make_float2(1.0f, 0.0f));  // X[0] and X[N]
                dft::static_for<1, R / 2 + 1>([&](auto r_) {
                    constexpr int r = decltype(r_)::value;
                    r2c_pair(row, N, r * NB, keep, v[2 * r], v[2 * (R - r)], wconst<r, 2 * R>());
                });
                dft::static_for<0, R / 2>([&](auto r_) {
                    constexpr int r = decltype(r_)::value;  // W_{2N}^(P + r NB) = W_{4R}^(1 + 2r)
                    r2c_pair(row, N, P + r * NB, keep, v[1 + 2 * r], v[1 + 2 * (R - 1 - r)],
                             wconst<1 + 2 * r, 4 * R>());
                });
            }
        } else if (t != 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int k = t + r * NB;
                r2c_pair(row, N, k, keep, v[2 * r], v[1 + 2 * (R - 1 - r)], c.extra[k]);
            }
        } else {
            r2c_pair(row, N, 0, keep, v[0], v[0], c.extra[0]);  // X[0] and X[N]
#pragma unroll
            for (int r = 1; r <= R / 2; ++r) {
                r2c_pair(row, N, r * NB, keep, v[2 * r], v[2 * (R - r)], c.extra[r * NB]);
            }
#pragma unroll
            for (int r = 0; r < R / 2; ++r) {
                r2c_pair(row, N, P + r * NB, keep, v[1 + 2 * r], v[1 + 2 * (R - 1 - r)],
                         c.extra[P + r * NB]);
            }
        }
    }
};
using R2cPairIo = R2cPairIoT<0>;

// Complex rows of `keep` values to real rows with the prepare step in registers (plans with
// kPairFirst). X[N] (the Nyquist value) is read by thread 0 alone. Derive: the prepare step's
// twiddles come from one table entry and constants, as in R2cPairIoT.
template <int Derive>
struct C2rPairIoT {
    static constexpr bool kMirrorFirst = true;
    static constexpr bool kMirrorLast = false;
    static constexpr int kDerive = Derive;
    const float2* x;
    float2* y;
    int keep;
    float scale;  // 1 / N

    template <class PL>
    __host__ __device__ static constexpr int extra() { return PL::N + 1; }
    template <class PL, bool Table>
    __device__ static void prologue(float2* w, const float2* table) { fill_half_turn<PL, Table>(w, table); }

    // The prepare step in two halves: gather the inputs of the thread's two mirrored butterflies
    // (raw[0 .. R-1] and raw[R .. 2R-1]; raw[2R] = X[N] for thread 0), then combine them. Split,
    // the gather of the next tile can be issued before this tile's passes (kSplitLoad).
    static constexpr bool kSplitLoad = true;

    template <class PL, class Get>
    __device__ __forceinline__ void gather(float2 (&raw)[PL::E + 1], const RowCtx& c, Get&& get) const
    {
        static_assert(PL::kPairFirst, "needs two butterflies per thread in the first pass");
        constexpr int R = PL::radix(0);
        constexpr int NB = PL::N / R;  // = 2P
#pragma unroll
        for (int r = 0; r < R; ++r) {
            raw[r] = get(butterfly<true, PL::P>(c.t, 0) + r * NB);
            raw[R + r] = get(butterfly<true, PL::P>(c.t, 1) + r * NB);
        }
        raw[2 * R] = c.t == 0 ? get(PL::N) : make_float2(0.0f, 0.0f);
    }

    template <class PL>
    __device__ __forceinline__ void combine(float2 (&v)[PL::E], const float2 (&raw)[PL::E + 1],
                                            const RowCtx& c) const
    {
        constexpr int N = PL::N;
        constexpr int P = PL::P;
        constexpr int R = PL::radix(0);
        constexpr int NB = N / R;  // = 2P
        const int t = c.t;
        const float half = 0.5f * scale;  // the 1 / N of the inverse, folded in exactly
        const float2* a = raw;
        const float2* b = raw + R;
        if constexpr (Derive >= 1) {
            static_assert(NB == 2 * P, "half-turn twiddles W_{2N}^(t + r NB) = W_{2N}^t W_{2R}^r");
            if (t != 0) {
                const float2 base = c.extra[t];
                dft::static_for<0, R>([&](auto r_) {
                    constexpr int r = decltype(r_)::value;
                    const float2 w = r == 0 ? base : dft::mul_w<r, 2 * R, false>(base);
                    c2r_pair(t + r * NB, a[r], b[R - 1 - r], w, v[2 * r], v[1 + 2 * (R - 1 - r)], half);
                });
            } else {
                float2 unused;
                c2r_pair(0, a[0], raw[2 * R], make_float2(1.0f, 0.0f), v[0], unused, half);
                dft::static_for<1, R / 2 + 1>([&](auto r_) {
                    constexpr int r = decltype(r_)::value;
                    c2r_pair(r * NB, a[r], a[R - r], wconst<r, 2 * R>(), v[2 * r], v[2 * (R - r)], half);
                });
                dft::static_for<0, R / 2>([&](auto r_) {
                    constexpr int r = decltype(r_)::value;
                    c2r_pair(P + r * NB, b[r], b[R - 1 - r], wconst<1 + 2 * r, 4 * R>(), v[1 + 2 * r],
                             v[1 + 2 * (R - 1 - r)], half);
                });
            }
        } else if (t != 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int k = t + r * NB;
                c2r_pair(k, a[r], b[R - 1 - r], c.extra[k], v[2 * r], v[1 + 2 * (R - 1 - r)], half);
            }
        } else {
            float2 unused;
            c2r_pair(0, a[0], raw[2 * R], c.extra[0], v[0], unused, half);
#pragma unroll
            for (int r = 1; r <= R / 2; ++r) {
                c2r_pair(r * NB, a[r], a[R - r], c.extra[r * NB], v[2 * r], v[2 * (R - r)], half);
            }
#pragma unroll
            for (int r = 0; r < R / 2; ++r) {
                c2r_pair(P + r * NB, b[r], b[R - 1 - r], c.extra[P + r * NB], v[1 + 2 * r],
                         v[1 + 2 * (R - 1 - r)], half);
            }
        }
    }

    template <class PL, class Get>
    __device__ __forceinline__ void prepare(float2 (&v)[PL::E], const RowCtx& c, Get&& get) const
    {
        float2 raw[PL::E + 1];
        gather<PL>(raw, c, get);
        combine<PL>(v, raw, c);
    }

    template <class PL>
    __device__ __forceinline__ void fetch(float2 (&raw)[PL::E + 1], const RowCtx& c) const
    {
        if (!c.active) {
#pragma unroll
            for (int i = 0; i <= PL::E; ++i) {
                raw[i] = make_float2(0.0f, 0.0f);
            }
            return;
        }
        const float2* row = x + c.tf * keep;
        const int kp = keep;
        gather<PL>(raw, c, [&](int k) { return k < kp ? __ldg(row + k) : make_float2(0.0f, 0.0f); });
    }

    template <class PL>
    __device__ __forceinline__ void finish(float2 (&v)[PL::E], const float2 (&raw)[PL::E + 1],
                                           const RowCtx& c) const
    {
        if (!c.active) {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = make_float2(0.0f, 0.0f);
            }
            return;
        }
        combine<PL>(v, raw, c);
    }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        const float2 zero = make_float2(0.0f, 0.0f);
        if (!c.active) {
#pragma unroll
            for (int i = 0; i < PL::E; ++i) {
                v[i] = zero;
            }
            return;
        }
        const float2* row = x + c.tf * keep;
        const int kp = keep;
        prepare<PL>(v, c, [&](int k) { return k < kp ? __ldg(row + k) : zero; });
    }

    // The 1 / N scale was applied in the prepare step (combine).
    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        if (!c.active) {
            return;
        }
        float2* row = y + c.tf * PL::N + c.t;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            row[i * PL::P] = v[i];
        }
    }
};
using C2rPairIo = C2rPairIoT<0>;

}  // namespace spectral::engine
