#pragma once

// Fused pruned 2D real transforms for FNO spectral convolutions: one kernel per direction, one
// field per CTA iteration, the intermediate kept in shared memory.
//
// The reference runs these as two launches with an n1 x m2 intermediate in global memory
// (csrc/fft/pruned.cu:163-209): 67 MB of extra traffic at 128 x 128 x 4096 fields. Here the
// whole field fits on chip. Forward (rfft2_truncated): the N1 rows are real transforms of
// M = N2 / 2 packed complex points (RG rows at a time, P_r threads each), combined into only
// their m2 kept outputs, which go into a [row][column] tile in shared memory; then the m2 kept
// columns are N1-point transforms in the column-interleaved layout, and only the 2 m1 kept rows
// are written out. The inverse runs the same steps backwards. Global memory sees the field once
// and the modes once: 4 n1 n2 + 8 (2 m1 m2) bytes per field and direction.

#include "columns.cuh"

namespace spectral::engine {

template <int N1, int N2, int B, bool Table, int T = 256, bool Compact = true>
struct Pruned2d {
    static constexpr int M = N2 / 2;  // packed complex points per row
    using RP = PlanFor<M>;
    using CP = PlanFor<N1>;
    static constexpr int THREADS = T;
    static_assert(RP::P <= THREADS && CP::P <= THREADS, "field too large for one CTA");
    static constexpr int RG = THREADS / RP::P;  // rows in flight
    static constexpr int CW = THREADS / CP::P;  // columns in flight: the largest m2 supported
    // The [row][column] tile: rows of CW entries. When they are whole 128-byte lines, a
    // half-warp of the row stage (16 / RP::P rows, RP::P consecutive columns each) would hit the
    // same bank pairs in every row, so each row permutes its column chunks: column c of row r is
    // stored at tcol(r, c) = c ^ ((r mod 16 / RP::P) RP::P), which puts those rows' chunks on
    // distinct bank pairs and keeps every aligned block of 16 columns (a half-warp of the column
    // stage) in place as a set. This replaces 8 pad entries per row: a third less shared memory.
    // Without `Compact` the rows keep the 8 pad entries instead (fewer index operations for a
    // kernel whose occupancy is set by its registers, not its shared memory).
    static constexpr int CS = CW % 16 == 0 && !Compact ? CW + 8 : CW;
    static constexpr bool kPermute = CW % 16 == 0 && Compact;
    static_assert(RP::P <= 16, "a half-warp must span whole rows");
    __device__ static int tcol(int r, int c)
    {
        if constexpr (kPermute) {
            return c ^ ((r & (16 / RP::P - 1)) * RP::P);
        } else {
            return c;
        }
    }

    static constexpr int kTwR = (RP::TW + 1) & ~1;
    static constexpr int kHalf = (M + 2) & ~1;
    static constexpr int kTwC = (CP::TW + 1) & ~1;
    static constexpr int kRowBuf = RG * RP::BUF;
    static constexpr int kColBuf = N1 * CS;
    static constexpr std::size_t kSmem = sizeof(float2) * (kTwR + kHalf + kTwC + kRowBuf + kColBuf);

    struct Smem {
        float2* twr;
        float2* half;
        float2* twc;
        float2* rowbuf;
        float2* colbuf;
    };

    __device__ static Smem carve(float2* base)
    {
        Smem s;
        s.twr = base;
        s.half = s.twr + kTwR;
        s.twc = s.half + kHalf;
        s.rowbuf = s.twc + kTwC;
        s.colbuf = s.rowbuf + kRowBuf;
        return s;
    }

    __device__ static void fill(const Smem& s, const float2* twr_g, const float2* half_g,
                                const float2* twc_g)
    {
        fill_pass_twiddles<RP, Table>(s.twr, twr_g);
        fill_half_turn<RP, Table>(s.half, half_g);
        fill_pass_twiddles<CP, Table>(s.twc, twc_g);
    }
};

template <int N1, int N2, int B, bool Table, int T, int MinBlocks, bool Compact>
__global__ void __launch_bounds__(T, MinBlocks)
    pruned2d_forward(const float2* __restrict__ x, float2* __restrict__ modes, long long fields,
                     int m1, int m2, const float2* __restrict__ twr_g,
                     const float2* __restrict__ half_g, const float2* __restrict__ twc_g)
{
    wait_for_previous_grid();
    allow_next_grid();
    using K = Pruned2d<N1, N2, B, Table, T, Compact>;
    using RP = typename K::RP;
    using CP = typename K::CP;
    constexpr int M = K::M;
    extern __shared__ float4 smem_raw[];
    const typename K::Smem s = K::carve(reinterpret_cast<float2*>(smem_raw));
    K::fill(s, twr_g, half_g, twc_g);
    __syncthreads();

    const int rg = threadIdx.x / RP::P;
    const int rt = threadIdx.x - rg * RP::P;
    const int cc = threadIdx.x % K::CW;
    const int ct = threadIdx.x / K::CW;
    float2* slot = s.rowbuf + rg * RP::BUF;
    const float2 zero = make_float2(0.0f, 0.0f);

    // Each row group's loads are issued one group ahead (after a field's last group, the next
    // field's first), so every thread has two groups of loads in flight while it computes.
    float2 next[RP::E];
    auto load_group = [&](long long f, int r0) {
        const int r = r0 + rg;
        const bool act = f < fields && r < N1;
#pragma unroll
        for (int i = 0; i < RP::E; ++i) {
            next[i] = act ? __ldg(x + f * (static_cast<long long>(N1) * M) + r * M + rt + i * RP::P) : zero;
        }
    };
    load_group(blockIdx.x, 0);

    for (long long f = blockIdx.x; f < fields; f += gridDim.x) {
        // Rows: real transforms, only the m2 kept outputs, into the [row][column] tile.
        for (int r0 = 0; r0 < N1; r0 += K::RG) {
            const int r = r0 + rg;
            const bool act = r < N1;
            float2 v[RP::E];
#pragma unroll
            for (int i = 0; i < RP::E; ++i) {
                v[i] = next[i];
            }
            if (r0 + K::RG < N1) {
                load_group(f, r0 + K::RG);
            } else {
                load_group(f + gridDim.x, 0);
            }
            run_passes<RP, false, B>(v, rt, slot, s.twr);
            // Combine the m2 kept outputs. Thread rt holds Z[rt + i P]; the partner Z[M - k] of
            // k = rt + i P is register E-1-i of thread P - rt in the same warp (a row's P <= 32
            // threads are consecutive lanes), or, for rt = 0, its own register (E - i) mod E. So
            // a shuffle replaces staging the row's spectrum in shared memory.
            static_assert(RP::P <= 32, "a row's threads must share a warp");
            const int lane = threadIdx.x & 31;
            const int partner = (lane & ~(RP::P - 1)) | ((RP::P - rt) & (RP::P - 1));
#pragma unroll
            for (int i = 0; i < RP::E; ++i) {
                if (i * RP::P >= m2) {
                    break;  // uniform across the warp: depends on i only
                }
                const float2 mine = v[RP::E - 1 - i];
                float2 zmk;
                zmk.x = __shfl_sync(0xffffffffu, mine.x, partner);
                zmk.y = __shfl_sync(0xffffffffu, mine.y, partner);
                if (rt == 0) {
                    zmk = v[(RP::E - i) % RP::E];
                }
                const int k = rt + i * RP::P;
                if (act && k < m2) {
                    s.colbuf[r * K::CS + K::tcol(r, k)] = r2c_combine(v[i], zmk, s.half[k]);
                }
            }
            if (act && rt == 0 && M < m2) {  // the Nyquist output, X[M] = Z[0].x - Z[0].y
                s.colbuf[r * K::CS + K::tcol(r, M)] = r2c_combine(v[0], v[0], s.half[M]);
            }
        }
        __syncthreads();
        // Columns: N1-point transforms of the m2 kept columns, only the 2 m1 kept rows written.
        float2 v[CP::E];
#pragma unroll
        for (int i = 0; i < CP::E; ++i) {
            const int row = ct + i * CP::P;
            v[i] = s.colbuf[row * K::CS + K::tcol(row, cc)];
        }
        __syncthreads();
        run_passes<CP, false, B, K::CS, true>(v, ct, s.colbuf + cc, s.twc);
        if (cc < m2) {
            float2* mf = modes + f * (2LL * m1 * m2);
#pragma unroll
            for (int i = 0; i < CP::E; ++i) {
                const int row = mode_row(ct + i * CP::P, N1, m1);
                if (row >= 0) {
                    mf[row * m2 + cc] = v[i];
                }
            }
        }
        __syncthreads();
    }
}

template <int N1, int N2, int B, bool Table, int T, int MinBlocks, bool Compact>
__global__ void __launch_bounds__(T, MinBlocks)
    pruned2d_inverse(const float2* __restrict__ modes, float2* __restrict__ y, long long fields,
                     int m1, int m2, const float2* __restrict__ twr_g,
                     const float2* __restrict__ half_g, const float2* __restrict__ twc_g)
{
    wait_for_previous_grid();
    allow_next_grid();
    using K = Pruned2d<N1, N2, B, Table, T, Compact>;
    using RP = typename K::RP;
    using CP = typename K::CP;
    constexpr int M = K::M;
    extern __shared__ float4 smem_raw[];
    const typename K::Smem s = K::carve(reinterpret_cast<float2*>(smem_raw));
    K::fill(s, twr_g, half_g, twc_g);
    __syncthreads();

    const int rg = threadIdx.x / RP::P;
    const int rt = threadIdx.x - rg * RP::P;
    const int cc = threadIdx.x % K::CW;
    const int ct = threadIdx.x / K::CW;
    float2* slot = s.rowbuf + rg * RP::BUF;
    const float2 zero = make_float2(0.0f, 0.0f);

    for (long long f = blockIdx.x; f < fields; f += gridDim.x) {
        // Columns: the kept rows of each kept column, the rest zero, N1-point inverse transforms.
        const float2* mf = modes + f * (2LL * m1 * m2);
        float2 v[CP::E];
#pragma unroll
        for (int i = 0; i < CP::E; ++i) {
            const int row = mode_row(ct + i * CP::P, N1, m1);
            v[i] = (cc < m2 && row >= 0) ? __ldg(mf + row * m2 + cc) : zero;
        }
        run_passes<CP, true, B, K::CS, true>(v, ct, s.colbuf + cc, s.twc);
        __syncthreads();  // the last exchange's reads (and the previous field's rows) are done
        constexpr float kColScale = 1.0f / N1;
        if (cc < m2) {
#pragma unroll
            for (int i = 0; i < CP::E; ++i) {
                const int row = ct + i * CP::P;
                s.colbuf[row * K::CS + K::tcol(row, cc)] = cscale(v[i], kColScale);
            }
        }
        __syncthreads();
        // Rows: real inverse transforms from the m2 kept values of each row (the rest zero).
        float2* yf = y + f * (static_cast<long long>(N1) * M);
        constexpr float kRowScale = 1.0f / M;
        for (int r0 = 0; r0 < N1; r0 += K::RG) {
            const int r = r0 + rg;
            const bool act = r < N1;
            float2 u[RP::E];
#pragma unroll
            for (int i = 0; i < RP::E; ++i) {
                const int k = rt + i * RP::P;
                const bool has_k = act && k < m2;
                const bool has_mk = act && M - k < m2;
                u[i] = zero;
                if (has_k || has_mk) {  // most of a row's spectrum is zero: skip it whole
                    float2 xk = has_k ? s.colbuf[r * K::CS + K::tcol(r, k)] : zero;
                    float2 xmk = has_mk ? s.colbuf[r * K::CS + K::tcol(r, M - k)] : zero;
                    if (k == 0) {
                        xk.y = 0.0f;
                        xmk.y = 0.0f;
                    }
                    u[i] = c2r_prepare(xk, xmk, s.half[k]);
                }
            }
            run_passes<RP, true, B>(u, rt, slot, s.twr);
            if (act) {
#pragma unroll
                for (int i = 0; i < RP::E; ++i) {
                    yf[r * M + rt + i * RP::P] = cscale(u[i], kRowScale);
                }
            }
        }
        __syncthreads();
    }
}

template <int B, bool Table>
struct Pruned2dEngine {
    static constexpr int kMin = 16;
    static constexpr int kMax = 256;

    static bool supported(int n1, int n2, int m1, int m2)
    {
        if (!is_pow2(n1) || !is_pow2(n2) || n1 < kMin || n2 < kMin || n1 > kMax || n2 > kMax) {
            return false;
        }
        bool ok = false;
        dispatch_pow2<kMin, kMax>(n1, [&](auto n1_) {
            constexpr int N1 = decltype(n1_)::value;
            ok = m1 >= 1 && 2 * m1 <= n1 && m2 >= 1 && m2 <= Pruned2d<N1, kMin, B, Table>::CW
                 && m2 <= n2 / 2 + 1;
        });
        return ok;
    }

    // The forward kernel's loads run a row group ahead, so it gains from every CTA that fits:
    // it takes the compact tile. The inverse is limited by its registers, not its shared memory,
    // and keeps the padded tile, which needs fewer index operations.
    static constexpr bool kCompactForward = true;
    static constexpr bool kCompactInverse = false;

    template <int N1, int N2, int T, int MinBlocks, bool Compact, bool Forward>
    static void launch_with(const float2* in, float2* out, int m1, int m2, long long fields,
                            cudaStream_t stream)
    {
        using K = Pruned2d<N1, N2, B, Table, T, Compact>;
        auto kernel = Forward ? pruned2d_forward<N1, N2, B, Table, T, MinBlocks, Compact>
                              : pruned2d_inverse<N1, N2, B, Table, T, MinBlocks, Compact>;
        static std::atomic<int> cache[kMaxDevices];
        const float2* twr = Table ? twiddles::pass_table(K::M, K::RP::E) : nullptr;
        const float2* half = Table ? twiddles::half_turn(K::M) : nullptr;
        const float2* twc = Table ? twiddles::pass_table(N1, K::CP::E) : nullptr;
        const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel), K::THREADS,
                                              K::kSmem, cache, fields);
        launch_pdl(kernel, grid, static_cast<unsigned>(K::THREADS), K::kSmem, stream, in, out, fields,
                   m1, m2, twr, half, twc);
    }

    template <int N1, int N2, int T, bool Forward>
    static void launch(const float2* in, float2* out, int m1, int m2, long long fields, cudaStream_t stream)
    {
        // MinBlocks 0 leaves the register budget to the compiler (__launch_bounds__ with a
        // minimum of 1 CTA per SM lets it take 106-140 registers here instead of 77-96).
        launch_with<N1, N2, T, 0, Forward ? kCompactForward : kCompactInverse, Forward>(in, out, m1, m2,
                                                                                       fields, stream);
    }

    template <bool Forward>
    static void run(const float2* in, float2* out, int n1, int n2, int m1, int m2, long long fields,
                    cudaStream_t stream)
    {
        dispatch_pow2<kMin, kMax>(n1, [&](auto n1_) {
            dispatch_pow2<kMin, kMax>(n2, [&](auto n2_) {
                constexpr int N1 = decltype(n1_)::value;
                constexpr int N2 = decltype(n2_)::value;
                // 128-thread CTAs hold half the columns in flight: where the kept columns fit,
                // the column stage computes no discarded columns and twice the CTAs fit per SM.
                if (m2 <= Pruned2d<N1, N2, B, Table, 128>::CW) {
                    launch<N1, N2, 128, Forward>(in, out, m1, m2, fields, stream);
                } else {
                    launch<N1, N2, 256, Forward>(in, out, m1, m2, fields, stream);
                }
            });
        });
    }

    static void forward(const float* x, float2* modes, int n1, int n2, int m1, int m2,
                        long long fields, cudaStream_t s)
    {
        run<true>(reinterpret_cast<const float2*>(x), modes, n1, n2, m1, m2, fields, s);
    }

    static void inverse(const float2* modes, float* y, int n1, int n2, int m1, int m2,
                        long long fields, cudaStream_t s)
    {
        run<false>(modes, reinterpret_cast<float2*>(y), n1, n2, m1, m2, fields, s);
    }
};

}  // namespace spectral::engine
