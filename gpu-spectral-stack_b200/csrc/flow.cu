// One stage of the Navier-Stokes solver's time step (the predictor or the corrector of IMEX
// Crank-Nicolson / Heun) on the pruned spectral layout, in three kernels. The reference's GPU
// solver (python/spectral/flow/gpu.py:115-129) evaluates the nonlinear term with a stack of four
// derived spectra, one batched inverse 2D transform into four physical fields, their product in
// PyTorch, one forward transform, and elementwise PyTorch passes for the mask, the forcing and
// the update: the four physical fields (4 n^2 floats per trajectory) go through global memory
// twice. Here the physical fields never leave the chip:
//
//   derive    (column kernel) column kx of trajectory b, field q: the pruned column of the
//             state times the field's factor (i ky / |k|^2, -i kx / |k|^2, i kx or i ky), an
//             inverse n-point column transform -> Y[q][b][y][kx], y = 0 .. n-1, kx < m;
//   product   (row kernel) row y of trajectory b: the four fields' real inverse row transforms
//             (C2R of their m kept columns), u wx + v wy in registers, the forward real
//             transform of the product, its m kept columns -> Z[b][y][kx];
//   update    (column kernel) column kx of Z[b]: the forward n-point column transform, its 2m kept
//             rows, then N = that * mask, F = f_hat - N and the stage's update:
//               predictor  f0 = F,  out = (E w + dt F) I
//               corrector  out = (E w + dt/2 (f0 + F)) I
//             (E = 1 + dt/2 L, I = 1 / (1 - dt/2 L), L = -nu |k|^2 - alpha, real per mode).
//
// Y and Z (5 n m complex values per trajectory) are the only intermediates; at the reference's
// throughput configuration (256 trajectories of 128^2, m = 43) they take 56 MB, inside the L2.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "columns.cuh"

#include <string>
#include <type_traits>

namespace spectral {
namespace {

using namespace engine;

// Column kx of field q of trajectory b: f = (q batch + b) m + kx.
struct DeriveColumnIo {
    const float2* w;       // (batch, 2m, m) pruned state
    const float2* derive;  // (4, 2m, m)
    float2* y;             // (4, batch, n, m)
    long long batch;
    int m;
    float scale;           // 1 / n

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        const long long qb = c.active ? c.f / m : 0;
        const int col = static_cast<int>(c.f - qb * m);
        const long long q = qb / batch;
        const long long b = qb - q * batch;
        const float2* ws = w + b * 2 * m * m + col;
        const float2* ds = derive + q * 2 * m * m + col;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int row = mode_row(c.t + i * PL::P, PL::N, m);
            v[i] = (c.active && row >= 0) ? cmul(__ldg(ws + row * m), __ldg(ds + row * m)) : make_float2(0.0f, 0.0f);
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
            return;
        }
        const long long qb = c.f / m;
        const int col = static_cast<int>(c.f - qb * m);
        float2* out = y + qb * PL::N * m + col;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            out[static_cast<long long>(c.t + i * PL::P) * m] = cscale(v[i], scale);
        }
    }
};

// Row r = b n + y: the four fields' rows of m values at y + (q rows + r) m. The kernel's own
// passes transform field 0 (u); the store transforms the other three and the product.
template <int B>
struct ProductRowIo {
    static constexpr bool kMirrorFirst = false;
    static constexpr bool kMirrorLast = false;
    const float2* y;   // (4, batch n, m)
    float2* z;         // (batch n, m)
    const float2* tw;  // the plan's pass tables in global memory
    long long rows;    // batch n
    int m;
    float scale;       // 1 / M^2: both factors come unscaled from M-point inverse transforms

    template <class PL>
    __host__ __device__ static constexpr int extra() { return PL::N + 1; }
    template <class PL, bool Table>
    __device__ static void prologue(float2* w, const float2* table) { fill_half_turn<PL, Table>(w, table); }

    template <class PL>
    __device__ __forceinline__ void field(float2 (&v)[PL::E], const RowCtx& c, int q) const
    {
        C2rIo{y + q * rows * m, nullptr, m, 1.0f}.template load<PL>(v, c);
    }

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const RowCtx& c) const
    {
        field<PL>(v, c, 0);
    }

    // The raw loads of field q's row (X[k] and X[M - k] of every element k the thread prepares),
    // issued early so that they are in flight during the previous field's passes; finish() is
    // C2rIo's prepare step on them.
    template <class PL>
    __device__ __forceinline__ void fetch(float2 (&a)[PL::E], float2 (&b)[PL::E], const RowCtx& c, int q) const
    {
        constexpr int N = PL::N;
        const float2 zero = make_float2(0.0f, 0.0f);
        const float2* row = y + (q * rows + c.tf) * m;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = c.t + i * PL::P;
            a[i] = (c.active && k < m) ? __ldg(row + k) : zero;
            b[i] = (c.active && N - k < m) ? __ldg(row + (N - k)) : zero;
        }
    }

    template <class PL>
    __device__ __forceinline__ void finish(float2 (&v)[PL::E], float2 (&a)[PL::E], float2 (&b)[PL::E],
                                           const RowCtx& c) const
    {
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int k = c.t + i * PL::P;
            if (k == 0) {
                a[i].y = 0.0f;
                b[i].y = 0.0f;
            }
            v[i] = c2r_prepare(a[i], b[i], c.extra[k]);
        }
    }

    template <class PL, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const RowCtx& c) const
    {
        // v = u as packed real pairs (x[2k], x[2k+1]); a product of real fields is the packed
        // product of the pairs. Each field's loads are issued before the previous field's passes.
        float2 acc[PL::E];
        float2 t[PL::E];
        float2 a[PL::E];
        float2 b[PL::E];
        fetch<PL>(a, b, c, 2);
        finish<PL>(t, a, b, c);
        fetch<PL>(a, b, c, 1);
        run_passes<PL, true, B>(t, c.t, c.buf, tw);
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            acc[i] = __fmul2_rn(v[i], t[i]);  // u wx
        }
        finish<PL>(v, a, b, c);
        fetch<PL>(a, b, c, 3);
        run_passes<PL, true, B>(v, c.t, c.buf, tw);
        finish<PL>(t, a, b, c);
        run_passes<PL, true, B>(t, c.t, c.buf, tw);
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            acc[i] = cscale(__ffma2_rn(v[i], t[i], acc[i]), scale);  // (u wx + v wy) / M^2, exact scale
        }
        run_passes<PL, false, B>(acc, c.t, c.buf, tw);
        R2cIo{nullptr, z, m}.template store<PL, false>(acc, c);
    }
};

// Column kx of trajectory b: f = b m + kx.
struct UpdateColumnIo {
    const float2* z;        // (batch, n, m)
    const float2* w;        // (batch, 2m, m) the state at the start of the step
    float2* f0;             // (batch, 2m, m) the predictor's tendency
    float2* out;            // (batch, 2m, m); may be w (each element is read and written by one thread)
    const float2* forcing;  // (2m, m), masked
    const float* mask;      // (2m, m)
    const float* expl;      // (., 2m, m): 1 + dt/2 L
    const float* impl;      // (., 2m, m): 1 / (1 - dt/2 L)
    long long visc_stride;  // 2 m m when each trajectory has its own viscosity, else 0
    int m;
    float dt;
    int stage;              // 0 predictor, 1 corrector

    template <class PL>
    __device__ __forceinline__ void load(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        const long long b = c.active ? c.f / m : 0;
        const int col = static_cast<int>(c.f - b * m);
        const float2* zs = z + b * PL::N * m + col;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            v[i] = c.active ? zs[static_cast<long long>(c.t + i * PL::P) * m] : make_float2(0.0f, 0.0f);
        }
    }

    template <class PL, int C, bool Inv>
    __device__ __forceinline__ void store(float2 (&v)[PL::E], const ColumnCtx& c) const
    {
        if (!c.active) {
            return;
        }
        const long long b = c.f / m;
        const int col = static_cast<int>(c.f - b * m);
        const long long plane = 2LL * m * m;
#pragma unroll
        for (int i = 0; i < PL::E; ++i) {
            const int row = mode_row(c.t + i * PL::P, PL::N, m);
            if (row < 0) {
                continue;
            }
            // The operations and their order are the reference's float32 ones, each rounded
            // (no contraction into fused multiply-adds).
            const int k = row * m + col;
            const long long s = b * plane + k;
            const float mk = __ldg(mask + k);
            const float2 fh = __ldg(forcing + k);
            const float2 tend = make_float2(__fsub_rn(fh.x, __fmul_rn(v[i].x, mk)), __fsub_rn(fh.y, __fmul_rn(v[i].y, mk)));
            const float e = __ldg(expl + b * visc_stride + k);
            const float ii = __ldg(impl + b * visc_stride + k);
            const float2 ws = w[s];
            const float2 held = make_float2(__fmul_rn(e, ws.x), __fmul_rn(e, ws.y));
            float2 r;
            if (stage == 0) {
                f0[s] = tend;
                r = make_float2(__fadd_rn(held.x, __fmul_rn(dt, tend.x)), __fadd_rn(held.y, __fmul_rn(dt, tend.y)));
            } else {
                const float2 f = f0[s];
                const float h = 0.5f * dt;
                r = make_float2(__fadd_rn(held.x, __fmul_rn(h, __fadd_rn(f.x, tend.x))),
                                __fadd_rn(held.y, __fmul_rn(h, __fadd_rn(f.y, tend.y))));
            }
            out[s] = make_float2(__fmul_rn(r.x, ii), __fmul_rn(r.y, ii));
        }
    }
};

template <class F>
void with_variant(const char* impl, F&& f)
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
        throw InvalidArgument("flow_stage: no fused kernels for implementation '" + name
                              + "' (the stockham implementations have them)");
    }
}

void need(bool ok, const std::string& message)
{
    if (!ok) {
        throw InvalidArgument(message);
    }
}

struct StageArgs {
    const float2* x;
    const float2* w;
    float2* f0;
    float2* out;
    const float2* derive;
    const float2* forcing;
    const float* mask;
    const float* expl;
    const float* impl;
    long long visc_stride;
    float2* work;
    long long batch;
    int m;
    float dt;
    int stage;
};

template <int N, int B, bool Table>
void run_stage(const StageArgs& a, cudaStream_t s)
{
    constexpr int M = N / 2;
    // Register budgets for occupancy: the column stages are latency-bound loops over small
    // columns (up to n = 128: 64 registers, 8 CTAs of 128 threads per SM); the product stage
    // holds three rows of registers (up to n = 256: two CTAs per SM). At n = 128 nothing spills.
    using CP = Plan<N, default_e(N), false, default_threads(N), (N <= 128 ? 8 : N == 256 ? 3 : 1)>;
    constexpr RowChoice rc = row_choice(RowKind::C2r, M);
    using RP = Plan<M, default_e(M), false, rc.threads, (M <= 128 ? 2 : 1)>;
    const long long fields = 4 * a.batch;
    float2* y = a.work;
    float2* z = a.work + fields * N * a.m;
    launch_columns<CP, true, B, Table>(DeriveColumnIo{a.x, a.derive, y, a.batch, a.m, 1.0f / N},
                                       fields * a.m, s);
    const float2* tw = row_pass_table<RP, Table, false>();
    const float2* half = row_half_turn<M, Table, false>();
    const long long rows = a.batch * N;
    launch_rows<RP, true, B, Table, false, rc.persistent>(
        ProductRowIo<B>{y, z, tw, rows, a.m, 1.0f / (static_cast<float>(M) * M)}, rows, s, half);
    launch_columns<CP, false, B, Table>(
        UpdateColumnIo{z, a.w, a.f0, a.out, a.forcing, a.mask, a.expl, a.impl, a.visc_stride, a.m, a.dt, a.stage},
        a.batch * a.m, s);
}

void check_stage(int n, int m, long long batch)
{
    need(n >= 16 && n <= 512 && (n & (n - 1)) == 0,
         "flow_stage: n must be a power of two from 16 to 512, got " + std::to_string(n));
    need(m >= 1 && 2 * m <= n, "flow_stage: need 1 <= m <= n/2, got m = " + std::to_string(m));
    need(batch >= 0, "flow_stage: batch must not be negative");
}

}  // namespace
}  // namespace spectral

extern "C" int spectral_flow_workspace(int n, int m, long long batch, size_t* count)
{
    using namespace spectral;
    try {
        check_stage(n, m, batch);
        need(count != nullptr, "flow_workspace: count must not be null");
        *count = static_cast<size_t>(5) * static_cast<size_t>(batch) * n * m;
        return SPECTRAL_OK;
    } catch (const InvalidArgument& e) {
        set_last_error(e.what());
        return SPECTRAL_INVALID_ARGUMENT;
    }
}

extern "C" int spectral_flow_stage(const char* impl, const void* x, const void* w, void* f0, void* out,
                                   const void* derive, const void* forcing, const float* mask,
                                   const float* explicit_factor, const float* implicit_factor,
                                   long long visc_stride, void* work, int n, int m, long long batch,
                                   float dt, int stage, void* stream)
{
    using namespace spectral;
    try {
        check_stage(n, m, batch);
        need(stage == 0 || stage == 1, "flow_stage: stage must be 0 (predictor) or 1 (corrector)");
        need(visc_stride == 0 || visc_stride == 2LL * m * m, "flow_stage: visc_stride must be 0 or 2 m m");
        need(out != x && (stage == 1 || out != w), "flow_stage: out must not be x (nor w for the predictor)");
        for (const void* p : {x, w, static_cast<const void*>(f0), static_cast<const void*>(out), derive, forcing,
                              static_cast<const void*>(work)}) {
            need((reinterpret_cast<unsigned long long>(p) & 7u) == 0, "flow_stage: arrays must be 8-byte aligned");
        }
        with_variant(impl, [&](auto b_, auto table_) {
            if (batch == 0) {
                return;
            }
            const StageArgs a{static_cast<const float2*>(x), static_cast<const float2*>(w), static_cast<float2*>(f0),
                              static_cast<float2*>(out), static_cast<const float2*>(derive),
                              static_cast<const float2*>(forcing), mask, explicit_factor, implicit_factor,
                              visc_stride, static_cast<float2*>(work), batch, m, dt, stage};
            const auto s = static_cast<cudaStream_t>(stream);
            dispatch_pow2<16, 512>(n, [&](auto n_) {
                run_stage<decltype(n_)::value, decltype(b_)::value, decltype(table_)::value>(a, s);
            });
        });
        return SPECTRAL_OK;
    } catch (const InvalidArgument& e) {
        set_last_error(e.what());
        return SPECTRAL_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return SPECTRAL_CUDA_ERROR;
    }
}
