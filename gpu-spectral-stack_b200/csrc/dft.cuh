#pragma once

// In-register DFTs of 2 to 32 points with compile-time twiddle constants.
//
// Dft<R, B, Inv>::run(v) replaces v[0 .. R-1] by its R-point DFT, in natural order in and out,
// with the forward sign exp(-2 pi i k n / R) or, for Inv, the inverse sign exp(+2 pi i k n / R)
// (unscaled). Every index is a compile-time constant, so the whole transform lives in registers.
//
// B is the building block: the largest DFT written out directly (2, 4 or 8 points). Larger
// sizes split as R = B x (R / B): B-point DFTs down the columns of an B x (R / B) view, a
// multiplication by exp(-+2 pi i k1 n2 / R), then (R / B)-point DFTs along the rows. This is
// the radix-B decomposition the registry's stockham_r2 / _r4 / _r8 names select; it changes the
// arithmetic (r2 spends the most additions and multiplications) but not the memory traffic.
//
// Multiplications by twiddle constants are specialised at compile time: angles that are
// multiples of pi/2 cost only sign flips and swaps, odd multiples of pi/4 cost two
// multiplications, and only the rest are full complex products. The constants are computed in
// double precision at compile time by cs2pi() below and rounded once to float.

#include "common.cuh"

#include <type_traits>

namespace spectral::dft {

// --- compile-time helpers ----------------------------------------------------------------------

template <int Begin, int End, class F>
__host__ __device__ __forceinline__ constexpr void static_for(F&& f)
{
    if constexpr (Begin < End) {
        f(std::integral_constant<int, Begin>{});
        static_for<Begin + 1, End>(static_cast<F&&>(f));
    }
}

struct CosSin {
    double c;
    double s;
};

// Taylor series around 0, accurate to double rounding for |x| <= pi / 4.
__host__ __device__ constexpr double taylor_sin(double x)
{
    double term = x;
    double sum = x;
    for (int k = 1; k < 16; ++k) {
        term *= -x * x / static_cast<double>((2 * k) * (2 * k + 1));
        sum += term;
    }
    return sum;
}

__host__ __device__ constexpr double taylor_cos(double x)
{
    double term = 1.0;
    double sum = 1.0;
    for (int k = 1; k < 16; ++k) {
        term *= -x * x / static_cast<double>((2 * k - 1) * (2 * k));
        sum += term;
    }
    return sum;
}

// cos and sin of 2 pi j / m for integers j, m > 0. The angle is first reduced exactly (in
// integers) into [0, pi/4] with the symmetries of the circle, so the series only ever sees a
// small argument and the result is accurate to about one unit in the last place of a double.
__host__ __device__ constexpr CosSin cs2pi(long long j, long long m)
{
    j %= m;
    if (j < 0) {
        j += m;
    }
    if (2 * j > m) {  // t in (1/2, 1): reflect about the real axis
        const CosSin r = cs2pi(m - j, m);
        return {r.c, -r.s};
    }
    if (4 * j > m) {  // t in (1/4, 1/2]: cos(2 pi t) = -cos(2 pi (1/2 - t))
        const CosSin r = cs2pi(m - 2 * j, 2 * m);
        return {-r.c, r.s};
    }
    if (8 * j > m) {  // t in (1/8, 1/4]: swap cos and sin about pi/4
        const CosSin r = cs2pi(m - 4 * j, 4 * m);
        return {r.s, r.c};
    }
    constexpr double kTwoPi = 6.283185307179586476925286766559;
    const double x = kTwoPi * static_cast<double>(j) / static_cast<double>(m);
    return {taylor_cos(x), taylor_sin(x)};
}

// --- multiplication by a constant twiddle W_M^J = exp(-+2 pi i J / M) --------------------------

template <int J, int M, bool Inv>
__device__ __forceinline__ float2 mul_w(float2 a)
{
    constexpr int j = ((J % M) + M) % M;
    if constexpr (j == 0) {
        return a;
    } else if constexpr ((8 * j) % M == 0) {
        // Forward factor exp(-i pi o / 4); the inverse uses the conjugate, octant 8 - o.
        constexpr int o = Inv ? 8 - (8 * j) / M : (8 * j) / M;
        constexpr float h = 0.70710678118654752440f;
        if constexpr (o == 4) {
            return make_float2(-a.x, -a.y);
        } else if constexpr (o == 2) {  // -i
            return make_float2(a.y, -a.x);
        } else if constexpr (o == 6) {  // +i
            return make_float2(-a.y, a.x);
        } else if constexpr (o == 1) {  // h (1 - i)
            return make_float2(h * (a.x + a.y), h * (a.y - a.x));
        } else if constexpr (o == 3) {  // h (-1 - i)
            return make_float2(h * (a.y - a.x), -h * (a.x + a.y));
        } else if constexpr (o == 5) {  // h (-1 + i)
            return make_float2(-h * (a.x + a.y), h * (a.x - a.y));
        } else {  // o == 7: h (1 + i)
            return make_float2(h * (a.x - a.y), h * (a.x + a.y));
        }
    } else {
        constexpr CosSin w = cs2pi(j, M);
        constexpr float c = static_cast<float>(w.c);
        constexpr float s = static_cast<float>(w.s);
        if constexpr (Inv) {  // a (c + i s)
            return make_float2(fmaf(a.x, c, -(a.y * s)), fmaf(a.y, c, a.x * s));
        } else {  // a (c - i s)
            return make_float2(fmaf(a.x, c, a.y * s), fmaf(a.y, c, -(a.x * s)));
        }
    }
}

// --- the DFTs ----------------------------------------------------------------------------------

template <int R, int B, bool Inv>
struct Dft;

template <int B, bool Inv>
struct Dft<1, B, Inv> {
    __device__ __forceinline__ static void run(float2 (&)[1]) {}
};

template <int B, bool Inv>
struct Dft<2, B, Inv> {
    __device__ __forceinline__ static void run(float2 (&v)[2])
    {
        const float2 a = v[0];
        v[0] = cadd(a, v[1]);
        v[1] = csub(a, v[1]);
    }
};

// Split R = A x C with A = min(B, R / 2): A-point DFTs over n1 for each n2 (input n = C n1 + n2),
// twiddles W_R^(k1 n2), then C-point DFTs over n2 for each k1 (output k = k1 + A k2).
template <int A, int C, int B, bool Inv>
__device__ __forceinline__ void dft_split(float2 (&v)[A * C])
{
    float2 y[A][C];
    static_for<0, C>([&](auto n2_) {
        constexpr int n2 = decltype(n2_)::value;
        float2 u[A];
        static_for<0, A>([&](auto n1_) { u[decltype(n1_)::value] = v[C * decltype(n1_)::value + n2]; });
        Dft<A, B, Inv>::run(u);
        static_for<0, A>([&](auto k1_) {
            constexpr int k1 = decltype(k1_)::value;
            y[k1][n2] = mul_w<k1 * n2, A * C, Inv>(u[k1]);
        });
    });
    static_for<0, A>([&](auto k1_) {
        constexpr int k1 = decltype(k1_)::value;
        float2 w[C];
        static_for<0, C>([&](auto n2_) { w[decltype(n2_)::value] = y[k1][decltype(n2_)::value]; });
        Dft<C, B, Inv>::run(w);
        static_for<0, C>([&](auto k2_) {
            constexpr int k2 = decltype(k2_)::value;
            v[k1 + A * k2] = w[k2];
        });
    });
}

// The 4-point DFT written out: X0 = (a + c) + (b + d), X2 = (a + c) - (b + d),
// X1 = (a - c) -+ i (b - d), X3 = (a - c) +- i (b - d).
template <bool Inv>
__device__ __forceinline__ void dft4(float2 (&v)[4])
{
    const float2 s02 = cadd(v[0], v[2]);
    const float2 d02 = csub(v[0], v[2]);
    const float2 s13 = cadd(v[1], v[3]);
    const float2 d13 = csub(v[1], v[3]);
    v[0] = cadd(s02, s13);
    v[2] = csub(s02, s13);
    // d02 -+ i d13: the rotation swaps real and imaginary parts, so it stays scalar (a packed
    // operand would need the swapped pair built first).
    if constexpr (Inv) {
        v[1] = make_float2(d02.x - d13.y, d02.y + d13.x);
        v[3] = make_float2(d02.x + d13.y, d02.y - d13.x);
    } else {
        v[1] = make_float2(d02.x + d13.y, d02.y - d13.x);
        v[3] = make_float2(d02.x - d13.y, d02.y + d13.x);
    }
}

template <int R, int B, bool Inv>
struct Dft {
    static_assert(R >= 4 && (R & (R - 1)) == 0, "power-of-two DFT sizes only");
    __device__ __forceinline__ static void run(float2 (&v)[R])
    {
        if constexpr (R == 4 && B >= 4) {
            dft4<Inv>(v);
        } else if constexpr (R == 8 && B >= 8) {
            // Radix 8 as 4 x 2 with the three non-trivial factors at pi/4 multiples.
            dft_split<4, 2, 4, Inv>(v);
        } else {
            constexpr int A = B < R ? B : R / 2;
            dft_split<A, R / A, B, Inv>(v);
        }
    }
};

}  // namespace spectral::dft
