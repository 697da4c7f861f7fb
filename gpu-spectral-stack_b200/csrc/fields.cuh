#pragma once

// Whole-field 2D real transforms (rfft2 / irfft2) in one kernel per direction, for fields whose
// row spectrum fits comfortably in L2. Each CTA takes whole fields: the row transforms write the
// field's row spectrum to a scratch region in global memory, the same CTA then runs the column
// transforms out of it, and finally discards the region from L2 (discard.global.L2), so the
// intermediate is written and read through L2 only and never reaches HBM. HBM sees each field's
// input once and its output once: 4 n1 n2 + 8 n1 (n2/2+1) bytes per field, half of what a row
// pass and a column pass through global memory move (the reference's fft2_r2c / fft2_c2r,
// csrc/fft/fft2d.cu:132-187 there).
//
// The row spectrum of a real field has n2/2 + 1 columns; its DC and Nyquist columns are real, so
// the scratch holds M = n2/2 columns, column 0 packing X[., 0] + i X[., M] into one complex column
// that the column stage transforms once and separates (forward). The inverse builds that packed
// column from the Hermitian parts of the two spectrum columns: the row transforms use only the
// real parts of their DC and Nyquist inputs, which are exactly the inverse transforms of those
// Hermitian parts, so a non-Hermitian spectrum gives what numpy and torch give.

#include "columns.cuh"
#include "twiddles.cuh"

namespace spectral::engine {

template <int N1, int N2>
struct Fields {
    static constexpr int M = N2 / 2;
    using RP = PlanFor<M>;
    using CP = PlanFor<N1>;
    static constexpr int THREADS = 256;
    static_assert(RP::P <= 32 && CP::P <= THREADS, "field shape outside the kernel's range");
    static constexpr int RG = THREADS / RP::P;  // rows in flight
    static constexpr int CF = THREADS / CP::P;  // columns in flight
    static constexpr int kRowBuf = RG * RP::BUF;
    static constexpr int kColBuf = N1 * CF;
    static constexpr int kWork = ((kRowBuf > kColBuf ? kRowBuf : kColBuf) + 1) & ~1;
    static constexpr std::size_t kSmem = sizeof(float2) * (kWork + N1);
    static constexpr long long kScratch = static_cast<long long>(N1) * M;  // per field
};

// Drops the lines of [p, p + bytes) from L2 without writing them back (their contents become
// undefined); p and bytes are multiples of 128. The block's reads of the range must be complete
// (a barrier before).
__device__ __forceinline__ void discard_l2(const float2* p, long long bytes)
{
    const char* base = reinterpret_cast<const char*>(p);
    for (long long off = static_cast<long long>(threadIdx.x) * 128; off < bytes;
         off += static_cast<long long>(blockDim.x) * 128) {
        asm volatile("discard.global.L2 [%0], 128;" ::"l"(base + off) : "memory");
    }
}

template <int N1, int N2, int B>
__global__ void __launch_bounds__(256)
    fields_forward(const float2* __restrict__ x, float2* __restrict__ y, float2* __restrict__ scratch,
                   long long fields, bool discard, const float2* __restrict__ twr,
                   const float2* __restrict__ half, const float2* __restrict__ twc)
{
    using K = Fields<N1, N2>;
    using RP = typename K::RP;
    using CP = typename K::CP;
    constexpr int M = K::M;
    extern __shared__ float4 smem_raw[];
    float2* work = reinterpret_cast<float2*>(smem_raw);
    float2* packed = work + K::kWork;

    const int rg = threadIdx.x / RP::P;
    const int rt = threadIdx.x - rg * RP::P;
    const int cc = threadIdx.x % K::CF;
    const int ct = threadIdx.x / K::CF;
    float2* slot = work + rg * RP::BUF;
    const int lane = threadIdx.x & 31;
    const int partner = (lane & ~(RP::P - 1)) | ((RP::P - rt) & (RP::P - 1));

    for (long long f = blockIdx.x; f < fields; f += gridDim.x) {
        const float2* xf = x + f * K::kScratch;  // N1 rows of M packed complex values
        float2* sf = scratch + f * K::kScratch;
        // Rows: M-point transforms of the packed real rows, combined into X[k], k = 0 .. M;
        // column 0 of the scratch packs the real X[0] and X[M].
        for (int r0 = 0; r0 < N1; r0 += K::RG) {
            const int r = r0 + rg;
            const bool act = r < N1;
            float2 v[RP::E];
#pragma unroll
            for (int i = 0; i < RP::E; ++i) {
                v[i] = act ? __ldg(xf + static_cast<long long>(r) * M + rt + i * RP::P)
                           : make_float2(0.0f, 0.0f);
            }
            run_passes<RP, false, B>(v, rt, slot, twr);
            // Z[M - k] of k = rt + i P is register E-1-i of thread P - rt (a row's threads are
            // consecutive lanes of one warp), or register (E - i) mod E of thread 0 itself.
#pragma unroll
            for (int i = 0; i < RP::E; ++i) {
                const float2 mine = v[RP::E - 1 - i];
                float2 zmk;
                zmk.x = __shfl_sync(0xffffffffu, mine.x, partner);
                zmk.y = __shfl_sync(0xffffffffu, mine.y, partner);
                if (rt == 0) {
                    zmk = v[(RP::E - i) % RP::E];
                }
                const int k = rt + i * RP::P;
                if (act) {
                    sf[static_cast<long long>(r) * M + k] =
                        k == 0 ? make_float2(v[0].x + v[0].y, v[0].x - v[0].y)
                               : r2c_combine(v[i], zmk, __ldg(half + k));
                }
            }
        }
        __syncthreads();  // the field's row spectrum is in the scratch

        // Columns: N1-point transforms of the M scratch columns, CF at a time.
        float2* yf = y + f * (static_cast<long long>(N1) * (M + 1));
        for (int g = 0; g < M; g += K::CF) {
            const int col = g + cc;
            const bool act = col < M;
            float2 v[CP::E];
#pragma unroll
            for (int i = 0; i < CP::E; ++i) {
                v[i] = act ? sf[static_cast<long long>(ct + i * CP::P) * M + col] : make_float2(0.0f, 0.0f);
            }
            run_passes<CP, false, B, K::CF, true>(v, ct, work + cc, twc);
            if (act) {
                if (col == 0) {
#pragma unroll
                    for (int i = 0; i < CP::E; ++i) {
                        packed[ct + i * CP::P] = v[i];
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < CP::E; ++i) {
                        yf[static_cast<long long>(ct + i * CP::P) * (M + 1) + col] = v[i];
                    }
                }
            }
        }
        __syncthreads();  // the packed column is complete; every scratch read is done
        // Separate the DC and Nyquist columns: A = (Z[k1] + conj Z[-k1]) / 2,
        // B = (Z[k1] - conj Z[-k1]) / (2 i).
        for (int k1 = threadIdx.x; k1 < N1; k1 += blockDim.x) {
            const float2 z = packed[k1];
            const float2 zm = packed[(N1 - k1) & (N1 - 1)];
            float2* row = yf + static_cast<long long>(k1) * (M + 1);
            row[0] = make_float2(0.5f * (z.x + zm.x), 0.5f * (z.y - zm.y));
            row[M] = make_float2(0.5f * (z.y + zm.y), -0.5f * (z.x - zm.x));
        }
        if (discard) {
            discard_l2(sf, K::kScratch * 8);
        }
        __syncthreads();  // the packed column is read before the next field rewrites it
    }
}

template <int N1, int N2, int B>
__global__ void __launch_bounds__(256)
    fields_inverse(const float2* __restrict__ y, float2* __restrict__ x, float2* __restrict__ scratch,
                   long long fields, bool discard, const float2* __restrict__ twr,
                   const float2* __restrict__ half, const float2* __restrict__ twc)
{
    using K = Fields<N1, N2>;
    using RP = typename K::RP;
    using CP = typename K::CP;
    constexpr int M = K::M;
    extern __shared__ float4 smem_raw[];
    float2* work = reinterpret_cast<float2*>(smem_raw);

    const int rg = threadIdx.x / RP::P;
    const int rt = threadIdx.x - rg * RP::P;
    const int cc = threadIdx.x % K::CF;
    const int ct = threadIdx.x / K::CF;
    float2* slot = work + rg * RP::BUF;
    const float2 zero = make_float2(0.0f, 0.0f);
    constexpr float kColScale = 1.0f / N1;
    constexpr float kRowScale = 1.0f / M;

    for (long long f = blockIdx.x; f < fields; f += gridDim.x) {
        const float2* yf = y + f * (static_cast<long long>(N1) * (M + 1));
        float2* sf = scratch + f * K::kScratch;
        // Columns: inverse N1-point transforms of the spectrum's columns 1 .. M-1 and of the
        // packed DC / Nyquist column, into the scratch.
        for (int g = 0; g < M; g += K::CF) {
            const int col = g + cc;
            const bool act = col < M;
            float2 v[CP::E];
            if (act && col == 0) {
                // z = H0 + i HM, H the Hermitian parts of the DC and Nyquist spectrum columns.
#pragma unroll
                for (int i = 0; i < CP::E; ++i) {
                    const int k1 = ct + i * CP::P;
                    const long long a = static_cast<long long>(k1) * (M + 1);
                    const long long b = static_cast<long long>((N1 - k1) & (N1 - 1)) * (M + 1);
                    const float2 d = __ldg(yf + a);
                    const float2 dm = __ldg(yf + b);
                    const float2 q = __ldg(yf + a + M);
                    const float2 qm = __ldg(yf + b + M);
                    v[i] = make_float2(0.5f * (d.x + dm.x) - 0.5f * (q.y - qm.y),
                                       0.5f * (d.y - dm.y) + 0.5f * (q.x + qm.x));
                }
            } else {
#pragma unroll
                for (int i = 0; i < CP::E; ++i) {
                    v[i] = act ? __ldg(yf + static_cast<long long>(ct + i * CP::P) * (M + 1) + col) : zero;
                }
            }
            run_passes<CP, true, B, K::CF, true>(v, ct, work + cc, twc);
            if (act) {
#pragma unroll
                for (int i = 0; i < CP::E; ++i) {
                    sf[static_cast<long long>(ct + i * CP::P) * M + col] = cscale(v[i], kColScale);
                }
            }
        }
        __syncthreads();  // every column is in the scratch

        // Rows: X_r[k], k = 0 .. M, from the scratch (column 0 packs the real X[0] and X[M]),
        // prepared in mirror pairs, inverse M-point transforms, stored as 2 M reals.
        float2* xf = x + f * K::kScratch;
        for (int r0 = 0; r0 < N1; r0 += K::RG) {
            const int r = r0 + rg;
            const bool act = r < N1;
            const float2* srow = sf + static_cast<long long>(r) * M;
            float2 u[RP::E];
#pragma unroll
            for (int i = 0; i < RP::E; ++i) {
                const int k = rt + i * RP::P;
                float2 xk = zero;
                float2 xmk = zero;
                if (act) {
                    if (k == 0) {
                        const float2 p = srow[0];
                        xk = make_float2(p.x, 0.0f);
                        xmk = make_float2(p.y, 0.0f);
                    } else {
                        xk = srow[k];
                        xmk = srow[M - k];
                    }
                }
                u[i] = c2r_prepare(xk, xmk, __ldg(half + k));
            }
            run_passes<RP, true, B>(u, rt, slot, twr);
            if (act) {
#pragma unroll
                for (int i = 0; i < RP::E; ++i) {
                    xf[static_cast<long long>(r) * M + rt + i * RP::P] = cscale(u[i], kRowScale);
                }
            }
        }
        __syncthreads();  // every scratch read is done
        if (discard) {
            discard_l2(sf, K::kScratch * 8);
        }
    }
}

template <int B, bool Table>
struct FieldsEngine {
    static constexpr int kMinN1 = 16;
    static constexpr int kMaxN1 = 1024;
    static constexpr int kMinN2 = 16;
    static constexpr int kMaxN2 = 1024;
    static constexpr long long kMaxScratchBytes = 512 * 1024;  // per field: stays in L2

    static bool supported(int n1, int n2)
    {
        return is_pow2(n1) && is_pow2(n2) && n1 >= kMinN1 && n1 <= kMaxN1 && n2 >= kMinN2
               && n2 <= kMaxN2 && static_cast<long long>(n1) * (n2 / 2) * 8 <= kMaxScratchBytes;
    }

    // Scratch values (complex) for `fields` fields.
    static long long scratch(int n1, int n2, long long fields)
    {
        return static_cast<long long>(n1) * (n2 / 2) * fields;
    }

    template <bool Forward>
    static void run(const float2* in, float2* out, float2* scratch, int n1, int n2, long long fields,
                    cudaStream_t stream)
    {
        if (fields <= 0) {
            return;
        }
        dispatch_pow2<kMinN1, kMaxN1>(n1, [&](auto n1_) {
            dispatch_pow2<kMinN2, kMaxN2>(n2, [&](auto n2_) {
                constexpr int N1 = decltype(n1_)::value;
                constexpr int N2 = decltype(n2_)::value;
                if constexpr (static_cast<long long>(N1) * (N2 / 2) * 8 <= kMaxScratchBytes) {
                    using K = Fields<N1, N2>;
                    constexpr int M = K::M;
                    const float2* twr = Table ? twiddles::pass_table(M, K::RP::E)
                                              : twiddles::pass_table_computed(M, K::RP::E);
                    const float2* half = Table ? twiddles::half_turn(M) : twiddles::half_turn_computed(M);
                    const float2* twc = Table ? twiddles::pass_table(N1, K::CP::E)
                                              : twiddles::pass_table_computed(N1, K::CP::E);
                    auto kernel = Forward ? fields_forward<N1, N2, B> : fields_inverse<N1, N2, B>;
                    static std::atomic<int> cache[kMaxDevices];
                    const unsigned grid = persistent_grid(reinterpret_cast<const void*>(kernel),
                                                          K::THREADS, K::kSmem, cache, fields);
                    // The scratch lines are dropped from L2 after use when the scratch is 128-byte
                    // aligned (whole lines); otherwise they are left to be written back.
                    const bool discard = (reinterpret_cast<unsigned long long>(scratch) & 127u) == 0;
                    kernel<<<grid, K::THREADS, K::kSmem, stream>>>(in, out, scratch, fields, discard,
                                                                   twr, half, twc);
                    SPECTRAL_CUDA(cudaGetLastError());
                } else {
                    throw InvalidArgument("fused rfft2: field too large");
                }
            });
        });
    }
};

}  // namespace spectral::engine
