// The C ABI (include/spectral_b200.h): the registry of implementations, the argument checks, and
// the drivers that compose row, column, transpose and gather kernels into the 2D and pruned
// transforms. Exceptions never cross the ABI: every entry point catches them and returns a
// status code, keeping the message for spectral_last_error().
//
// The checks and their messages follow the reference's drivers (csrc/fft/fft2d.cu:59-87,
// csrc/fft/pruned.cu:265-304, csrc/fft/stockham.cuh:489-528, csrc/fft/real.cu:160-180), so a
// caller that matches on them keeps working.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "simple.cuh"

#include <climits>
#include <cstring>
#include <string>

namespace spectral {
namespace {

thread_local std::string g_last_error;

struct Impl {
    const char* name;
    const Backend* backend;
    int max_n;       // largest transform in one kernel (2D, pruned)
    int max_c2c_n;   // largest 1D complex transform
    int max_real_n;  // largest real transform
    bool real_needs_work;
    bool has_columns() const { return backend->columns != nullptr; }
    bool has_pruned() const { return backend->columns != nullptr; }
};

constexpr int kRowMaxN = 4096;
constexpr int kFourStepMaxN = kRowMaxN * kRowMaxN;

// The reference's registry (csrc/fft/registry.hpp:28-40): same names, order and limits.
const Impl kImpls[] = {
    {"naive", &kNaive, 1 << 30, 1 << 30, 1 << 30, true},
    {"stockham_r2", &kEngineR2, kRowMaxN, kFourStepMaxN, 2 * kRowMaxN, false},
    {"stockham_r4", &kEngineR4, kRowMaxN, kFourStepMaxN, 2 * kRowMaxN, false},
    {"stockham_r8", &kEngineR8, kRowMaxN, kFourStepMaxN, 2 * kRowMaxN, false},
    {"stockham_r8_table", &kEngineR8Table, kRowMaxN, kFourStepMaxN, 2 * kRowMaxN, false},
};
constexpr int kImplCount = static_cast<int>(sizeof(kImpls) / sizeof(kImpls[0]));

std::string impl_names()
{
    std::string names;
    for (const Impl& impl : kImpls) {
        names += names.empty() ? "" : ", ";
        names += impl.name;
    }
    return names;
}

const Impl& find(const char* name)
{
    if (name != nullptr) {
        for (const Impl& impl : kImpls) {
            if (std::strcmp(name, impl.name) == 0) {
                return impl;
            }
        }
    }
    throw InvalidArgument(std::string("unknown FFT implementation '") + (name ? name : "(null)")
                          + "' (available: " + impl_names() + ")");
}

template <class F>
int guarded(F&& f)
{
    try {
        f();
        return SPECTRAL_OK;
    } catch (const InvalidArgument& e) {
        g_last_error = e.what();
        return SPECTRAL_INVALID_ARGUMENT;
    } catch (const CudaError& e) {
        g_last_error = e.what();
        return SPECTRAL_CUDA_ERROR;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return SPECTRAL_INTERNAL_ERROR;
    } catch (...) {
        g_last_error = "unknown error";
        return SPECTRAL_INTERNAL_ERROR;
    }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

std::string str(long long v) { return std::to_string(v); }

bool overlap(const void* a, std::size_t a_bytes, const void* b, std::size_t b_bytes)
{
    const auto* p = static_cast<const char*>(a);
    const auto* q = static_cast<const char*>(b);
    return p < q + b_bytes && q < p + a_bytes;
}

void need(bool ok, const std::string& message)
{
    if (!ok) {
        throw InvalidArgument(message);
    }
}

std::size_t count3(long long a, long long b, long long c)
{
    return static_cast<std::size_t>(a) * static_cast<std::size_t>(b) * static_cast<std::size_t>(c);
}

// --- 1D complex --------------------------------------------------------------------------------

void check_c2c(const Impl& impl, const void* x, const void* y, int n, long long batch, int row_in,
               int row_out, const char* who)
{
    need(is_pow2(n) && n <= impl.max_c2c_n, std::string(who) + ": " + impl.name
                                                  + " needs n to be a power of two up to "
                                                  + str(impl.max_c2c_n) + ", got " + str(n));
    need(batch >= 1, std::string(who) + ": batch must be at least 1, got " + str(batch));
    need(!overlap(x, static_cast<std::size_t>(batch) * row_in * sizeof(float2), y,
                  static_cast<std::size_t>(batch) * row_out * sizeof(float2)),
         std::string(who) + ": x and y must not overlap (out-of-place only)");
}

// Any n, including 1 (a copy) and the four-step sizes; keep < n only for n <= max_n.
void c2c_any(const Impl& impl, const float2* x, float2* y, int n, long long batch, Direction d,
             int keep, cudaStream_t s)
{
    if (n == 1) {
        SPECTRAL_CUDA(cudaMemcpyAsync(y, x, static_cast<std::size_t>(batch) * sizeof(float2),
                                      cudaMemcpyDeviceToDevice, s));
        return;
    }
    impl.backend->c2c(x, y, n, batch, d, keep, s);
}

// Columns of any length, including 1.
void columns_any(const Impl& impl, const float2* x, float2* y, int n, int cols, long long slabs,
                 int m1_in, int m1_out, Direction d, cudaStream_t s)
{
    if (n == 1) {
        if (x != y) {
            SPECTRAL_CUDA(cudaMemcpyAsync(y, x, count3(slabs, cols, 1) * sizeof(float2),
                                          cudaMemcpyDeviceToDevice, s));
        }
        return;
    }
    impl.backend->columns(x, y, n, cols, slabs, m1_in, m1_out, d, s);
}

// --- real --------------------------------------------------------------------------------------

void check_real(const Impl& impl, const void* real_side, const void* complex_side, int n,
                long long batch, int complex_row, const char* who)
{
    need(is_pow2(n) && n >= 2 && n <= impl.max_real_n,
         std::string(who) + ": n must be a power of two from 2 to " + str(impl.max_real_n)
             + ", got " + str(n));
    need(batch >= 1, std::string(who) + ": batch must be at least 1, got " + str(batch));
    need(!overlap(real_side, static_cast<std::size_t>(batch) * n * sizeof(float), complex_side,
                  static_cast<std::size_t>(batch) * complex_row * sizeof(float2)),
         std::string(who) + ": input and output must not overlap");
}

std::size_t real_work(const Impl& impl, int n1, int n2, long long batch)
{
    return impl.real_needs_work ? count3(batch, n1, n2 / 2) : 0;
}

// Every array is read and written as 8-byte values (complex float2; real arrays two samples at
// a time), so every pointer must be 8-byte aligned; a misaligned one is refused before any
// launch.
void need_aligned(const void* p, const char* who)
{
    if ((reinterpret_cast<unsigned long long>(p) & 7u) != 0) {
        throw InvalidArgument(std::string(who) + ": arrays must be 8-byte aligned");
    }
}

void need_work(const void* work, std::size_t count, const char* who)
{
    need(count == 0 || work != nullptr, std::string(who) + ": this call needs a workspace of "
                                            + str(static_cast<long long>(count))
                                            + " complex values");
}

// --- 2D ----------------------------------------------------------------------------------------

enum class Columns { Transpose = SPECTRAL_COLUMNS_TRANSPOSE, Strided = SPECTRAL_COLUMNS_STRIDED };

Columns to_columns(int c)
{
    need(c == SPECTRAL_COLUMNS_TRANSPOSE || c == SPECTRAL_COLUMNS_STRIDED,
         "columns must be SPECTRAL_COLUMNS_TRANSPOSE or SPECTRAL_COLUMNS_STRIDED, got " + str(c));
    return static_cast<Columns>(c);
}

void check_2d(const Impl& impl, Columns columns, int n1, int n2, long long batch, bool real)
{
    const std::string name = impl.name;
    const int max_n2 = real ? impl.max_real_n : impl.max_n;
    need(is_pow2(n1) && n1 <= impl.max_n, "fft2: " + name + " needs n1 to be a power of two up to "
                                              + str(impl.max_n) + ", got " + str(n1));
    need(is_pow2(n2) && n2 <= max_n2 && (!real || n2 >= 2),
         "fft2: " + name + " needs n2 to be a power of two" + (real ? " from 2" : "") + " up to "
             + str(max_n2) + ", got " + str(n2));
    need(batch >= 1, "fft2: batch must be at least 1, got " + str(batch));
    need(batch * (n1 > n2 ? n1 : n2) <= INT_MAX, "fft2: too many transforms");
    need(columns == Columns::Transpose || impl.has_columns(),
         "fft2: " + name + " has no strided column kernel; use the transpose method");
}

std::size_t fft2_c2c_work(const Impl&, Columns columns, int n1, int n2, long long batch)
{
    return columns == Columns::Strided ? 0 : 2 * count3(batch, n1, n2);
}

std::size_t fft2_r2c_work(const Impl& impl, Columns columns, int n1, int n2, long long batch)
{
    const std::size_t half = columns == Columns::Strided ? 0 : 2 * count3(batch, n1, n2 / 2 + 1);
    return half + real_work(impl, n1, n2, batch);
}

std::size_t fft2_c2r_work(const Impl& impl, Columns columns, int n1, int n2, long long batch)
{
    const std::size_t q = count3(batch, n1, n2 / 2 + 1);
    return (columns == Columns::Strided ? q : 2 * q) + real_work(impl, n1, n2, batch);
}

void fft2_c2c(const Impl& impl, Columns columns, const float2* x, float2* y, int n1, int n2,
              long long batch, Direction d, float2* work, cudaStream_t s)
{
    if (columns == Columns::Strided) {
        c2c_any(impl, x, y, n2, batch * n1, d, n2, s);            // rows
        columns_any(impl, y, y, n1, n2, batch, 0, 0, d, s);       // columns, in place
        return;
    }
    float2* a = work;
    float2* b = work + count3(batch, n1, n2);
    c2c_any(impl, x, a, n2, batch * n1, d, n2, s);
    simple::transpose(a, b, n1, n2, batch, s);
    c2c_any(impl, b, a, n1, batch * n2, d, n1, s);
    simple::transpose(a, y, n2, n1, batch, s);
}

void fft2_r2c(const Impl& impl, Columns columns, const float* x, float2* y, int n1, int n2,
              long long batch, float2* work, cudaStream_t s)
{
    const int w = n2 / 2 + 1;
    if (columns == Columns::Strided) {
        impl.backend->r2c(x, y, n2, batch * n1, w, work, s);
        columns_any(impl, y, y, n1, w, batch, 0, 0, Direction::Forward, s);
        return;
    }
    float2* a = work;
    float2* b = work + count3(batch, n1, w);
    float2* rwork = work + 2 * count3(batch, n1, w);
    impl.backend->r2c(x, a, n2, batch * n1, w, rwork, s);
    simple::transpose(a, b, n1, w, batch, s);
    c2c_any(impl, b, a, n1, batch * w, Direction::Forward, n1, s);
    simple::transpose(a, y, w, n1, batch, s);
}

void fft2_c2r(const Impl& impl, Columns columns, const float2* x, float* y, int n1, int n2,
              long long batch, float2* work, cudaStream_t s)
{
    const int w = n2 / 2 + 1;
    const std::size_t q = count3(batch, n1, w);
    if (columns == Columns::Strided) {
        // Columns first, out of place (the input is not ours to overwrite), then rows.
        float2* a = work;
        columns_any(impl, x, a, n1, w, batch, 0, 0, Direction::Inverse, s);
        impl.backend->c2r(a, y, n2, batch * n1, w, work + q, s);
        return;
    }
    float2* a = work;
    float2* b = work + q;
    simple::transpose(x, a, n1, w, batch, s);
    c2c_any(impl, a, b, n1, batch * w, Direction::Inverse, n1, s);
    simple::transpose(b, a, w, n1, batch, s);
    impl.backend->c2r(a, y, n2, batch * n1, w, work + 2 * q, s);
}

// --- pruned ------------------------------------------------------------------------------------

void check_pruned_1d(const Impl& impl, int n, int keep, long long batch)
{
    need(is_pow2(n) && n <= impl.max_n, "fft_c2c_pruned: " + std::string(impl.name)
                                            + " needs n to be a power of two up to "
                                            + str(impl.max_n) + ", got " + str(n));
    need(keep >= 1 && keep <= n,
         "fft_c2c_pruned: keep must be in [1, " + str(n) + "], got " + str(keep));
    need(batch >= 1, "fft_c2c_pruned: batch must be at least 1");
}

void check_pruned_2d(const Impl& impl, int n1, int n2, int m1, int m2, long long batch)
{
    const std::string name = impl.name;
    need(is_pow2(n1) && n1 <= impl.max_n, "rfft2 modes: " + name
                                              + " needs n1 to be a power of two up to "
                                              + str(impl.max_n) + ", got " + str(n1));
    need(is_pow2(n2) && n2 >= 2 && n2 <= impl.max_real_n,
         "rfft2 modes: " + name + " needs n2 to be a power of two from 2 up to "
             + str(impl.max_real_n) + ", got " + str(n2));
    need(m1 >= 1 && 2 * m1 <= n1 && m2 >= 1 && m2 <= n2 / 2 + 1,
         "rfft2 modes: need 1 <= m1 <= n1/2 and 1 <= m2 <= n2/2 + 1, got m1 = " + str(m1)
             + ", m2 = " + str(m2) + " for " + str(n1) + " x " + str(n2));
    need(batch >= 1 && batch * (n1 > n2 ? n1 : n2) <= INT_MAX, "rfft2 modes: batch out of range");
}

std::size_t c2c_pruned_work(const Impl& impl, int n, int, long long batch)
{
    return impl.has_pruned() ? 0 : count3(batch, 1, n);
}

// Whether spectral_rfft2_modes / spectral_irfft2_modes take the tensor-core kernels
// (pruned_tc.cu) where they fit.
constexpr bool kAutoTensorModes = true;
constexpr bool kAutoTensorInverse = true;

bool fused_pruned(const Impl& impl, int n1, int n2, int m1, int m2)
{
    return impl.backend->pruned2d_supported != nullptr
           && impl.backend->pruned2d_supported(n1, n2, m1, m2);
}

std::size_t rfft2_modes_work(const Impl& impl, int n1, int n2, int m1, int m2, long long batch)
{
    if (fused_pruned(impl, n1, n2, m1, m2)) {
        return 0;
    }
    if (impl.has_pruned()) {
        return count3(batch, n1, m2);
    }
    return count3(batch, n1, n2 / 2 + 1) + fft2_r2c_work(impl, Columns::Transpose, n1, n2, batch);
}

std::size_t irfft2_modes_work(const Impl& impl, int n1, int n2, int m1, int m2, long long batch)
{
    if (fused_pruned(impl, n1, n2, m1, m2)) {
        return 0;
    }
    if (impl.has_pruned()) {
        return count3(batch, n1, m2);
    }
    return count3(batch, n1, n2 / 2 + 1) + fft2_c2r_work(impl, Columns::Transpose, n1, n2, batch);
}

}  // namespace

void set_last_error(const std::string& message) { g_last_error = message; }

int run_fft2_c2r_strided(const char* impl, const void* x, float* y, int n1, int n2,
                         long long batch, float2* work, std::size_t work_values, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "fft2_c2r");
        need_aligned(y, "fft2_c2r");
        need(i.has_columns(), std::string(impl) + " has no strided column kernel");
        check_2d(i, Columns::Strided, n1, n2, batch, true);
        const std::size_t needed = fft2_c2r_work(i, Columns::Strided, n1, n2, batch);
        need(needed <= work_values, "fft2_c2r: needs " + str(static_cast<long long>(needed))
                                        + " complex values of scratch, more than the "
                                        + str(static_cast<long long>(work_values)) + " available");
        fft2_c2r(i, Columns::Strided, static_cast<const float2*>(x), y, n1, n2, batch, work,
                 as_stream(stream));
    });
}

}  // namespace spectral

using namespace spectral;

extern "C" {

const char* spectral_last_error(void) { return g_last_error.c_str(); }

int spectral_impl_count(void) { return kImplCount; }

const char* spectral_impl_name(int index)
{
    return index >= 0 && index < kImplCount ? kImpls[index].name : nullptr;
}

int spectral_impl_find(const char* name)
{
    for (int i = 0; i < kImplCount; ++i) {
        if (name != nullptr && std::strcmp(name, kImpls[i].name) == 0) {
            return i;
        }
    }
    return -1;
}

int spectral_impl_limits(const char* impl, int* max_n, int* max_c2c_n, int* max_real_n,
                         int* has_columns, int* has_pruned, int* real_needs_work)
{
    return guarded([&] {
        const Impl& i = find(impl);
        if (max_n) *max_n = i.max_n;
        if (max_c2c_n) *max_c2c_n = i.max_c2c_n;
        if (max_real_n) *max_real_n = i.max_real_n;
        if (has_columns) *has_columns = i.has_columns() ? 1 : 0;
        if (has_pruned) *has_pruned = i.has_pruned() ? 1 : 0;
        if (real_needs_work) *real_needs_work = i.real_needs_work ? 1 : 0;
    });
}

int spectral_scale(const void* x, void* y, size_t count, float alpha, void* stream)
{
    return guarded([&] {
        simple::scale(static_cast<const float2*>(x), static_cast<float2*>(y), count, alpha,
                      as_stream(stream));
    });
}

int spectral_c2c(const char* impl, const void* x, void* y, int n, long long batch, int inverse,
                 void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "fft");
        need_aligned(y, "fft");
        check_c2c(i, x, y, n, batch, n, n, "fft");
        c2c_any(i, static_cast<const float2*>(x), static_cast<float2*>(y), n, batch,
                inverse ? Direction::Inverse : Direction::Forward, n, as_stream(stream));
    });
}

int spectral_real_workspace(const char* impl, int n, long long batch, size_t* count)
{
    return guarded([&] { *count = real_work(find(impl), 1, n, batch); });
}

int spectral_r2c(const char* impl, const float* x, void* y, int n, long long batch, void* work,
                 void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "r2c");
        need_aligned(y, "r2c");
        check_real(i, x, y, n, batch, n / 2 + 1, "r2c");
        need_work(work, real_work(i, 1, n, batch), "r2c");
        i.backend->r2c(x, static_cast<float2*>(y), n, batch, n / 2 + 1, static_cast<float2*>(work),
                       as_stream(stream));
    });
}

int spectral_c2r(const char* impl, const void* x, float* y, int n, long long batch, void* work,
                 void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "c2r");
        need_aligned(y, "c2r");
        check_real(i, y, x, n, batch, n / 2 + 1, "c2r");
        need_work(work, real_work(i, 1, n, batch), "c2r");
        i.backend->c2r(static_cast<const float2*>(x), y, n, batch, n / 2 + 1,
                       static_cast<float2*>(work), as_stream(stream));
    });
}

int spectral_columns(const char* impl, const void* x, void* y, int n, int cols, long long slabs,
                     int inverse, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "columns");
        need_aligned(y, "columns");
        need(i.has_columns(), std::string(i.name) + " has no strided column kernel");
        need(is_pow2(n) && n <= i.max_n, "columns: n must be a power of two from 1 to "
                                             + str(i.max_n) + ", got " + str(n));
        need(cols >= 1 && slabs >= 1, "columns: need cols >= 1 and slabs >= 1");
        columns_any(i, static_cast<const float2*>(x), static_cast<float2*>(y), n, cols, slabs, 0, 0,
                    inverse ? Direction::Inverse : Direction::Forward, as_stream(stream));
    });
}

int spectral_fft2_c2c_workspace(const char* impl, int columns, int n1, int n2, long long batch,
                                size_t* count)
{
    return guarded([&] { *count = fft2_c2c_work(find(impl), to_columns(columns), n1, n2, batch); });
}

int spectral_fft2_r2c_workspace(const char* impl, int columns, int n1, int n2, long long batch,
                                size_t* count)
{
    return guarded([&] { *count = fft2_r2c_work(find(impl), to_columns(columns), n1, n2, batch); });
}

int spectral_fft2_c2r_workspace(const char* impl, int columns, int n1, int n2, long long batch,
                                size_t* count)
{
    return guarded([&] { *count = fft2_c2r_work(find(impl), to_columns(columns), n1, n2, batch); });
}

int spectral_fft2_c2c(const char* impl, int columns, const void* x, void* y, int n1, int n2,
                      long long batch, int inverse, void* work, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "fft2_c2c");
        need_aligned(y, "fft2_c2c");
        const Columns c = to_columns(columns);
        check_2d(i, c, n1, n2, batch, false);
        need_work(work, fft2_c2c_work(i, c, n1, n2, batch), "fft2_c2c");
        fft2_c2c(i, c, static_cast<const float2*>(x), static_cast<float2*>(y), n1, n2, batch,
                 inverse ? Direction::Inverse : Direction::Forward, static_cast<float2*>(work),
                 as_stream(stream));
    });
}

int spectral_fft2_r2c(const char* impl, int columns, const float* x, void* y, int n1, int n2,
                      long long batch, void* work, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "fft2_r2c");
        need_aligned(y, "fft2_r2c");
        const Columns c = to_columns(columns);
        check_2d(i, c, n1, n2, batch, true);
        need_work(work, fft2_r2c_work(i, c, n1, n2, batch), "fft2_r2c");
        fft2_r2c(i, c, x, static_cast<float2*>(y), n1, n2, batch, static_cast<float2*>(work),
                 as_stream(stream));
    });
}

int spectral_fft2_c2r(const char* impl, int columns, const void* x, float* y, int n1, int n2,
                      long long batch, void* work, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "fft2_c2r");
        need_aligned(y, "fft2_c2r");
        const Columns c = to_columns(columns);
        check_2d(i, c, n1, n2, batch, true);
        need_work(work, fft2_c2r_work(i, c, n1, n2, batch), "fft2_c2r");
        fft2_c2r(i, c, static_cast<const float2*>(x), y, n1, n2, batch, static_cast<float2*>(work),
                 as_stream(stream));
    });
}

int spectral_c2c_pruned_workspace(const char* impl, int n, int keep, long long batch, size_t* count)
{
    return guarded([&] { *count = c2c_pruned_work(find(impl), n, keep, batch); });
}

int spectral_c2c_pruned(const char* impl, const void* x, void* y, int n, int keep, long long batch,
                        int inverse, void* work, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need_aligned(x, "fft_c2c_pruned");
        need_aligned(y, "fft_c2c_pruned");
        check_pruned_1d(i, n, keep, batch);
        const Direction d = inverse ? Direction::Inverse : Direction::Forward;
        const auto* xs = static_cast<const float2*>(x);
        auto* ys = static_cast<float2*>(y);
        auto* ws = static_cast<float2*>(work);
        const cudaStream_t s = as_stream(stream);
        need_work(work, c2c_pruned_work(i, n, keep, batch), "fft_c2c_pruned");
        if (i.has_pruned()) {
            if (n == 1) {
                c2c_any(i, xs, ys, 1, batch, d, 1, s);
            } else {
                i.backend->c2c(xs, ys, n, batch, d, keep, s);
            }
            return;
        }
        if (d == Direction::Forward) {
            c2c_any(i, xs, ws, n, batch, d, n, s);
            simple::gather_modes(ws, ys, 1, n, 0, keep, batch, s);
        } else {
            simple::scatter_modes(xs, ws, 1, n, 0, keep, batch, s);
            c2c_any(i, ws, ys, n, batch, d, n, s);
        }
    });
}

int spectral_rfft2_modes_workspace(const char* impl, int n1, int n2, int m1, int m2,
                                   long long batch, size_t* count)
{
    return guarded([&] { *count = rfft2_modes_work(find(impl), n1, n2, m1, m2, batch); });
}

int spectral_irfft2_modes_workspace(const char* impl, int n1, int n2, int m1, int m2,
                                    long long batch, size_t* count)
{
    return guarded([&] { *count = irfft2_modes_work(find(impl), n1, n2, m1, m2, batch); });
}

int spectral_rfft2_modes(const char* impl, const float* x, void* modes, int n1, int n2, int m1,
                         int m2, long long batch, void* work, void* stream)
{
    return spectral_rfft2_modes_method(impl, x, modes, n1, n2, m1, m2, batch, SPECTRAL_MODES_AUTO, work, stream);
}

int spectral_rfft2_modes_method(const char* impl, const float* x, void* modes, int n1, int n2, int m1,
                                int m2, long long batch, int method, void* work, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need(method >= SPECTRAL_MODES_AUTO && method <= SPECTRAL_MODES_TENSOR,
             "rfft2_modes: method must be SPECTRAL_MODES_AUTO, _FP32 or _TENSOR");
        need_aligned(x, "rfft2_modes");
        need_aligned(modes, "rfft2_modes");
        check_pruned_2d(i, n1, n2, m1, m2, batch);
        need_work(work, rfft2_modes_work(i, n1, n2, m1, m2, batch), "rfft2_modes");
        // The kernels read x through the read-only path (or TMA) while modes are written.
        need(!overlap(x, count3(batch, n1, n2) * sizeof(float), modes,
                      count3(batch, 2 * m1, m2) * sizeof(float2)),
             "rfft2_modes: x and modes must not overlap");
        auto* ms = static_cast<float2*>(modes);
        auto* ws = static_cast<float2*>(work);
        const cudaStream_t s = as_stream(stream);
        const bool fused = fused_pruned(i, n1, n2, m1, m2);
        const bool tensor_fits = fused && pruned_tc_fits(x, n1, n2, m1, m2, batch);
        need(method != SPECTRAL_MODES_TENSOR || tensor_fits,
             "rfft2_modes: the tensor-core method needs an engine implementation, n1 = n2 = 128, "
             "m2 <= 16 and a 16-byte aligned x");
        if (method == SPECTRAL_MODES_TENSOR || (method == SPECTRAL_MODES_AUTO && tensor_fits && kAutoTensorModes)) {
            pruned_tc_forward(x, ms, m1, m2, batch, s);
            return;
        }
        if (fused) {
            i.backend->rfft2_modes(x, ms, n1, n2, m1, m2, batch, s);
            return;
        }
        if (i.has_pruned()) {
            i.backend->r2c(x, ws, n2, batch * n1, m2, nullptr, s);                      // n1 x m2
            columns_any(i, ws, ms, n1, m2, batch, 0, m1, Direction::Forward, s);
            return;
        }
        float2* full = ws;
        float2* rest = ws + count3(batch, n1, n2 / 2 + 1);
        fft2_r2c(i, Columns::Transpose, x, full, n1, n2, batch, rest, s);
        simple::gather_modes(full, ms, n1, n2 / 2 + 1, m1, m2, batch, s);
    });
}

int spectral_irfft2_modes(const char* impl, const void* modes, float* y, int n1, int n2, int m1,
                          int m2, long long batch, void* work, void* stream)
{
    return spectral_irfft2_modes_method(impl, modes, y, n1, n2, m1, m2, batch, SPECTRAL_MODES_AUTO, work, stream);
}

int spectral_irfft2_modes_method(const char* impl, const void* modes, float* y, int n1, int n2, int m1,
                                 int m2, long long batch, int method, void* work, void* stream)
{
    return guarded([&] {
        const Impl& i = find(impl);
        need(method >= SPECTRAL_MODES_AUTO && method <= SPECTRAL_MODES_TENSOR,
             "irfft2_modes: method must be SPECTRAL_MODES_AUTO, _FP32 or _TENSOR");
        need_aligned(modes, "irfft2_modes");
        need_aligned(y, "irfft2_modes");
        check_pruned_2d(i, n1, n2, m1, m2, batch);
        need_work(work, irfft2_modes_work(i, n1, n2, m1, m2, batch), "irfft2_modes");
        need(!overlap(modes, count3(batch, 2 * m1, m2) * sizeof(float2), y,
                      count3(batch, n1, n2) * sizeof(float)),
             "irfft2_modes: modes and y must not overlap");
        const auto* ms = static_cast<const float2*>(modes);
        auto* ws = static_cast<float2*>(work);
        const cudaStream_t s = as_stream(stream);
        const bool fused = fused_pruned(i, n1, n2, m1, m2);
        const bool tensor_fits = fused && pruned_tc_fits(y, n1, n2, m1, m2, batch);
        need(method != SPECTRAL_MODES_TENSOR || tensor_fits,
             "irfft2_modes: the tensor-core method needs an engine implementation, n1 = n2 = 128, "
             "m2 <= 16 and a 16-byte aligned y");
        if (method == SPECTRAL_MODES_TENSOR || (method == SPECTRAL_MODES_AUTO && tensor_fits && kAutoTensorInverse)) {
            pruned_tc_inverse(ms, y, m1, m2, batch, s);
            return;
        }
        if (fused) {
            i.backend->irfft2_modes(ms, y, n1, n2, m1, m2, batch, s);
            return;
        }
        if (i.has_pruned()) {
            columns_any(i, ms, ws, n1, m2, batch, m1, 0, Direction::Inverse, s);
            i.backend->c2r(ws, y, n2, batch * n1, m2, nullptr, s);                      // m2.. zero
            return;
        }
        float2* full = ws;
        float2* rest = ws + count3(batch, n1, n2 / 2 + 1);
        simple::scatter_modes(ms, full, n1, n2 / 2 + 1, m1, m2, batch, s);
        fft2_c2r(i, Columns::Transpose, full, y, n1, n2, batch, rest, s);
    });
}

}  // extern "C"
