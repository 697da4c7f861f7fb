// spectral._C: the torch.ops.spectral operators, a thin shim over the C ABI
// (include/spectral_b200.h).
//
// The schemas, defaults, argument checks and messages are the reference's
// (csrc/torch/ops.cpp:47-475), so code and tests written against it keep working: the checks
// made here raise RuntimeError (TORCH_CHECK), the C ABI's SPECTRAL_INVALID_ARGUMENT is rethrown
// as std::invalid_argument (ValueError), as the reference's drivers do. Every operator is
// registered for the CUDA dispatch key only, so CPU tensors get the dispatcher's
// NotImplementedError. A binding checks, makes its input contiguous, allocates the output and
// any workspace with at::empty (torch's caching allocator, stream-ordered), and launches on the
// current stream under a device guard. Nothing here runs on the CPU.

#include <Python.h>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "../../include/spectral_b200.h"

#include <climits>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void check_status(int status)
{
    if (status == SPECTRAL_OK) {
        return;
    }
    const std::string message = spectral_last_error();
    if (status == SPECTRAL_INVALID_ARGUMENT) {
        throw std::invalid_argument(message);
    }
    TORCH_CHECK(false, message);
}

void* stream() { return static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

const void* cptr(const at::Tensor& t) { return t.const_data_ptr(); }
void* mptr(at::Tensor& t) { return t.numel() == 0 ? nullptr : t.mutable_data_ptr(); }

void check_complex64_cuda(const at::Tensor& t, const char* name)
{
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == at::kComplexFloat, name, " must be complex64, got ",
                t.scalar_type());
}

void check_float32_cuda(const at::Tensor& t)
{
    TORCH_CHECK(t.is_cuda(), "x must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == at::kFloat, "x must be float32, got ", t.scalar_type());
}

struct ImplInfo {
    std::string name;
    int max_n;
    int max_c2c_n;
    int max_real_n;
    bool has_columns;
};

std::string impl_names()
{
    std::string names;
    for (int i = 0; i < spectral_impl_count(); ++i) {
        names += names.empty() ? "" : ", ";
        names += spectral_impl_name(i);
    }
    return names;
}

ImplInfo find_impl(c10::string_view impl_name)
{
    const std::string name(impl_name.data(), impl_name.size());
    TORCH_CHECK(spectral_impl_find(name.c_str()) >= 0, "unknown FFT implementation '", name,
                "' (available: ", impl_names(), ")");
    ImplInfo info{name, 0, 0, 0, false};
    int has_columns = 0;
    check_status(spectral_impl_limits(name.c_str(), &info.max_n, &info.max_c2c_n,
                                      &info.max_real_n, &has_columns, nullptr, nullptr));
    info.has_columns = has_columns != 0;
    return info;
}

int batch_of(const at::Tensor& x, int64_t row, const char* op)
{
    const int64_t batch = x.numel() / row;
    TORCH_CHECK(batch <= INT_MAX, op, ": too many transforms");
    return static_cast<int>(batch);
}

// The library reads and writes every array as 8-byte values; a contiguous float32 view can start
// at an odd element, so such an input is copied to a fresh (aligned) allocation first.
at::Tensor contiguous_aligned(const at::Tensor& x)
{
    at::Tensor c = x.contiguous();
    if ((reinterpret_cast<uintptr_t>(c.const_data_ptr()) & 7u) != 0) {
        c = c.clone(at::MemoryFormat::Contiguous);
    }
    return c;
}

at::Tensor workspace(size_t count, const at::Tensor& like)
{
    return at::empty({static_cast<int64_t>(count)}, like.options().dtype(at::kComplexFloat));
}

void check_real_size(int64_t n, const ImplInfo& impl, const char* op)
{
    TORCH_CHECK(n >= 2 && (n & (n - 1)) == 0, op,
                ": the real transform size must be a power of two of at least 2, got ", n);
    TORCH_CHECK(n <= impl.max_real_n, op, ": ", impl.name, " supports real sizes up to ",
                impl.max_real_n, ", got ", n);
}

at::Tensor scale_cuda(const at::Tensor& x, double alpha)
{
    check_complex64_cuda(x, "x");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    at::Tensor y = at::empty_like(xc);
    check_status(spectral_scale(cptr(xc), mptr(y), static_cast<size_t>(xc.numel()),
                                static_cast<float>(alpha), stream()));
    return y;
}

at::Tensor fft_c2c_cuda(const at::Tensor& x, bool inverse, c10::string_view impl_name)
{
    check_complex64_cuda(x, "x");
    TORCH_CHECK(x.dim() >= 1, "fft_c2c: x needs at least one dimension");
    const ImplInfo impl = find_impl(impl_name);
    if (x.numel() == 0) {
        return at::empty_like(x, at::MemoryFormat::Contiguous);
    }
    const int64_t n = x.size(-1);
    TORCH_CHECK((n & (n - 1)) == 0, "fft_c2c: the last dimension must be a power of two, got ", n);
    TORCH_CHECK(n <= impl.max_c2c_n, "fft_c2c: ", impl.name, " supports sizes up to ",
                impl.max_c2c_n, ", got ", n);
    const int batch = batch_of(x, n, "fft_c2c");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    at::Tensor y = at::empty_like(xc);
    check_status(spectral_c2c(impl.name.c_str(), cptr(xc), mptr(y), static_cast<int>(n), batch,
                              inverse ? 1 : 0, stream()));
    return y;
}

at::Tensor fft_r2c_cuda(const at::Tensor& x, c10::string_view impl_name)
{
    check_float32_cuda(x);
    TORCH_CHECK(x.dim() >= 1, "fft_r2c: x needs at least one dimension");
    const ImplInfo impl = find_impl(impl_name);
    const int64_t n = x.size(-1);
    check_real_size(n, impl, "fft_r2c");
    std::vector<int64_t> shape = x.sizes().vec();
    shape.back() = n / 2 + 1;
    at::Tensor y = at::empty(shape, x.options().dtype(at::kComplexFloat));
    if (x.numel() == 0) {
        return y;
    }
    const int batch = batch_of(x, n, "fft_r2c");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    size_t count = 0;
    check_status(spectral_real_workspace(impl.name.c_str(), static_cast<int>(n), batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_r2c(impl.name.c_str(), xc.const_data_ptr<float>(), mptr(y),
                              static_cast<int>(n), batch, mptr(work), stream()));
    return y;
}

at::Tensor fft_c2r_cuda(const at::Tensor& x, int64_t n, c10::string_view impl_name)
{
    check_complex64_cuda(x, "x");
    TORCH_CHECK(x.dim() >= 1, "fft_c2r: x needs at least one dimension");
    const ImplInfo impl = find_impl(impl_name);
    check_real_size(n, impl, "fft_c2r");
    TORCH_CHECK(x.size(-1) == n / 2 + 1, "fft_c2r: an output of ", n, " points needs n/2 + 1 = ",
                n / 2 + 1, " inputs per transform, got ", x.size(-1));
    std::vector<int64_t> shape = x.sizes().vec();
    shape.back() = n;
    at::Tensor y = at::empty(shape, x.options().dtype(at::kFloat));
    if (x.numel() == 0) {
        return y;
    }
    const int batch = batch_of(x, n / 2 + 1, "fft_c2r");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    size_t count = 0;
    check_status(spectral_real_workspace(impl.name.c_str(), static_cast<int>(n), batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_c2r(impl.name.c_str(), cptr(xc), y.mutable_data_ptr<float>(),
                              static_cast<int>(n), batch, mptr(work), stream()));
    return y;
}

// "auto" picks the strided column kernel when the implementation has one (ops.cpp:187-202).
int parse_columns(c10::string_view text, const ImplInfo& impl)
{
    const std::string s(text.data(), text.size());
    if (s == "auto") {
        return impl.has_columns ? SPECTRAL_COLUMNS_STRIDED : SPECTRAL_COLUMNS_TRANSPOSE;
    }
    if (s == "strided") {
        TORCH_CHECK(impl.has_columns, impl.name,
                    " has no strided column kernel; use columns=\"transpose\"");
        return SPECTRAL_COLUMNS_STRIDED;
    }
    TORCH_CHECK(s == "transpose", "columns must be \"auto\", \"strided\", or \"transpose\", got '",
                s, "'");
    return SPECTRAL_COLUMNS_TRANSPOSE;
}

struct Shape2d {
    int64_t n1;
    int64_t n2;
    int batch;
};

Shape2d shape2d(const at::Tensor& x, int64_t n2, int64_t n2_stored, const char* op)
{
    TORCH_CHECK(x.dim() >= 2, op, ": x needs at least two dimensions");
    const int64_t n1 = x.size(-2);
    TORCH_CHECK(n1 >= 1 && n2 >= 1, op, ": empty transform dimensions");
    return {n1, n2, batch_of(x, n1 * n2_stored, op)};
}

at::Tensor fft2_c2c_cuda(const at::Tensor& x, bool inverse, c10::string_view impl_name,
                         c10::string_view columns)
{
    check_complex64_cuda(x, "x");
    const ImplInfo impl = find_impl(impl_name);
    const int method = parse_columns(columns, impl);
    TORCH_CHECK(x.dim() >= 2, "fft2_c2c: x needs at least two dimensions");
    if (x.numel() == 0) {
        return at::empty_like(x, at::MemoryFormat::Contiguous);
    }
    const Shape2d s = shape2d(x, x.size(-1), x.size(-1), "fft2_c2c");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    at::Tensor y = at::empty_like(xc);
    const auto n1 = static_cast<int>(s.n1);
    const auto n2 = static_cast<int>(s.n2);
    size_t count = 0;
    check_status(spectral_fft2_c2c_workspace(impl.name.c_str(), method, n1, n2, s.batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_fft2_c2c(impl.name.c_str(), method, cptr(xc), mptr(y), n1, n2, s.batch,
                                   inverse ? 1 : 0, mptr(work), stream()));
    return y;
}

at::Tensor fft2_r2c_cuda(const at::Tensor& x, c10::string_view impl_name, c10::string_view columns)
{
    check_float32_cuda(x);
    const ImplInfo impl = find_impl(impl_name);
    const int method = parse_columns(columns, impl);
    TORCH_CHECK(x.dim() >= 2, "fft2_r2c: x needs at least two dimensions");
    const int64_t n2 = x.size(-1);
    check_real_size(n2, impl, "fft2_r2c");
    std::vector<int64_t> shape = x.sizes().vec();
    shape.back() = n2 / 2 + 1;
    at::Tensor y = at::empty(shape, x.options().dtype(at::kComplexFloat));
    if (x.numel() == 0) {
        return y;
    }
    const Shape2d s = shape2d(x, n2, n2, "fft2_r2c");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    const auto n1 = static_cast<int>(s.n1);
    size_t count = 0;
    check_status(spectral_fft2_r2c_workspace(impl.name.c_str(), method, n1, static_cast<int>(n2),
                                             s.batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_fft2_r2c(impl.name.c_str(), method, xc.const_data_ptr<float>(), mptr(y),
                                   n1, static_cast<int>(n2), s.batch, mptr(work), stream()));
    return y;
}

at::Tensor fft2_c2r_cuda(const at::Tensor& x, int64_t n2, c10::string_view impl_name,
                         c10::string_view columns)
{
    check_complex64_cuda(x, "x");
    const ImplInfo impl = find_impl(impl_name);
    const int method = parse_columns(columns, impl);
    TORCH_CHECK(x.dim() >= 2, "fft2_c2r: x needs at least two dimensions");
    check_real_size(n2, impl, "fft2_c2r");
    TORCH_CHECK(x.size(-1) == n2 / 2 + 1, "fft2_c2r: an output of ", n2,
                " columns needs n2/2 + 1 = ", n2 / 2 + 1, " input columns, got ", x.size(-1));
    std::vector<int64_t> shape = x.sizes().vec();
    shape.back() = n2;
    at::Tensor y = at::empty(shape, x.options().dtype(at::kFloat));
    if (x.numel() == 0) {
        return y;
    }
    const Shape2d s = shape2d(x, n2, n2 / 2 + 1, "fft2_c2r");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    const auto n1 = static_cast<int>(s.n1);
    size_t count = 0;
    check_status(spectral_fft2_c2r_workspace(impl.name.c_str(), method, n1, static_cast<int>(n2),
                                             s.batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_fft2_c2r(impl.name.c_str(), method, cptr(xc), y.mutable_data_ptr<float>(),
                                   n1, static_cast<int>(n2), s.batch, mptr(work), stream()));
    return y;
}

at::Tensor fft_c2c_pruned_cuda(const at::Tensor& x, int64_t n, int64_t keep, bool inverse,
                               c10::string_view impl_name)
{
    check_complex64_cuda(x, "x");
    TORCH_CHECK(x.dim() >= 1, "fft_c2c_pruned: x needs at least one dimension");
    const ImplInfo impl = find_impl(impl_name);
    TORCH_CHECK(n >= 1 && n <= INT_MAX && keep >= 1 && keep <= n,
                "fft_c2c_pruned: need 1 <= keep <= n, got keep = ", keep, ", n = ", n);
    const int64_t row_in = inverse ? keep : n;
    TORCH_CHECK(x.size(-1) == row_in, "fft_c2c_pruned: expected ", row_in,
                " values in the last dimension, got ", x.size(-1));
    std::vector<int64_t> shape = x.sizes().vec();
    shape.back() = inverse ? n : keep;
    at::Tensor y = at::empty(shape, x.options());
    if (x.numel() == 0) {
        return y;
    }
    const int batch = batch_of(x, row_in, "fft_c2c_pruned");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    size_t count = 0;
    check_status(spectral_c2c_pruned_workspace(impl.name.c_str(), static_cast<int>(n),
                                               static_cast<int>(keep), batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_c2c_pruned(impl.name.c_str(), cptr(xc), mptr(y), static_cast<int>(n),
                                     static_cast<int>(keep), batch, inverse ? 1 : 0, mptr(work),
                                     stream()));
    return y;
}

at::Tensor rfft2_modes_cuda(const at::Tensor& x, int64_t m1, int64_t m2, c10::string_view impl_name)
{
    check_float32_cuda(x);
    TORCH_CHECK(x.dim() >= 2, "rfft2_modes: x needs at least two dimensions");
    const ImplInfo impl = find_impl(impl_name);
    const int64_t n1 = x.size(-2);
    const int64_t n2 = x.size(-1);
    TORCH_CHECK(m1 >= 1 && 2 * m1 <= n1 && m2 >= 1 && m2 <= n2 / 2 + 1,
                "rfft2_modes: need 1 <= m1 <= n1/2 and 1 <= m2 <= n2/2 + 1, got m1 = ", m1,
                ", m2 = ", m2, " for ", n1, " x ", n2);
    std::vector<int64_t> shape = x.sizes().vec();
    shape[shape.size() - 2] = 2 * m1;
    shape.back() = m2;
    at::Tensor y = at::empty(shape, x.options().dtype(at::kComplexFloat));
    if (x.numel() == 0) {
        return y;
    }
    const int batch = batch_of(x, n1 * n2, "rfft2_modes");
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    const int a = static_cast<int>(n1);
    const int b = static_cast<int>(n2);
    const int p = static_cast<int>(m1);
    const int q = static_cast<int>(m2);
    size_t count = 0;
    check_status(spectral_rfft2_modes_workspace(impl.name.c_str(), a, b, p, q, batch, &count));
    at::Tensor work = workspace(count, x);
    check_status(spectral_rfft2_modes(impl.name.c_str(), xc.const_data_ptr<float>(), mptr(y), a, b,
                                      p, q, batch, mptr(work), stream()));
    return y;
}

at::Tensor irfft2_modes_cuda(const at::Tensor& modes, int64_t n1, int64_t n2,
                             c10::string_view impl_name)
{
    check_complex64_cuda(modes, "modes");
    TORCH_CHECK(modes.dim() >= 2, "irfft2_modes: modes needs at least two dimensions");
    const ImplInfo impl = find_impl(impl_name);
    const int64_t two_m1 = modes.size(-2);
    const int64_t m2 = modes.size(-1);
    TORCH_CHECK(two_m1 % 2 == 0 && two_m1 >= 2 && two_m1 <= n1 && m2 >= 1 && m2 <= n2 / 2 + 1,
                "irfft2_modes: modes of shape (", two_m1, ", ", m2, ") do not fit an output of ", n1,
                " x ", n2);
    std::vector<int64_t> shape = modes.sizes().vec();
    shape[shape.size() - 2] = n1;
    shape.back() = n2;
    at::Tensor y = at::empty(shape, modes.options().dtype(at::kFloat));
    if (modes.numel() == 0) {
        return y;
    }
    const int batch = batch_of(modes, two_m1 * m2, "irfft2_modes");
    const c10::cuda::CUDAGuard guard(modes.device());
    const at::Tensor mc = contiguous_aligned(modes);
    const int a = static_cast<int>(n1);
    const int b = static_cast<int>(n2);
    const int p = static_cast<int>(two_m1 / 2);
    const int q = static_cast<int>(m2);
    size_t count = 0;
    check_status(spectral_irfft2_modes_workspace(impl.name.c_str(), a, b, p, q, batch, &count));
    at::Tensor work = workspace(count, modes);
    check_status(spectral_irfft2_modes(impl.name.c_str(), cptr(mc), y.mutable_data_ptr<float>(), a,
                                       b, p, q, batch, mptr(work), stream()));
    return y;
}

// x (..., cin, modes...) complex64, w (cin, cout, modes...) complex64 -> (..., cout, modes...):
// the per-mode contraction of an FNO spectral convolution. Not one of the reference's operators
// (it has no implementation of it); an addition of this library.
at::Tensor mode_contract_cuda(const at::Tensor& x, const at::Tensor& w)
{
    check_complex64_cuda(x, "x");
    check_complex64_cuda(w, "w");
    TORCH_CHECK(x.dim() >= 2 && w.dim() == x.dim(),
                "mode_contract: x (batch..., cin, modes...) and w (cin, cout, modes...) need the "
                "same number of mode dimensions");
    const int64_t mode_dims = w.dim() - 2;
    const int64_t lead = x.dim() - mode_dims - 1;  // batch dimensions of x
    TORCH_CHECK(lead == 1, "mode_contract: x must be (batch, cin, modes...)");
    TORCH_CHECK(x.size(1) == w.size(0), "mode_contract: x has ", x.size(1), " channels, w expects ",
                w.size(0));
    for (int64_t d = 0; d < mode_dims; ++d) {
        TORCH_CHECK(x.size(2 + d) == w.size(2 + d), "mode_contract: mode shapes differ");
    }
    std::vector<int64_t> shape = x.sizes().vec();
    shape[1] = w.size(1);
    at::Tensor y = at::empty(shape, x.options());
    if (y.numel() == 0) {
        return y;
    }
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    const at::Tensor wc = contiguous_aligned(w);
    const int64_t modes = x.numel() / (x.size(0) * x.size(1));
    check_status(spectral_mode_contract(cptr(xc), cptr(wc), mptr(y), x.size(0),
                                        static_cast<int>(x.size(1)), static_cast<int>(w.size(1)),
                                        modes, stream()));
    return y;
}

// The fused radio-signal kernels behind spectral.rf: x is (..., n) complex64, each leading index
// one signal. The Python layer picks these for the stockham implementations and nfft <= 4096.
at::Tensor spectrum_frames_cuda(const at::Tensor& x, int64_t nfft, const c10::optional<at::Tensor>& window,
                                c10::string_view impl_name)
{
    check_complex64_cuda(x, "x");
    TORCH_CHECK(x.dim() >= 1, "spectrum: x needs at least one dimension");
    const std::string impl(impl_name.data(), impl_name.size());
    const int64_t n = x.size(-1);
    int64_t rows = 1;  // the product of the leading dimensions (x may be empty)
    for (int64_t d = 0; d + 1 < x.dim(); ++d) {
        rows *= x.size(d);
    }
    TORCH_CHECK(nfft >= 2 && nfft <= 4096 && (nfft & (nfft - 1)) == 0,
                "spectrum: nfft must be a power of two from 2 to 4096, got ", nfft);
    const int64_t frames = n == 0 ? 1 : (n + nfft - 1) / nfft;
    std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end() - 1);
    shape.push_back(frames);
    shape.push_back(nfft);
    at::Tensor y = at::empty(shape, x.options());
    at::Tensor wc;
    if (window.has_value()) {
        TORCH_CHECK(window->is_cuda() && window->scalar_type() == at::kFloat && window->dim() == 1
                        && window->size(0) == nfft,
                    "spectrum: the window must be a float32 CUDA tensor of nfft = ", nfft, " values");
        wc = window->contiguous();
    }
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    check_status(spectral_spectrum(impl.c_str(), n == 0 ? nullptr : cptr(xc),
                                   window.has_value() ? wc.const_data_ptr<float>() : nullptr, mptr(y), n,
                                   static_cast<int>(nfft), rows, stream()));
    return y;
}

at::Tensor fir_overlap_save_cuda(const at::Tensor& x, const at::Tensor& taps_spectrum, int64_t taps,
                                 int64_t nfft, c10::string_view impl_name)
{
    check_complex64_cuda(x, "x");
    check_complex64_cuda(taps_spectrum, "taps_spectrum");
    TORCH_CHECK(x.dim() >= 1, "fir: x needs at least one dimension");
    TORCH_CHECK(taps_spectrum.dim() == 1 && taps_spectrum.size(0) == nfft,
                "fir: taps_spectrum must hold nfft = ", nfft, " values");
    TORCH_CHECK(taps >= 1 && taps <= nfft, "fir: need 1 <= taps <= nfft");
    const std::string impl(impl_name.data(), impl_name.size());
    at::Tensor y = at::empty(x.sizes(), x.options());
    const int64_t n = x.size(-1);
    const int64_t rows = n == 0 ? 0 : x.numel() / n;
    const c10::cuda::CUDAGuard guard(x.device());
    const at::Tensor xc = contiguous_aligned(x);
    const at::Tensor hc = contiguous_aligned(taps_spectrum);
    check_status(spectral_fir(impl.c_str(), n == 0 ? nullptr : cptr(xc), cptr(hc),
                              n == 0 ? nullptr : mptr(y), n, static_cast<int>(nfft),
                              static_cast<int>(taps), rows, stream()));
    return y;
}

// One stage of the Navier-Stokes step (spectral.flow.gpu): writes f0 (predictor) and out.
void flow_stage_cuda(const at::Tensor& x, const at::Tensor& w, at::Tensor& f0, at::Tensor& out,
                     const at::Tensor& derive, const at::Tensor& forcing, const at::Tensor& mask,
                     const at::Tensor& explicit_factor, const at::Tensor& implicit_factor, at::Tensor& work,
                     int64_t n, int64_t m, double dt, int64_t stage, c10::string_view impl_name)
{
    for (const at::Tensor* t : {&x, &w, const_cast<const at::Tensor*>(&f0), const_cast<const at::Tensor*>(&out),
                                &derive, &forcing, const_cast<const at::Tensor*>(&work)}) {
        check_complex64_cuda(*t, "flow_stage arrays");
        TORCH_CHECK(t->is_contiguous(), "flow_stage: arrays must be contiguous");
    }
    for (const at::Tensor* t : {&mask, &explicit_factor, &implicit_factor}) {
        TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous(),
                    "flow_stage: mask and factors must be contiguous float32 CUDA tensors");
    }
    const int64_t plane = 2 * m * m;
    TORCH_CHECK(x.numel() % plane == 0 && w.numel() == x.numel() && f0.numel() == x.numel() && out.numel() == x.numel(),
                "flow_stage: states must be (batch, 2m, m)");
    TORCH_CHECK(derive.numel() == 4 * plane && forcing.numel() == plane && mask.numel() == plane,
                "flow_stage: derive (4, 2m, m), forcing and mask (2m, m)");
    const int64_t batch = x.numel() / plane;
    const int64_t vs = explicit_factor.numel() == plane ? 0 : plane;
    TORCH_CHECK(explicit_factor.numel() == implicit_factor.numel()
                    && (vs == 0 || explicit_factor.numel() == batch * plane),
                "flow_stage: the factors must be (2m, m) or (batch, 2m, m)");
    size_t count = 0;
    check_status(spectral_flow_workspace(static_cast<int>(n), static_cast<int>(m), batch, &count));
    TORCH_CHECK(static_cast<size_t>(work.numel()) >= count, "flow_stage: work needs ", count, " values");
    const std::string impl(impl_name.data(), impl_name.size());
    const c10::cuda::CUDAGuard guard(x.device());
    check_status(spectral_flow_stage(impl.c_str(), cptr(x), cptr(w), mptr(f0), mptr(out), cptr(derive), cptr(forcing),
                                     mask.const_data_ptr<float>(), explicit_factor.const_data_ptr<float>(),
                                     implicit_factor.const_data_ptr<float>(), vs, mptr(work), static_cast<int>(n),
                                     static_cast<int>(m), batch, static_cast<float>(dt), static_cast<int>(stage),
                                     stream()));
}

// spectral._C.fft_impls(): the registry's names, in order, as a tuple of str.
PyObject* py_fft_impls(PyObject*, PyObject*)
{
    const int count = spectral_impl_count();
    PyObject* names = PyTuple_New(count);
    if (names == nullptr) {
        return nullptr;
    }
    for (int i = 0; i < count; ++i) {
        PyObject* name = PyUnicode_FromString(spectral_impl_name(i));
        if (name == nullptr) {
            Py_DECREF(names);
            return nullptr;
        }
        PyTuple_SET_ITEM(names, i, name);
    }
    return names;
}

PyMethodDef module_methods[] = {
    {"fft_impls", py_fft_impls, METH_NOARGS, "Names of the FFT implementations, in order."},
    {nullptr, nullptr, 0, nullptr},
};

}  // namespace

TORCH_LIBRARY(spectral, m)
{
    m.def("scale(Tensor x, float alpha) -> Tensor");
    m.def("fft_c2c(Tensor x, bool inverse=False, str impl=\"naive\") -> Tensor");
    m.def("fft_r2c(Tensor x, str impl=\"naive\") -> Tensor");
    m.def("fft_c2r(Tensor x, int n, str impl=\"naive\") -> Tensor");
    m.def("fft2_c2c(Tensor x, bool inverse=False, str impl=\"naive\", str columns=\"auto\")"
          " -> Tensor");
    m.def("fft2_r2c(Tensor x, str impl=\"naive\", str columns=\"auto\") -> Tensor");
    m.def("fft2_c2r(Tensor x, int n2, str impl=\"naive\", str columns=\"auto\") -> Tensor");
    m.def("fft_c2c_pruned(Tensor x, int n, int keep, bool inverse=False, str impl=\"naive\")"
          " -> Tensor");
    m.def("rfft2_modes(Tensor x, int m1, int m2, str impl=\"naive\") -> Tensor");
    m.def("irfft2_modes(Tensor modes, int n1, int n2, str impl=\"naive\") -> Tensor");
    m.def("mode_contract(Tensor x, Tensor w) -> Tensor");
    m.def("spectrum_frames(Tensor x, int nfft, Tensor? window=None, str impl=\"stockham_r8\") -> Tensor");
    m.def("fir_overlap_save(Tensor x, Tensor taps_spectrum, int taps, int nfft, str impl=\"stockham_r8\")"
          " -> Tensor");
    m.def("flow_stage(Tensor x, Tensor w, Tensor(a!) f0, Tensor(b!) out, Tensor derive, Tensor forcing, Tensor mask,"
          " Tensor explicit_factor, Tensor implicit_factor, Tensor(c!) work, int n, int m, float dt, int stage,"
          " str impl=\"stockham_r8\") -> ()");
}

TORCH_LIBRARY_IMPL(spectral, CUDA, m)
{
    m.impl("scale", &scale_cuda);
    m.impl("fft_c2c", &fft_c2c_cuda);
    m.impl("fft_r2c", &fft_r2c_cuda);
    m.impl("fft_c2r", &fft_c2r_cuda);
    m.impl("fft2_c2c", &fft2_c2c_cuda);
    m.impl("fft2_r2c", &fft2_r2c_cuda);
    m.impl("fft2_c2r", &fft2_c2r_cuda);
    m.impl("fft_c2c_pruned", &fft_c2c_pruned_cuda);
    m.impl("rfft2_modes", &rfft2_modes_cuda);
    m.impl("irfft2_modes", &irfft2_modes_cuda);
    m.impl("mode_contract", &mode_contract_cuda);
    m.impl("spectrum_frames", &spectrum_frames_cuda);
    m.impl("fir_overlap_save", &fir_overlap_save_cuda);
    m.impl("flow_stage", &flow_stage_cuda);
}

PyMODINIT_FUNC PyInit__C(void)
{
    static PyModuleDef module_def = {
        PyModuleDef_HEAD_INIT, "_C", nullptr, -1, module_methods,
    };
    return PyModule_Create(&module_def);
}
