// Correctly rounded twiddle tables (see twiddles.cuh).

#include "twiddles.cuh"

#include "dft.cuh"
#include "engine.cuh"

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace spectral::twiddles {
namespace {

// 4 MiB of tables per device, far more than every plan of this library needs together.
constexpr long long kPoolEntries = 1 << 19;
__device__ float2 g_pool[kPoolEntries];

using Key = std::tuple<int, long long, long long>;  // (kind, a, b)

struct DeviceTables {
    float2* base = nullptr;
    long long used = 0;
    std::map<Key, const float2*> tables;
};

std::mutex g_mutex;
std::map<int, DeviceTables> g_devices;

float2 forward_factor(long long j, long long m)
{
    const dft::CosSin w = dft::cs2pi(j, m);  // exact octant reduction, then a double series
    return make_float2(static_cast<float>(w.c), static_cast<float>(-w.s));
}

// Reserves `count` entries of the pool for `key` (16-byte aligned) and fills them with
// fill(device pointer, offset in the pool); returns the cached table when `key` was built before
// on this device.
template <class Fill>
const float2* get_filled(const Key& key, long long count, Fill&& fill)
{
    int device = 0;
    SPECTRAL_CUDA(cudaGetDevice(&device));
    const std::lock_guard<std::mutex> lock(g_mutex);
    DeviceTables& dt = g_devices[device];
    auto it = dt.tables.find(key);
    if (it != dt.tables.end()) {
        return it->second;
    }
    if (dt.base == nullptr) {
        void* p = nullptr;
        SPECTRAL_CUDA(cudaGetSymbolAddress(&p, g_pool));
        dt.base = static_cast<float2*>(p);
    }
    const long long aligned = (dt.used + 1) & ~1LL;
    if (aligned + count > kPoolEntries) {
        throw InvalidArgument("twiddle tables: pool exhausted");
    }
    float2* ptr = dt.base + aligned;
    fill(ptr, aligned);
    dt.used = aligned + count;
    dt.tables.emplace(key, ptr);
    return ptr;
}

template <class Build>
const float2* get(const Key& key, long long count, Build&& build)
{
    return get_filled(key, count, [&](float2*, long long offset) {
        std::vector<float2> host(static_cast<std::size_t>(count));
        build(host);
        SPECTRAL_CUDA(cudaMemcpyToSymbol(g_pool, host.data(), host.size() * sizeof(float2),
                                         static_cast<std::size_t>(offset) * sizeof(float2),
                                         cudaMemcpyHostToDevice));
    });
}

__global__ void computed_pass_kernel(float2* out, int n, int e, bool small_last)
{
    const int passes = engine::plan_passes(n, e);
    const int entries = engine::plan_tw_entries(n, e, small_last);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < entries; i += gridDim.x * blockDim.x) {
        int s = 1;
        while (s + 1 < passes && i >= engine::plan_tw_offset(n, e, s + 1, small_last)) {
            ++s;
        }
        out[i] = engine::computed_pass_twiddle(i - engine::plan_tw_offset(n, e, s, small_last),
                                               engine::plan_span(n, e, s, small_last),
                                               engine::plan_radix(n, e, s, small_last));
    }
}

__global__ void computed_half_turn_kernel(float2* out, int n)
{
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k <= n; k += gridDim.x * blockDim.x) {
        out[k] = engine::computed_half_turn(k, n);
    }
}

// Runs a table-filling kernel on the legacy default stream and waits for it, so the table is
// complete before any stream uses it.
template <class Launch>
void fill_on_device(Launch&& launch)
{
    launch();
    SPECTRAL_CUDA(cudaGetLastError());
    SPECTRAL_CUDA(cudaStreamSynchronize(0));
}

}  // namespace

const float2* pass_table(int n, int e, bool small_last)
{
    const int entries = engine::plan_tw_entries(n, e, small_last);
    return get(Key{small_last ? 3 : 0, n, e}, entries < 1 ? 1 : entries, [&](std::vector<float2>& t) {
        const int passes = engine::plan_passes(n, e);
        for (int s = 1; s < passes; ++s) {
            const int L = engine::plan_span(n, e, s, small_last);
            const int R = engine::plan_radix(n, e, s, small_last);
            const int off = engine::plan_tw_offset(n, e, s, small_last);
            for (int r = 0; r < R; ++r) {
                for (int k = 0; k < L; ++k) {
                    t[static_cast<std::size_t>(off + r * L + k)] = forward_factor(
                        static_cast<long long>(k) * r, static_cast<long long>(L) * R);
                }
            }
        }
    });
}

const float2* pass_table_computed(int n, int e, bool small_last)
{
    const int entries = engine::plan_tw_entries(n, e, small_last);
    return get_filled(Key{small_last ? 5 : 4, n, e}, entries < 1 ? 1 : entries, [&](float2* p, long long) {
        if (entries > 0) {
            fill_on_device([&] { computed_pass_kernel<<<(entries + 255) / 256, 256>>>(p, n, e, small_last); });
        }
    });
}

const float2* half_turn_computed(int n)
{
    return get_filled(Key{6, n, 0}, n + 1, [&](float2* p, long long) {
        fill_on_device([&] { computed_half_turn_kernel<<<(n + 256) / 256, 256>>>(p, n); });
    });
}

const float2* half_turn(int n)
{
    return get(Key{1, n, 0}, n + 1, [&](std::vector<float2>& t) {
        for (int k = 0; k <= n; ++k) {
            t[static_cast<std::size_t>(k)] = forward_factor(k, 2LL * n);
        }
    });
}

namespace {

// a rounded to TF32 (10 fraction bits), to nearest with ties away from zero, as the tensor-core
// kernels split their FP32 operands on the GPU.
float tf32_round_host(float a)
{
    unsigned u = 0;
    std::memcpy(&u, &a, sizeof u);
    u = (u + 0x1000u) & 0xFFFFE000u;
    float r = 0.0f;
    std::memcpy(&r, &u, sizeof r);
    return r;
}

}  // namespace

const float2* tf32_dft_rows(int n, int m)
{
    if (n % 8 != 0 || m < 1 || m > kTf32DftOutputs) {
        throw InvalidArgument("tf32_dft_rows: n must be a multiple of 8 and 1 <= m <= 16");
    }
    const long long floats = 4LL * kTf32DftOutputs * n;
    return get(Key{7, n, m}, floats / 2, [&](std::vector<float2>& t) {
        float* f = reinterpret_cast<float*>(t.data());
        constexpr int kRows = 4 * kTf32DftOutputs;
        constexpr int kLboFloats = kRows / 8 * 32;  // one 8-row x 16-byte core matrix per 32 floats
        for (int b = 0; b < kRows; ++b) {
            const int k = b % kTf32DftOutputs;     // output index of this row
            const int part = b / kTf32DftOutputs;  // 0 cos hi, 1 -sin hi, 2 cos lo, 3 -sin lo
            for (int j = 0; j < n; ++j) {
                float v = 0.0f;
                if (k < m) {
                    const dft::CosSin w = dft::cs2pi(static_cast<long long>(k) * j, n);
                    const double exact = (part % 2 == 0) ? w.c : -w.s;
                    const float hi = tf32_round_host(static_cast<float>(exact));
                    v = part < 2 ? hi : tf32_round_host(static_cast<float>(exact - static_cast<double>(hi)));
                }
                f[(j / 4) * kLboFloats + (b / 8) * 32 + (b % 8) * 4 + j % 4] = v;
            }
        }
    });
}

const float2* tf32_idft_rows(int n)
{
    if (n % 8 != 0 || n > 256) {
        throw InvalidArgument("tf32_idft_rows: n must be a multiple of 8 up to 256");
    }
    constexpr int kK = 2 * kTf32DftOutputs;  // cos k, then sin k, k = 0 .. 15
    const long long floats = 2LL * n * kK;
    return get(Key{8, n, 0}, floats / 2, [&](std::vector<float2>& t) {
        float* f = reinterpret_cast<float*>(t.data());
        const int rows = 2 * n;                // hi rows, then lo rows
        const int lbo_floats = rows / 8 * 32;  // one 8-row x 16-byte core matrix per 32 floats
        for (int b = 0; b < rows; ++b) {
            const int j = b % n;  // output position n2 of this row
            for (int kk = 0; kk < kK; ++kk) {
                const int k = kk % kTf32DftOutputs;
                const dft::CosSin w = dft::cs2pi(static_cast<long long>(k) * j, n);
                const double exact = kk < kTf32DftOutputs ? w.c : w.s;
                const float hi = tf32_round_host(static_cast<float>(exact));
                const float v = b < n ? hi : tf32_round_host(static_cast<float>(exact - static_cast<double>(hi)));
                f[(kk / 4) * lbo_floats + (b / 8) * 32 + (b % 8) * 4 + kk % 4] = v;
            }
        }
    });
}

const float2* turn(long long total, int count)
{
    return get(Key{2, total, count}, count, [&](std::vector<float2>& t) {
        for (int j = 0; j < count; ++j) {
            t[static_cast<std::size_t>(j)] = forward_factor(j, total);
        }
    });
}

}  // namespace spectral::twiddles
