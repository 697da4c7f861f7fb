// Correctly rounded twiddle tables (see twiddles.cuh).

#include "twiddles.cuh"

#include "dft.cuh"
#include "engine.cuh"

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

template <class Build>
const float2* get(const Key& key, long long count, Build&& build)
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
    const long long aligned = (dt.used + 1) & ~1LL;  // 16-byte aligned tables
    if (aligned + count > kPoolEntries) {
        throw InvalidArgument("twiddle tables: pool exhausted");
    }
    std::vector<float2> host(static_cast<std::size_t>(count));
    build(host);
    SPECTRAL_CUDA(cudaMemcpyToSymbol(g_pool, host.data(), host.size() * sizeof(float2),
                                     static_cast<std::size_t>(aligned) * sizeof(float2),
                                     cudaMemcpyHostToDevice));
    const float2* ptr = dt.base + aligned;
    dt.used = aligned + count;
    dt.tables.emplace(key, ptr);
    return ptr;
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

const float2* half_turn(int n)
{
    return get(Key{1, n, 0}, n + 1, [&](std::vector<float2>& t) {
        for (int k = 0; k <= n; ++k) {
            t[static_cast<std::size_t>(k)] = forward_factor(k, 2LL * n);
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
