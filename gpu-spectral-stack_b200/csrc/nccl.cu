// The slab transform's exchange on a caller's NCCL communicator, for C and C++ callers that run
// the whole 2D transform through the C ABI (spectral_fft2_slab) rather than through
// torch.distributed (spectral.distributed.fft2_slab).
//
// The library does not link NCCL: a communicator must come from the same NCCL the caller uses,
// so the entry points are resolved at run time from the libnccl.so.2 already loaded into the
// process (torch's, or the caller's), else from the one the loader finds. nccl.h supplies the
// types only.

#include "../../include/spectral_b200.h"

#include "backend.hpp"

#include <dlfcn.h>
#include <nccl.h>

#include <climits>
#include <cstring>
#include <string>

namespace spectral {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    std::string missing;  // empty when every entry point resolved
};

template <class F>
void bind(void* handle, const char* name, F& fn, std::string& missing)
{
    fn = reinterpret_cast<F>(dlsym(handle, name));
    if (fn == nullptr) {
        missing += std::string(missing.empty() ? "" : ", ") + name;
    }
}

NcclApi load_nccl()
{
    NcclApi api;
    void* handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (handle == nullptr) {
        handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    }
    if (handle == nullptr) {
        api.missing = "libnccl.so.2 (not loaded and not found)";
        return api;
    }
    bind(handle, "ncclGetUniqueId", api.get_unique_id, api.missing);
    bind(handle, "ncclCommInitRank", api.comm_init_rank, api.missing);
    bind(handle, "ncclCommDestroy", api.comm_destroy, api.missing);
    bind(handle, "ncclGroupStart", api.group_start, api.missing);
    bind(handle, "ncclGroupEnd", api.group_end, api.missing);
    bind(handle, "ncclSend", api.send, api.missing);
    bind(handle, "ncclRecv", api.recv, api.missing);
    bind(handle, "ncclGetErrorString", api.error_string, api.missing);
    return api;
}

const NcclApi& nccl()
{
    static const NcclApi api = load_nccl();  // thread-safe one-time initialisation
    if (!api.missing.empty()) {
        throw CudaError("NCCL unavailable: " + api.missing);
    }
    return api;
}

void nccl_check(ncclResult_t r, const char* what)
{
    if (r != ncclSuccess) {
        throw CudaError(std::string(what) + ": " + nccl().error_string(r));
    }
}

template <class F>
int nccl_guarded(F&& f)
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

// Chunk s of `send` (values complex values) to rank s, chunk s of `recv` from rank s, every s.
void exchange(const float2* send, float2* recv, long long values, int ranks, ncclComm_t comm,
              cudaStream_t s)
{
    const NcclApi& api = nccl();
    const size_t floats = static_cast<size_t>(values) * 2;
    nccl_check(api.group_start(), "ncclGroupStart");
    for (int q = 0; q < ranks; ++q) {
        nccl_check(api.send(send + static_cast<long long>(q) * values, floats, ncclFloat32, q, comm, s), "ncclSend");
        nccl_check(api.recv(recv + static_cast<long long>(q) * values, floats, ncclFloat32, q, comm, s), "ncclRecv");
    }
    nccl_check(api.group_end(), "ncclGroupEnd");
}

void check_field(int n, int rank, int ranks)
{
    if (n < 2 || n > 16384 || (n & (n - 1)) != 0) {
        throw InvalidArgument("fft2_slab: n must be a power of two from 2 to 16384, got " + std::to_string(n));
    }
    if (ranks < 1 || (ranks & (ranks - 1)) != 0 || ranks > n) {
        throw InvalidArgument("fft2_slab: the ranks (" + std::to_string(ranks)
                              + ") must be a power of two dividing n = " + std::to_string(n));
    }
    if (rank < 0 || rank >= ranks) {
        throw InvalidArgument("fft2_slab: rank " + std::to_string(rank) + " outside 0 .. " + std::to_string(ranks - 1));
    }
}

void status(int code)
{
    if (code == SPECTRAL_INVALID_ARGUMENT) {
        throw InvalidArgument(spectral_last_error());
    }
    if (code != SPECTRAL_OK) {
        throw CudaError(spectral_last_error());
    }
}

}  // namespace
}  // namespace spectral

static_assert(sizeof(ncclUniqueId) == SPECTRAL_NCCL_ID_BYTES, "NCCL unique id size");

extern "C" int spectral_nccl_unique_id(void* id)
{
    using namespace spectral;
    return nccl_guarded([&] {
        if (id == nullptr) {
            throw InvalidArgument("nccl_unique_id: id must not be null");
        }
        ncclUniqueId u;
        nccl_check(nccl().get_unique_id(&u), "ncclGetUniqueId");
        std::memcpy(id, &u, sizeof(u));
    });
}

extern "C" int spectral_nccl_comm_init(const void* id, int rank, int ranks, void** comm)
{
    using namespace spectral;
    return nccl_guarded([&] {
        if (id == nullptr || comm == nullptr || ranks < 1 || rank < 0 || rank >= ranks) {
            throw InvalidArgument("nccl_comm_init: need an id, a comm pointer and 0 <= rank < ranks");
        }
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        ncclComm_t c = nullptr;
        nccl_check(nccl().comm_init_rank(&c, ranks, u, rank), "ncclCommInitRank");
        *comm = c;
    });
}

extern "C" int spectral_nccl_comm_destroy(void* comm)
{
    using namespace spectral;
    return nccl_guarded([&] { nccl_check(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy"); });
}

extern "C" int spectral_slab_exchange(const void* send, void* recv, long long values_per_rank, int ranks,
                                      void* comm, void* stream)
{
    using namespace spectral;
    return nccl_guarded([&] {
        if (values_per_rank < 0 || ranks < 1 || comm == nullptr || send == recv) {
            throw InvalidArgument("slab_exchange: need values_per_rank >= 0, ranks >= 1, a communicator and send != recv");
        }
        exchange(static_cast<const float2*>(send), static_cast<float2*>(recv), values_per_rank, ranks,
                 static_cast<ncclComm_t>(comm), static_cast<cudaStream_t>(stream));
    });
}

extern "C" int spectral_fft2_slab_workspace(int n, int ranks, size_t* count)
{
    using namespace spectral;
    return nccl_guarded([&] {
        check_field(n, 0, ranks);
        if (count == nullptr) {
            throw InvalidArgument("fft2_slab_workspace: count must not be null");
        }
        *count = 2 * static_cast<size_t>(n) * static_cast<size_t>(n / ranks);
    });
}

extern "C" int spectral_fft2_slab(const void* x, void* y, void* work, int n, int rank, int ranks,
                                  int inverse, void* comm, void* stream)
{
    using namespace spectral;
    return nccl_guarded([&] {
        check_field(n, rank, ranks);
        if (x == nullptr || y == nullptr || work == nullptr || comm == nullptr) {
            throw InvalidArgument("fft2_slab: x, y, work and comm must not be null");
        }
        const int w = n / ranks;
        const long long slab = static_cast<long long>(n) * w;  // complex values per rank
        float2* a = static_cast<float2*>(work);
        float2* b = a + slab;
        const auto s = static_cast<cudaStream_t>(stream);
        const auto c = static_cast<ncclComm_t>(comm);
        if (!inverse) {
            // rows of x -> chunks (a) -> exchange (b) -> columns (b is scratch) -> y
            status(spectral_slab_rows(x, a, n, w, ranks, 0, stream));
            exchange(a, b, slab / ranks, ranks, c, s);
            status(spectral_slab_columns(b, y, n, w, 0, stream));
        } else {
            // column slab x (copied: the column stage uses its input as scratch) -> columns (b)
            // -> exchange of its row blocks (a) -> rows -> y
            SPECTRAL_CUDA(cudaMemcpyAsync(a, x, static_cast<size_t>(slab) * sizeof(float2),
                                          cudaMemcpyDeviceToDevice, s));
            status(spectral_slab_columns(a, b, n, w, 1, stream));
            exchange(b, a, slab / ranks, ranks, c, s);
            status(spectral_slab_rows(a, y, n, w, ranks, 1, stream));
        }
    });
}
