// Device buffers shared between the processes of one node (one process per GPU) through CUDA IPC,
// for the slab transform's peer-memory exchange (slab.cu: spectral_slab_rows_peer). A rank
// allocates its receive buffer here, passes the 64-byte handle to the other ranks (any host
// channel: torch.distributed's all_gather_object in spectral.distributed), and each of them maps
// it into its own address space. Plain device memory and plain loads and stores over NVLink: no
// multicast object is created.

#include "../../include/spectral_b200.h"

#include "backend.hpp"

#include <cstring>
#include <string>

namespace {

int ipc_status(cudaError_t e, const char* what)
{
    if (e == cudaSuccess) {
        return SPECTRAL_OK;
    }
    spectral::set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
    return SPECTRAL_CUDA_ERROR;
}

}  // namespace

static_assert(sizeof(cudaIpcMemHandle_t) == SPECTRAL_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int spectral_ipc_alloc(unsigned long long bytes, void** ptr, void* handle)
{
    if (ptr == nullptr || handle == nullptr || bytes == 0) {
        spectral::set_last_error("ipc_alloc: need bytes > 0 and non-null ptr and handle");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    *ptr = nullptr;
    int st = ipc_status(cudaMalloc(ptr, bytes), "ipc_alloc: cudaMalloc");
    if (st != SPECTRAL_OK) {
        return st;
    }
    cudaIpcMemHandle_t h;
    st = ipc_status(cudaIpcGetMemHandle(&h, *ptr), "ipc_alloc: cudaIpcGetMemHandle");
    if (st != SPECTRAL_OK) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return st;
    }
    std::memcpy(handle, &h, sizeof(h));
    return SPECTRAL_OK;
}

extern "C" int spectral_ipc_open(const void* handle, void** ptr)
{
    if (ptr == nullptr || handle == nullptr) {
        spectral::set_last_error("ipc_open: need non-null handle and ptr");
        return SPECTRAL_INVALID_ARGUMENT;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return ipc_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                      "ipc_open: cudaIpcOpenMemHandle");
}

extern "C" int spectral_ipc_close(void* ptr)
{
    return ipc_status(cudaIpcCloseMemHandle(ptr), "ipc_close: cudaIpcCloseMemHandle");
}

extern "C" int spectral_ipc_free(void* ptr)
{
    return ipc_status(cudaFree(ptr), "ipc_free: cudaFree");
}
