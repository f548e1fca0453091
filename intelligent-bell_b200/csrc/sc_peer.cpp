// sc_peer.cpp — share a GPU buffer with the other processes of one machine (CUDA IPC), so that
// each GPU's restore kernel can store its KV-head shard straight into one consumer GPU's
// cache over NVLink (a gather with no separate collective and no staging copy).
//
// Plain CUDA IPC: the owner exports the allocation that holds its buffer; an importer maps
// it into its own device's address space with peer access enabled, and its kernels then
// write it with ordinary stores.  No multicast object is involved.
#include <string.h>

#include <mutex>

#include "sc_internal.h"

namespace {

using GetRangeFn = int (*)(unsigned long long*, size_t*, unsigned long long);  // CUresult(...)
GetRangeFn g_get_range = nullptr;
std::once_flag g_range_once;

int32_t allocation_base(const void* ptr, const void** base) {
    std::call_once(g_range_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_get_range = reinterpret_cast<GetRangeFn>(fn);
    });
    if (g_get_range == nullptr)
        return sc::set_error(SC_ERR_UNSUPPORTED, "cuMemGetAddressRange is not available");
    unsigned long long b = 0;
    size_t size = 0;
    const int r = g_get_range(&b, &size, reinterpret_cast<unsigned long long>(ptr));
    if (r != 0)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT,
                             "pointer %p is not inside a device allocation (driver error %d)", ptr, r);
    *base = reinterpret_cast<const void*>(b);
    return SC_OK;
}

}  // namespace

extern "C" int32_t sc_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
    if (!dev_ptr || !handle_out || !offset_out)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "null argument");
    const void* base = nullptr;
    const int32_t rc = allocation_base(dev_ptr, &base);
    if (rc != SC_OK) return rc;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
    if (e != cudaSuccess) return sc::cuda_error(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == SC_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    *offset_out = static_cast<const char*>(dev_ptr) - static_cast<const char*>(base);
    return sc::ok();
}

extern "C" int32_t sc_ipc_import(const void* handle, int64_t offset, void** base_out,
                                 void** ptr_out) {
    if (!handle || !base_out || !ptr_out || offset < 0)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "invalid argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return sc::cuda_error(e, "cudaIpcOpenMemHandle");
    *base_out = base;
    *ptr_out = static_cast<char*>(base) + offset;
    return sc::ok();
}

extern "C" int32_t sc_ipc_close(void* base) {
    if (!base) return sc::ok();
    const cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return sc::cuda_error(e, "cudaIpcCloseMemHandle");
    return sc::ok();
}
