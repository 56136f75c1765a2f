// Peer-memory mappings for the fused attention + all-gather (hb_paired_fwd_allgather):
// CUDA IPC handles of ordinary device allocations, opened in the other ranks'
// processes.  Plain mappings only — no multicast objects are created, so a rank
// that exits leaves nothing bound on its peers' GPUs.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/hilberta_b200.h"
#include "common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == HB_IPC_HANDLE_BYTES, "IPC handle size");

namespace {
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddressRangeFn>(ptr);
    });
    return fn;
}
}  // namespace

extern "C" int hb_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
    if (!ptr || !handle || !offset) return HB_ERR_ARG;
    AddressRangeFn range = address_range_fn();
    if (!range) return HB_ERR_CUDA;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return HB_ERR_ARG;
    cudaIpcMemHandle_t h;
    HB_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle, &h, sizeof(h));
    *offset = (uint64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
    return HB_OK;
}

extern "C" int hb_ipc_open(const void* handle, uint64_t offset, void** ptr) {
    if (!handle || !ptr) return HB_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    HB_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = static_cast<char*>(base) + offset;
    return HB_OK;
}

extern "C" int hb_ipc_close(void* ptr, uint64_t offset) {
    if (!ptr) return HB_ERR_ARG;
    HB_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
    return HB_OK;
}

extern "C" int hb_peer_copy(void* dst, const void* src, size_t bytes, void* stream) {
    if (!dst || !src) return HB_ERR_ARG;
    if (bytes == 0) return HB_OK;
    HB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    return HB_OK;
}
