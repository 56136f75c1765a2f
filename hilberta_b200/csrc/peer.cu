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

namespace {
struct ScatterDst {
    uint4* p[HB_MAX_RANKS];
};

// Grid-stride copy of n16 16-byte chunks to every destination: each lane loads
// one chunk (L2 only) and stores it to each destination before the next.
__global__ void __launch_bounds__(512) k_peer_scatter(const uint4* __restrict__ src, ScatterDst dst, int n_dst,
                                                      int64_t n16) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
        const uint4 v = __ldcg(src + i);
        for (int d = 0; d < n_dst; d++) dst.p[d][i] = v;
    }
}
}  // namespace

extern "C" int hb_peer_scatter(const void* src, void* const* dst, int n_dst, size_t bytes, void* stream) {
    if (!src || !dst || n_dst < 1 || n_dst > HB_MAX_RANKS || (bytes & 15) ||
        (reinterpret_cast<uintptr_t>(src) & 15))
        return HB_ERR_ARG;
    ScatterDst d;
    for (int i = 0; i < n_dst; i++) {
        if (!dst[i] || (reinterpret_cast<uintptr_t>(dst[i]) & 15)) return HB_ERR_ARG;
        d.p[i] = static_cast<uint4*>(dst[i]);
    }
    if (bytes == 0) return HB_OK;
    int dev = 0, sms = 0;
    HB_CUDA_TRY(cudaGetDevice(&dev));
    HB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t n16 = (int64_t)(bytes / 16);
    const int64_t want = (n16 + 511) / 512;
    const int grid = (int)(want < 2 * sms ? want : 2 * sms);
    k_peer_scatter<<<grid, 512, 0, (cudaStream_t)stream>>>(static_cast<const uint4*>(src), d, n_dst, n16);
    HB_LAUNCH_CHECK();
    return HB_OK;
}
