// Peer mappings of device buffers between the processes of one node (CUDA IPC), for kernels
// that store straight into other ranks' memory over NVLink (the attention epilogue's fused
// all-gather of head-sharded outputs).
//
// A buffer handed out by a caching allocator is usually an interior part of a larger
// allocation; an IPC handle always names a whole allocation.  Export therefore records the
// allocation's handle plus the buffer's byte offset inside it, and import opens the handle
// in the CALLING device's context with peer access enabled from that device -- opening it
// under the owner's device index instead (what a generic tensor-sharing path does, since its
// consumer runs on the owner's device) leaves the launching device without a mapping.
#include <string.h>

#include <cuda.h>

#include "skv_common.cuh"

namespace {

// The plain exchange: every 16-byte chunk of src loaded once and stored into each destination
// (this rank's buffer and its peers', over NVLink); four chunks in flight per thread.
__global__ void __launch_bounds__(256) peer_store_kernel(const uint4* __restrict__ src, int64_t n16,
                                                         const int64_t* __restrict__ dst, int n_dst, int64_t off16) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n16; i0 += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * stride < n16) v[u] = __ldg(src + i0 + u * stride);
        for (int r = 0; r < n_dst; ++r) {
            uint4* d = reinterpret_cast<uint4*>(dst[r]) + off16;
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i0 + u * stride < n16) d[i0 + u * stride] = v[u];
        }
    }
}

typedef CUresult (*PFN_addr_range)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange through the runtime's driver entry point (no link against libcuda).
PFN_addr_range address_range_fn() {
    static PFN_addr_range fn = nullptr;
    static bool tried = false;
    if (!tried) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_addr_range>(f);
        tried = true;
    }
    return fn;
}

}  // namespace

extern "C" {

int skv_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int skv_ipc_export(const void* ptr, void* handle, int64_t* offset) {
    if (!ptr || !handle || !offset) return skv::fail(SKV_ERR_INVALID_ARGUMENT, "ipc_export: null argument");
    PFN_addr_range range = address_range_fn();
    if (!range) return skv::fail(SKV_ERR_CUDA, "ipc_export: cuMemGetAddressRange is not available");
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = range(&base, &size, (CUdeviceptr)ptr);
    if (r != CUDA_SUCCESS) return skv::fail(SKV_ERR_CUDA, "ipc_export: cuMemGetAddressRange failed (%d)", (int)r);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
    if (e != cudaSuccess) return skv::fail(SKV_ERR_CUDA, "ipc_export: %s", cudaGetErrorString(e));
    memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)((CUdeviceptr)ptr - base);
    return SKV_OK;
}

int skv_ipc_open(const void* handle, int64_t offset, void** base, void** ptr) {
    if (!handle || !base || !ptr || offset < 0)
        return skv::fail(SKV_ERR_INVALID_ARGUMENT, "ipc_open: null argument or negative offset");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* b = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return skv::fail(SKV_ERR_CUDA, "ipc_open: %s", cudaGetErrorString(e));
    *base = b;
    *ptr = (char*)b + offset;
    return SKV_OK;
}

int skv_ipc_close(void* base) {
    if (!base) return skv::fail(SKV_ERR_INVALID_ARGUMENT, "ipc_close: null base");
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return skv::fail(SKV_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
    return SKV_OK;
}

int skv_peer_store(const void* src, int64_t bytes, const int64_t* dst_ptrs, int n_dst, int64_t dst_offset,
                   void* stream) {
    if (!src || !dst_ptrs || n_dst <= 0 || bytes < 0 || dst_offset < 0)
        return skv::fail(SKV_ERR_INVALID_ARGUMENT, "peer_store: null pointer or bad size");
    if ((bytes & 15) || (dst_offset & 15) || (reinterpret_cast<uintptr_t>(src) & 15))
        return skv::fail(SKV_ERR_INVALID_ARGUMENT, "peer_store: source, size and offset must be 16-byte multiples");
    if (bytes == 0) return SKV_OK;
    const int64_t n16 = bytes / 16;
    const int64_t want = (n16 + 1023) / 1024;
    const int64_t cap = (int64_t)skv::sm_count() * 8;
    const int blocks = (int)(want < cap ? want : cap);
    peer_store_kernel<<<blocks, 256, 0, skv::as_stream(stream)>>>(reinterpret_cast<const uint4*>(src), n16, dst_ptrs,
                                                                   n_dst, dst_offset / 16);
    return skv::check_launch("peer_store");
}

}  // extern "C"
