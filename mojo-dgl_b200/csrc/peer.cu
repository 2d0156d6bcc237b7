// Peer buffers for the multi-GPU halo: device memory shared between the
// processes of one node (one process per GPU) through CUDA IPC, and copies
// between them run by the copy engines, so a halo transfer over NVLink takes
// no SM time from the gSpMM passes it overlaps.
//
// Every entry point checks the byte range it is given against the device
// allocation that holds it (cuMemGetAddressRange) before it maps or queues
// anything: a range that leaves its allocation is rejected with
// BGL_E_INVALID, so no copy can reach outside a buffer.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace bgl {
namespace {

typedef CUresult (*AddrRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);

AddrRangeFn addr_range_fn() {
    static AddrRangeFn f = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f = reinterpret_cast<AddrRangeFn>(p);
    });
    return f;
}

// The allocation holding ptr (its base and size); fails unless
// [ptr, ptr + bytes) lies inside it.
int allocation_of(const void *ptr, int64_t bytes, const char *what, CUdeviceptr *base,
                  size_t *size) {
    if (ptr == nullptr || bytes < 0)
        return fail(BGL_E_INVALID, "%s: null pointer or negative size", what);
    AddrRangeFn f = addr_range_fn();
    if (!f) return fail(BGL_E_CUDA, "cuMemGetAddressRange is not available from the driver");
    CUresult r = f(base, size, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS)
        return fail(BGL_E_INVALID, "%s: %p is not device memory of this process (CUresult %d)",
                    what, ptr, (int)r);
    const uint64_t p = reinterpret_cast<uint64_t>(ptr), b = (uint64_t)*base;
    if (p < b || p - b + (uint64_t)bytes > (uint64_t)*size)
        return fail(BGL_E_INVALID, "%s: %lld bytes at offset %llu leave the %zu-byte allocation",
                    what, (long long)bytes, (unsigned long long)(p - b), *size);
    return BGL_OK;
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

int bgl_ipc_export(const void *ptr, int64_t bytes, void *handle, int64_t *offset) {
    if (!handle || !offset) return fail(BGL_E_INVALID, "bgl_ipc_export: null output");
    CUdeviceptr base;
    size_t size;
    int rc = allocation_of(ptr, bytes, "bgl_ipc_export", &base, &size);
    if (rc != BGL_OK) return rc;
    cudaIpcMemHandle_t h;
    BGL_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)));
    static_assert(sizeof(h) == BGL_IPC_HANDLE_BYTES, "cudaIpcMemHandle_t size");
    memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)(reinterpret_cast<uint64_t>(ptr) - (uint64_t)base);
    return BGL_OK;
}

int bgl_ipc_open(const void *handle, int64_t offset, int64_t bytes, void **ptr) {
    if (!handle || !ptr || offset < 0 || bytes < 0)
        return fail(BGL_E_INVALID, "bgl_ipc_open: null argument or negative offset/size");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *base = nullptr;
    BGL_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    CUdeviceptr b;
    size_t size;
    int rc = allocation_of(base, 0, "bgl_ipc_open", &b, &size);
    if (rc == BGL_OK && (uint64_t)offset + (uint64_t)bytes > (uint64_t)size)
        rc = fail(BGL_E_INVALID, "bgl_ipc_open: %lld bytes at offset %lld leave the %zu-byte "
                  "exported allocation", (long long)bytes, (long long)offset, size);
    if (rc != BGL_OK) {
        cudaIpcCloseMemHandle(base);
        return rc;
    }
    *ptr = static_cast<unsigned char *>(base) + offset;
    return BGL_OK;
}

int bgl_ipc_close(void *ptr) {
    if (!ptr) return fail(BGL_E_INVALID, "bgl_ipc_close: null pointer");
    CUdeviceptr base;
    size_t size;
    int rc = allocation_of(ptr, 0, "bgl_ipc_close", &base, &size);
    if (rc != BGL_OK) return rc;
    BGL_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void *>(base)));
    return BGL_OK;
}

int bgl_peer_copy(void *dst, const void *src, int64_t bytes, void *stream) {
    if (!dst || !src || bytes < 0)
        return fail(BGL_E_INVALID, "bgl_peer_copy: null pointer or negative size");
    if (bytes == 0) return BGL_OK;
    CUdeviceptr base;
    size_t size;
    int rc = allocation_of(dst, bytes, "bgl_peer_copy (destination)", &base, &size);
    if (rc != BGL_OK) return rc;
    rc = allocation_of(src, bytes, "bgl_peer_copy (source)", &base, &size);
    if (rc != BGL_OK) return rc;
    BGL_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault,
                             static_cast<cudaStream_t>(stream)));
    return BGL_OK;
}

}  // extern "C"
