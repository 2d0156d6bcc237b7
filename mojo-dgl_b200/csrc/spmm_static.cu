// bgl_gspmm_static_scratch: gSpMM for callers that cannot allocate device
// memory.
//
// bgl_gspmm needs a workspace (the merge-path chunk boundaries, and the pieces
// of rows split across chunks) that its caller allocates.  Some callers cannot
// do that: a plugin or serving runtime that owns every device allocation and
// hands a kernel library nothing but its input and output buffers, or a
// latency-critical request path where a cudaMalloc -- which can synchronise
// the device and fragments a pre-carved memory pool -- is not allowed.  This
// entry point serves them: it takes the same arguments as bgl_gspmm minus the
// workspace, and uses instead the fixed scratch array below, which every GPU
// that loads this library holds from the module's load until process exit.
//
// Limits and behaviour:
//  * the scratch holds BGL_STATIC_SCRATCH_BYTES (64 MiB); a call whose plan
//    needs more (bgl_gspmm_workspace_size) is rejected with BGL_E_INVALID and
//    a message giving both sizes, before any work is queued;
//  * every call on a device shares the one array, so calls whose kernels can
//    overlap on the GPU (different streams, or different host threads) race
//    on it and must be serialised by the caller;
//  * the array keeps the previous call's contents; nothing in it has to start
//    at zero, because every word a call reads was written earlier in the same
//    call (chunk boundaries by the boundary kernel, row ids and pieces by the
//    main kernel);
//  * the first call on each device resolves the array's device address with
//    cudaGetSymbolAddress while that device is current (this also loads the
//    module if it is not loaded yet); make that first call before any stream
//    capture.
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "common.cuh"

namespace bgl {
namespace {

constexpr size_t kStaticScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_spmm_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void *g_scratch_ptr[64] = {nullptr};

// The array's device address on the current device (resolved once per device).
int scratch_address(void **out) {
    int dev = 0;
    BGL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(BGL_E_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_ptr[dev] == nullptr) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_spmm_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(BGL_E_CUDA, "cudaGetSymbolAddress(static gspmm scratch) failed: %s",
                        cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return BGL_OK;
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_static_scratch_bytes(void) { return kStaticScratchBytes; }

int bgl_gspmm_static_scratch(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
                             const int64_t *deg, int64_t num_rows, int64_t num_edges,
                             const void *lhs, int64_t lhs_width, int64_t lhs_div, const void *rhs,
                             int64_t rhs_width, int64_t rhs_div, void *out, int64_t dout,
                             int64_t *arg_u, int64_t *arg_e, int dtype, int op, int reduce,
                             int flags, void *stream) {
    if (num_rows < 0 || num_edges < 0 || dout < 0)
        return fail(BGL_E_INVALID, "bgl_gspmm_static_scratch: negative size");
    const size_t need = bgl_gspmm_workspace_size(num_rows, num_edges, dout, dtype, reduce);
    if (need > kStaticScratchBytes)
        return fail(BGL_E_INVALID,
                    "bgl_gspmm_static_scratch: this call needs %zu bytes of scratch but the "
                    "built-in scratch holds %zu; pass a workspace to bgl_gspmm instead",
                    need, kStaticScratchBytes);
    void *scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc != BGL_OK) return rc;
    return bgl_gspmm(indptr, indices, eid, deg, num_rows, num_edges, lhs, lhs_width, lhs_div, rhs,
                     rhs_width, rhs_div, out, dout, arg_u, arg_e, dtype, op, reduce, flags,
                     scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
