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
//  * the array's device address belongs to one CUDA context: it is resolved
//    with cudaGetSymbolAddress the first time a call runs in a context (the
//    device's primary context, or one the caller created and made current)
//    and cached under that context's unique id, so a context created later,
//    also after a cudaDeviceReset, resolves its own address.  The resolving
//    call may load the module; make the first call in each context before
//    any stream capture.
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace bgl {
namespace {

constexpr size_t kStaticScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_spmm_scratch[kStaticScratchBytes];

// Driver entry points, fetched through the runtime (no link against the
// driver library): the current context and its process-unique id.
typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

struct CtxFns {
    CtxGetCurrentFn current = nullptr;
    CtxGetIdFn id = nullptr;
};

const CtxFns &ctx_fns() {
    static CtxFns f;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f.current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f.id = reinterpret_cast<CtxGetIdFn>(p);
    });
    return f;
}

// Resolved addresses by context id.  A context id is never reused within a
// process, so an entry can go stale only by its context being destroyed, and
// then no call can run in it again; the table evicts round robin when full.
constexpr int kSlots = 64;
struct Slot {
    bool used = false;
    unsigned long long ctx_id = 0;
    void *ptr = nullptr;
};
std::mutex g_scratch_mutex;
Slot g_slots[kSlots];
int g_next_slot = 0;

// The calling thread's current context's id; *have = false if no context is
// current.
int current_ctx_id(bool *have, unsigned long long *id) {
    const CtxFns &f = ctx_fns();
    if (!f.current || !f.id)
        return fail(BGL_E_CUDA, "cuCtxGetCurrent/cuCtxGetId are not available from the driver");
    CUcontext ctx = nullptr;
    *have = false;
    if (f.current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return BGL_OK;
    if (f.id(ctx, id) != CUDA_SUCCESS) return fail(BGL_E_CUDA, "cuCtxGetId failed");
    *have = true;
    return BGL_OK;
}

// The array's device address in the calling thread's current context.
int scratch_address(void **out) {
    bool have = false;
    unsigned long long id = 0;
    int rc = current_ctx_id(&have, &id);
    if (rc != BGL_OK) return rc;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (have)
        for (const Slot &s : g_slots)
            if (s.used && s.ctx_id == id) {
                *out = s.ptr;
                return BGL_OK;
            }
    // Not resolved in this context yet (or no context is current, in which
    // case the runtime binds the device's primary context here).
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_spmm_scratch);
    if (e != cudaSuccess || p == nullptr)
        return fail(BGL_E_CUDA, "cudaGetSymbolAddress(static gspmm scratch) failed: %s",
                    cudaGetErrorString(e));
    if (!have) {
        rc = current_ctx_id(&have, &id);
        if (rc != BGL_OK) return rc;
    }
    if (have) {
        g_slots[g_next_slot] = Slot{true, id, p};
        g_next_slot = (g_next_slot + 1) % kSlots;
    }
    *out = p;
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
