// Device CSR/CSC construction and the array primitives.
//
// CSR build (replaces python/mojodgl/heterograph.py:69-86): a stable LSD
// radix sort of (key, edge id) pairs over only the bits the node count needs,
// then row pointers from the run boundaries of the sorted keys, degrees as
// their differences, and the neighbour column gathered through the order.
// Radix sort is stable, so `order` is numpy's argsort(kind="stable") exactly.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace bgl {
namespace {

__global__ void k_prepare_keys(const int64_t *__restrict__ key, int32_t *__restrict__ k32,
                               int32_t *__restrict__ iota, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        k32[i] = static_cast<int32_t>(key[i]);
        iota[i] = static_cast<int32_t>(i);
    }
}

// Every row pointer is written by exactly one thread: thread i (< E) owns the
// rows (sorted[i-1], sorted[i]] and thread E owns (sorted[E-1], num_nodes].
__global__ void k_row_pointers(const int32_t *__restrict__ sorted, int64_t ne, int64_t nn,
                               int64_t *__restrict__ indptr) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= ne;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t prev = (i == 0) ? -1 : sorted[i - 1];
        int64_t cur = (i == ne) ? nn : sorted[i];
        for (int64_t r = prev + 1; r <= cur; ++r) indptr[r] = i;
    }
}

__global__ void k_degrees(const int64_t *__restrict__ indptr, int64_t *__restrict__ deg,
                          int64_t nn) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nn;
         i += (int64_t)gridDim.x * blockDim.x)
        deg[i] = indptr[i + 1] - indptr[i];
}

__global__ void k_gather_other(const int64_t *__restrict__ other,
                               const int32_t *__restrict__ order, int32_t *__restrict__ out,
                               int64_t ne) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < ne;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = static_cast<int32_t>(other[order[i]]);
}

__global__ void k_narrow(const int64_t *__restrict__ src, int32_t *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = static_cast<int32_t>(src[i]);
}

__global__ void k_clamp(const int64_t *__restrict__ src, int64_t *__restrict__ dst, int64_t n,
                        int64_t lo, int64_t hi) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t v = src[i];
        dst[i] = v < lo ? lo : (v > hi ? hi : v);
    }
}

template <typename T>
__global__ void k_riwz(const T *__restrict__ src, T *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        T v = src[i];
        dst[i] = isinf(v) ? T(0) : v;
    }
}

int grid_for(int64_t n, int block = 256) {
    int64_t g = (n + block - 1) / block;
    int64_t cap = int64_t(num_sms()) * 16;
    if (g > cap) g = cap;
    return g < 1 ? 1 : static_cast<int>(g);
}

int key_bits(int64_t num_nodes) {
    int b = 1;
    while (b < 31 && (int64_t(1) << b) < num_nodes) ++b;
    return b;
}

size_t sort_temp_bytes(int64_t ne, int64_t nn) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const int32_t *)nullptr, (int32_t *)nullptr,
                                    (const int32_t *)nullptr, (int32_t *)nullptr, (int)ne, 0,
                                    key_bits(nn));
    return bytes;
}

// bgl_check_csr: result[0] counts bad row pointers (indptr[0] != 0, a
// decrease, indptr[num_rows] != num_edges), result[1] bad ids (a neighbour id
// outside [0, num_src) or an edge id outside [0, num_eid)), result[2] the
// smallest CSR position holding a bad id (-1 if none).  Every read is inside
// the arrays whose sizes the caller gives; an id is only compared, never
// followed.
constexpr unsigned long long kNoPosition = ~0ull;  // reads -1 as int64

__global__ void k_check_init(unsigned long long *r) {
    r[0] = 0;
    r[1] = 0;
    r[2] = kNoPosition;
}

__global__ void k_check_csr(const int64_t *__restrict__ indptr, const int32_t *__restrict__ indices,
                            const int32_t *__restrict__ eid, int64_t rows, int64_t ne,
                            int64_t num_src, int64_t num_eid, unsigned long long *r) {
    const int64_t n = rows + 1 > ne ? rows + 1 : ne;
    unsigned long long bad_ptr = 0, bad_id = 0, first = kNoPosition;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i <= rows) {
            const int64_t p = indptr[i];
            const bool ok = i == 0 ? p == 0 : p >= indptr[i - 1];
            if (!ok || (i == rows && p != ne)) ++bad_ptr;
        }
        if (i < ne) {
            bool ok = true;
            if (indices) ok = ok && indices[i] >= 0 && indices[i] < num_src;
            if (eid) ok = ok && eid[i] >= 0 && eid[i] < num_eid;
            if (!ok) {
                ++bad_id;
                if ((unsigned long long)i < first) first = (unsigned long long)i;
            }
        }
    }
    if (bad_ptr) atomicAdd(&r[0], bad_ptr);
    if (bad_id) atomicAdd(&r[1], bad_id);
    if (first != kNoPosition) atomicMin(&r[2], first);
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_csr_build_workspace_size(int64_t num_edges, int64_t num_nodes) {
    if (num_edges < 0 || num_nodes < 0) return 0;
    Carver c(nullptr);
    c.take<int32_t>(num_edges);
    c.take<int32_t>(num_edges);
    c.take<int32_t>(num_edges);
    c.take<char>(sort_temp_bytes(num_edges, num_nodes));
    return c.used + 256;
}

int bgl_csr_build(const int64_t *key, const int64_t *other, int64_t num_edges, int64_t num_nodes,
                  int64_t *indptr, int64_t *deg, int32_t *order, int32_t *indices,
                  void *workspace, size_t workspace_bytes, void *stream) {
    if (num_edges < 0 || num_nodes < 0)
        return fail(BGL_E_INVALID, "bgl_csr_build: negative size");
    if (num_edges >= (int64_t(1) << 31) || num_nodes >= (int64_t(1) << 31))
        return fail(BGL_E_UNSUPPORTED, "bgl_csr_build: more than 2^31-1 nodes or edges");
    if (!indptr || (num_nodes && !deg) || (num_edges && (!key || !other || !order || !indices)))
        return fail(BGL_E_INVALID, "bgl_csr_build: null pointer");
    if (workspace_bytes < bgl_csr_build_workspace_size(num_edges, num_nodes))
        return fail(BGL_E_WORKSPACE, "bgl_csr_build: workspace too small");
    cudaStream_t s = as_stream(stream);
    Carver c(workspace);
    int32_t *k32 = c.take<int32_t>(num_edges);
    int32_t *ks = c.take<int32_t>(num_edges);
    int32_t *iota = c.take<int32_t>(num_edges);
    size_t tb = sort_temp_bytes(num_edges, num_nodes);
    void *temp = c.take<char>(tb);
    if (num_edges > 0) {
        k_prepare_keys<<<grid_for(num_edges), 256, 0, s>>>(key, k32, iota, num_edges);
        BGL_LAUNCH_CHECK();
        BGL_CUDA(cub::DeviceRadixSort::SortPairs(temp, tb, k32, ks, iota, order, (int)num_edges,
                                                 0, key_bits(num_nodes), s));
    }
    k_row_pointers<<<grid_for(num_edges + 1), 256, 0, s>>>(ks, num_edges, num_nodes, indptr);
    BGL_LAUNCH_CHECK();
    if (num_nodes > 0) {
        k_degrees<<<grid_for(num_nodes), 256, 0, s>>>(indptr, deg, num_nodes);
        BGL_LAUNCH_CHECK();
    }
    if (num_edges > 0) {
        k_gather_other<<<grid_for(num_edges), 256, 0, s>>>(other, order, indices, num_edges);
        BGL_LAUNCH_CHECK();
    }
    return BGL_OK;
}

int bgl_check_csr(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
                  int64_t num_rows, int64_t num_edges, int64_t num_src, int64_t num_eid,
                  int64_t *result, void *stream) {
    if (num_rows < 0 || num_edges < 0 || num_src < 0 || num_eid < 0)
        return fail(BGL_E_INVALID, "bgl_check_csr: negative size");
    if (!indptr || !result) return fail(BGL_E_INVALID, "bgl_check_csr: null indptr or result");
    cudaStream_t s = as_stream(stream);
    auto *r = reinterpret_cast<unsigned long long *>(result);
    k_check_init<<<1, 1, 0, s>>>(r);
    BGL_LAUNCH_CHECK();
    const int64_t n = num_rows + 1 > num_edges ? num_rows + 1 : num_edges;
    int64_t g = (n + 255) / 256;
    const int64_t cap = int64_t(num_sms()) * 16;
    k_check_csr<<<(int)(g < 1 ? 1 : g > cap ? cap : g), 256, 0, s>>>(
        indptr, indices, eid, num_rows, num_edges, num_src, num_eid, r);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

int bgl_narrow_i64(const int64_t *src, int32_t *dst, int64_t n, void *stream) {
    if (n < 0) return fail(BGL_E_INVALID, "bgl_narrow_i64: negative size");
    if (n == 0) return BGL_OK;
    k_narrow<<<grid_for(n), 256, 0, as_stream(stream)>>>(src, dst, n);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

size_t bgl_cumsum_workspace_size(int64_t n) {
    size_t bytes = 0;
    cub::DeviceScan::InclusiveSum(nullptr, bytes, (const int64_t *)nullptr, (int64_t *)nullptr,
                                  (int)(n > 0 ? n : 1));
    return bytes + 256;
}

int bgl_cumsum_i64(const int64_t *src, int64_t *dst, int64_t n, void *workspace,
                   size_t workspace_bytes, void *stream) {
    if (n < 0 || n >= (int64_t(1) << 31)) return fail(BGL_E_INVALID, "bgl_cumsum_i64: bad size");
    if (n == 0) return BGL_OK;
    size_t need = bgl_cumsum_workspace_size(n);
    if (workspace_bytes < need) return fail(BGL_E_WORKSPACE, "bgl_cumsum_i64: workspace too small");
    size_t tb = need - 256;
    BGL_CUDA(cub::DeviceScan::InclusiveSum(workspace, tb, src, dst, (int)n, as_stream(stream)));
    return BGL_OK;
}

int bgl_clamp_i64(const int64_t *src, int64_t *dst, int64_t n, int64_t lo, int64_t hi,
                  void *stream) {
    if (n < 0) return fail(BGL_E_INVALID, "bgl_clamp_i64: negative size");
    if (n == 0) return BGL_OK;
    k_clamp<<<grid_for(n), 256, 0, as_stream(stream)>>>(src, dst, n, lo, hi);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

int bgl_replace_inf_with_zero(const void *src, void *dst, int64_t n, int dtype, void *stream) {
    if (n < 0) return fail(BGL_E_INVALID, "bgl_replace_inf_with_zero: negative size");
    if (n == 0) return BGL_OK;
    cudaStream_t s = as_stream(stream);
    if (dtype == BGL_F32)
        k_riwz<float><<<grid_for(n), 256, 0, s>>>((const float *)src, (float *)dst, n);
    else if (dtype == BGL_F64)
        k_riwz<double><<<grid_for(n), 256, 0, s>>>((const double *)src, (double *)dst, n);
    else
        return fail(BGL_E_UNSUPPORTED, "bgl_replace_inf_with_zero: dtype %d", dtype);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

}  // extern "C"
