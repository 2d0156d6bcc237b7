// The reference-compatible C ABI: src/capi.mojo's eleven `mdgl_*` exports with
// the same names, all-int64 argument lists, host float64/int64 buffers and
// void returns, so the reference's own python/mojodgl/_lib.py can load this
// library (MOJODGL_LIB) unchanged.  Each call copies its host inputs to the
// current CUDA device, runs the float64 kernels of this library, and copies the
// result back before it returns; nothing persists between calls.
//
// The reference has no error channel (void returns, validation in Python);
// here a failure leaves `dst` untouched and is reported by bgl_last_error().
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace bgl {
namespace {

// A device allocation freed on scope exit (this layer owns its staging).
struct DevBuf {
    void *p = nullptr;
    cudaError_t err = cudaSuccess;
    explicit DevBuf(size_t bytes) {
        if (bytes) err = cudaMalloc(&p, bytes);
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    template <typename T>
    T *as() const {
        return static_cast<T *>(p);
    }
};

#define STAGE(name, bytes)                                                                  \
    DevBuf name{static_cast<size_t>(bytes)};                                                \
    if (name.err != cudaSuccess)                                                            \
        return fail(BGL_E_CUDA, "staging %s: %s", #name, cudaGetErrorString(name.err));

inline const double *hf(int64_t a) { return reinterpret_cast<const double *>(static_cast<uintptr_t>(a)); }
inline double *hfm(int64_t a) { return reinterpret_cast<double *>(static_cast<uintptr_t>(a)); }
inline const int64_t *hi(int64_t a) { return reinterpret_cast<const int64_t *>(static_cast<uintptr_t>(a)); }
inline int64_t *him(int64_t a) { return reinterpret_cast<int64_t *>(static_cast<uintptr_t>(a)); }

int h2d(void *dst, const void *src, size_t bytes) {
    if (bytes) BGL_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return BGL_OK;
}
int d2h(void *dst, const void *src, size_t bytes) {
    if (bytes) BGL_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return BGL_OK;
}

int64_t max_plus_one(const int64_t *a, int64_t n) {
    int64_t m = -1;
    for (int64_t i = 0; i < n; ++i) m = std::max(m, a[i]);
    return m + 1;
}

// int64 host ids -> int32 device ids.
int upload_ids(int32_t *dst, const int64_t *src, int64_t n) {
    std::vector<int32_t> tmp(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) tmp[i] = static_cast<int32_t>(src[i]);
    return h2d(dst, tmp.data(), size_t(n) * sizeof(int32_t));
}

#define TRY(x)            \
    do {                  \
        int rc_ = (x);    \
        if (rc_) return rc_; \
    } while (0)

int gspmm_host(int64_t indptr, int64_t indices, int64_t eid, int64_t lhs, int64_t rhs, int64_t dst,
               int64_t num_dst, int64_t op, int64_t dl, int64_t dr, int64_t dout,
               int64_t reduce_op, int64_t deg) {
    if (num_dst <= 0 || dout <= 0) return BGL_OK;
    const int64_t ne = hi(indptr)[num_dst];
    const bool need_l = op != BGL_OP_COPY_RHS, need_r = op != BGL_OP_COPY_LHS;
    const int64_t nl = need_l ? max_plus_one(hi(indices), ne) : 0;
    const int64_t nr = need_r ? max_plus_one(hi(eid), ne) : 0;
    STAGE(d_indptr, size_t(num_dst + 1) * 8);
    STAGE(d_indices, size_t(ne) * 4);
    STAGE(d_eid, size_t(ne) * 4);
    STAGE(d_deg, size_t(num_dst) * 8);
    STAGE(d_lhs, size_t(std::max<int64_t>(nl, 0)) * dl * 8);
    STAGE(d_rhs, size_t(std::max<int64_t>(nr, 0)) * dr * 8);
    STAGE(d_out, size_t(num_dst) * dout * 8);
    size_t wsb = bgl_gspmm_workspace_size(num_dst, ne, dout, BGL_F64, (int)reduce_op);
    STAGE(d_ws, wsb);
    TRY(h2d(d_indptr.p, hi(indptr), size_t(num_dst + 1) * 8));
    TRY(upload_ids(d_indices.as<int32_t>(), hi(indices), ne));
    TRY(upload_ids(d_eid.as<int32_t>(), hi(eid), ne));
    TRY(h2d(d_deg.p, hi(deg), size_t(num_dst) * 8));
    if (need_l) TRY(h2d(d_lhs.p, hf(lhs), size_t(nl) * dl * 8));
    if (need_r) TRY(h2d(d_rhs.p, hf(rhs), size_t(nr) * dr * 8));
    TRY(bgl_gspmm(d_indptr.as<int64_t>(), d_indices.as<int32_t>(), d_eid.as<int32_t>(),
                  d_deg.as<int64_t>(), num_dst, ne, d_lhs.p, dl, 1, d_rhs.p, dr, 1, d_out.p, dout,
                  nullptr, nullptr, BGL_F64, (int)op, (int)reduce_op, 0, d_ws.p, wsb, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(hfm(dst), d_out.p, size_t(num_dst) * dout * 8);
}

int gsddmm_host(int64_t uids, int64_t vids, int64_t lhs, int64_t rhs, int64_t dst, int64_t ne,
                int64_t lt, int64_t rt, int64_t op, int64_t dl, int64_t dr, int64_t dout) {
    if (ne <= 0 || dout <= 0) return BGL_OK;
    const bool need_l = op != BGL_OP_COPY_RHS, need_r = op != BGL_OP_COPY_LHS;
    auto rows_of = [&](int64_t tgt) {
        if (tgt == BGL_SRC) return max_plus_one(hi(uids), ne);
        if (tgt == BGL_DST) return max_plus_one(hi(vids), ne);
        return ne;
    };
    const int64_t nl = need_l ? rows_of(lt) : 0, nr = need_r ? rows_of(rt) : 0;
    STAGE(d_u, size_t(ne) * 4);
    STAGE(d_v, size_t(ne) * 4);
    STAGE(d_lhs, size_t(nl) * dl * 8);
    STAGE(d_rhs, size_t(nr) * dr * 8);
    STAGE(d_out, size_t(ne) * dout * 8);
    TRY(upload_ids(d_u.as<int32_t>(), hi(uids), ne));
    TRY(upload_ids(d_v.as<int32_t>(), hi(vids), ne));
    if (need_l) TRY(h2d(d_lhs.p, hf(lhs), size_t(nl) * dl * 8));
    if (need_r) TRY(h2d(d_rhs.p, hf(rhs), size_t(nr) * dr * 8));
    if (op == BGL_OP_DOT)
        TRY(bgl_gsddmm(d_u.as<int32_t>(), d_v.as<int32_t>(), ne, d_lhs.p, dl, 1, (int)lt, d_rhs.p,
                       dr, 1, (int)rt, d_out.p, 1, dl, BGL_F64, (int)op, nullptr));
    else
        TRY(bgl_gsddmm(d_u.as<int32_t>(), d_v.as<int32_t>(), ne, d_lhs.p, dl, 1, (int)lt, d_rhs.p,
                       dr, 1, (int)rt, d_out.p, dout, 0, BGL_F64, (int)op, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(hfm(dst), d_out.p, size_t(ne) * dout * 8);
}

// The reference's segment kernels clamp every segment into [0, n]
// independently (src/ported.mojo:599-607, 694-699).  A monotone in-range
// offsets array is used as is; anything else is turned into an explicit CSR
// over the clamped ranges, which reproduces the clamping exactly.
struct SegCsr {
    std::vector<int64_t> indptr;
    std::vector<int32_t> ids;
    bool identity = true;
};

SegCsr segment_csr(const int64_t *offsets, int64_t num_seg, int64_t n) {
    SegCsr c;
    bool ok = offsets[0] >= 0;
    for (int64_t s = 0; s < num_seg && ok; ++s)
        ok = offsets[s + 1] >= offsets[s] && offsets[s + 1] <= n;
    c.indptr.resize(size_t(num_seg + 1));
    if (ok) {
        std::memcpy(c.indptr.data(), offsets, size_t(num_seg + 1) * 8);
        return c;
    }
    c.identity = false;
    c.indptr[0] = 0;
    for (int64_t s = 0; s < num_seg; ++s) {
        int64_t a = std::max<int64_t>(offsets[s], 0), b = std::min(offsets[s + 1], n);
        if (b < a) b = a;
        for (int64_t i = a; i < b; ++i) c.ids.push_back(static_cast<int32_t>(i));
        c.indptr[s + 1] = c.indptr[s] + (b - a);
    }
    return c;
}

int segment_reduce_host(int64_t offsets, int64_t value, int64_t dst, int64_t num_seg, int64_t d,
                        int64_t reduce_op, int64_t n) {
    if (num_seg <= 0 || d <= 0) return BGL_OK;
    SegCsr c = segment_csr(hi(offsets), num_seg, n);
    const int64_t ne = c.indptr[num_seg];
    STAGE(d_indptr, size_t(num_seg + 1) * 8);
    STAGE(d_ids, c.ids.size() * 4);
    STAGE(d_val, size_t(n) * d * 8);
    STAGE(d_out, size_t(num_seg) * d * 8);
    size_t wsb = bgl_gspmm_workspace_size(num_seg, ne, d, BGL_F64, (int)reduce_op);
    STAGE(d_ws, wsb);
    TRY(h2d(d_indptr.p, c.indptr.data(), size_t(num_seg + 1) * 8));
    TRY(h2d(d_ids.p, c.ids.data(), c.ids.size() * 4));
    TRY(h2d(d_val.p, hf(value), size_t(n) * d * 8));
    TRY(bgl_gspmm(d_indptr.as<int64_t>(), nullptr, c.identity ? nullptr : d_ids.as<int32_t>(),
                  nullptr, num_seg, ne, nullptr, 1, 1, d_val.p, d, 1, d_out.p, d, nullptr, nullptr,
                  BGL_F64, BGL_OP_COPY_RHS, (int)reduce_op, 0, d_ws.p, wsb, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(hfm(dst), d_out.p, size_t(num_seg) * d * 8);
}

// Shared by segment_softmax and edge_softmax: rows of a CSR whose items index
// `logits`/`dst` rows [0, rows); `dst` is round-tripped so rows the kernel does
// not write keep the caller's contents, as in the reference.
int softmax_host(const std::vector<int64_t> &indptr, const int32_t *ids, int64_t n_ids,
                 const int8_t *mask, int64_t mask_len, int64_t num_rows, int64_t logits,
                 int64_t dst, int64_t rows, int64_t d) {
    STAGE(d_indptr, size_t(num_rows + 1) * 8);
    STAGE(d_ids, size_t(n_ids) * 4);
    STAGE(d_mask, size_t(mask_len));
    STAGE(d_log, size_t(rows) * d * 8);
    STAGE(d_out, size_t(rows) * d * 8);
    TRY(h2d(d_indptr.p, indptr.data(), size_t(num_rows + 1) * 8));
    if (ids) TRY(h2d(d_ids.p, ids, size_t(n_ids) * 4));
    if (mask) TRY(h2d(d_mask.p, mask, size_t(mask_len)));
    TRY(h2d(d_log.p, hf(logits), size_t(rows) * d * 8));
    TRY(h2d(d_out.p, hf(dst), size_t(rows) * d * 8));
    const int64_t items = indptr[num_rows];  // every row's items lie in [0, items)
    const size_t wsb = bgl_softmax_workspace_size(num_rows, items, d, BGL_F64);
    STAGE(d_ws, wsb);
    TRY(bgl_edge_softmax(d_indptr.as<int64_t>(), ids ? d_ids.as<int32_t>() : nullptr,
                         mask ? d_mask.as<int8_t>() : nullptr, num_rows, items, d_log.p, d_out.p,
                         d, BGL_F64, d_ws.p, wsb, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(hfm(dst), d_out.p, size_t(rows) * d * 8);
}

int segment_softmax_host(int64_t offsets, int64_t value, int64_t dst, int64_t num_seg, int64_t d,
                         int64_t n) {
    if (num_seg <= 0 || d <= 0 || n <= 0) return BGL_OK;
    SegCsr c = segment_csr(hi(offsets), num_seg, n);
    return softmax_host(c.indptr, c.identity ? nullptr : c.ids.data(), (int64_t)c.ids.size(),
                        nullptr, 0, num_seg, value, dst, n, d);
}

int edge_softmax_host(int64_t indptr, int64_t eid, int64_t mask, int64_t logits, int64_t dst,
                      int64_t num_nodes, int64_t all_ones, int64_t d) {
    if (num_nodes <= 0 || d <= 0) return BGL_OK;
    const int64_t *ip = hi(indptr);
    const int64_t ne = ip[num_nodes];
    if (ne <= 0) return BGL_OK;
    std::vector<int64_t> ptr(ip, ip + num_nodes + 1);
    std::vector<int32_t> ids(static_cast<size_t>(ne));
    int64_t rows = 0;
    for (int64_t i = 0; i < ne; ++i) {
        ids[i] = static_cast<int32_t>(hi(eid)[i]);
        rows = std::max(rows, hi(eid)[i] + 1);
    }
    const int8_t *m = all_ones == 1 ? nullptr
                                    : reinterpret_cast<const int8_t *>(static_cast<uintptr_t>(mask));
    return softmax_host(ptr, ids.data(), ne, m, m ? rows : 0, num_nodes, logits, dst, rows, d);
}

int segment_mm_host(int64_t a, int64_t b, int64_t dst, int64_t seglen_a, int64_t n, int64_t d1,
                    int64_t r, int64_t d2) {
    if (n <= 0 || d2 <= 0 || r <= 0) return BGL_OK;
    int64_t total = 0;
    for (int64_t i = 0; i < r; ++i) total += hi(seglen_a)[i];
    if (total > n) return fail(BGL_E_INVALID, "mdgl_segment_mm: segment lengths overrun n");
    STAGE(d_a, size_t(n) * d1 * 8);
    STAGE(d_b, size_t(r) * d1 * d2 * 8);
    STAGE(d_out, size_t(n) * d2 * 8);
    STAGE(d_len, size_t(r) * 8);
    size_t wsb = bgl_segment_mm_workspace_size(n, d1, r, d2, BGL_F64);
    STAGE(d_ws, wsb);
    TRY(h2d(d_a.p, hf(a), size_t(n) * d1 * 8));
    TRY(h2d(d_b.p, hf(b), size_t(r) * d1 * d2 * 8));
    TRY(h2d(d_len.p, hi(seglen_a), size_t(r) * 8));
    TRY(bgl_segment_mm(d_a.p, d_b.p, d_out.p, d_len.as<int64_t>(), n, d1, r, d2, BGL_F64, d_ws.p,
                       wsb, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    // rows past the segments are the caller's, as in the reference kernel
    return d2h(hfm(dst), d_out.p, size_t(total) * d2 * 8);
}

int gather_mm_host(int64_t a, int64_t b, int64_t idx_b, int64_t dst, int64_t n, int64_t d1,
                   int64_t d2) {
    if (n <= 0 || d2 <= 0) return BGL_OK;
    const int64_t r = max_plus_one(hi(idx_b), n);
    STAGE(d_a, size_t(n) * d1 * 8);
    STAGE(d_b, size_t(r) * d1 * d2 * 8);
    STAGE(d_idx, size_t(n) * 8);
    STAGE(d_out, size_t(n) * d2 * 8);
    size_t wsb = bgl_gather_mm_workspace_size(n, d1, r, d2, BGL_F64);
    STAGE(d_ws, wsb);
    TRY(h2d(d_a.p, hf(a), size_t(n) * d1 * 8));
    TRY(h2d(d_b.p, hf(b), size_t(r) * d1 * d2 * 8));
    TRY(h2d(d_idx.p, hi(idx_b), size_t(n) * 8));
    TRY(bgl_gather_mm(d_a.p, d_b.p, d_idx.as<int64_t>(), d_out.p, n, d1, r, d2, BGL_F64, d_ws.p,
                      wsb, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(hfm(dst), d_out.p, size_t(n) * d2 * 8);
}

int cumsum_host(int64_t src, int64_t dst, int64_t n) {
    if (n <= 0) return BGL_OK;
    STAGE(d_src, size_t(n) * 8);
    STAGE(d_dst, size_t(n) * 8);
    size_t wsb = bgl_cumsum_workspace_size(n);
    STAGE(d_ws, wsb);
    TRY(h2d(d_src.p, hi(src), size_t(n) * 8));
    TRY(bgl_cumsum_i64(d_src.as<int64_t>(), d_dst.as<int64_t>(), n, d_ws.p, wsb, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(him(dst), d_dst.p, size_t(n) * 8);
}

int clamp_host(int64_t src, int64_t dst, int64_t n, int64_t lo, int64_t hi_) {
    if (n <= 0) return BGL_OK;
    STAGE(d_src, size_t(n) * 8);
    STAGE(d_dst, size_t(n) * 8);
    TRY(h2d(d_src.p, hi(src), size_t(n) * 8));
    TRY(bgl_clamp_i64(d_src.as<int64_t>(), d_dst.as<int64_t>(), n, lo, hi_, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(him(dst), d_dst.p, size_t(n) * 8);
}

int riwz_host(int64_t src, int64_t dst, int64_t n) {
    if (n <= 0) return BGL_OK;
    STAGE(d_src, size_t(n) * 8);
    STAGE(d_dst, size_t(n) * 8);
    TRY(h2d(d_src.p, hf(src), size_t(n) * 8));
    TRY(bgl_replace_inf_with_zero(d_src.p, d_dst.p, n, BGL_F64, nullptr));
    BGL_CUDA(cudaDeviceSynchronize());
    return d2h(hfm(dst), d_dst.p, size_t(n) * 8);
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

int64_t mdgl_workers(void) { return 32; }  // src/capi.mojo:48-50; sizes the caller's scratch

void mdgl_cumsum(int64_t src, int64_t dst, int64_t n) {
    if (cumsum_host(src, dst, n) == BGL_OK) clear_error();
}

void mdgl_replace_inf_with_zero(int64_t src, int64_t dst, int64_t n) {
    if (riwz_host(src, dst, n) == BGL_OK) clear_error();
}

void mdgl_clamp_i64(int64_t src, int64_t dst, int64_t n, int64_t lo, int64_t hi) {
    if (clamp_host(src, dst, n, lo, hi) == BGL_OK) clear_error();
}

void mdgl_gsddmm(int64_t uids, int64_t vids, int64_t lhs, int64_t rhs, int64_t dst,
                 int64_t num_edges, int64_t lhs_target, int64_t rhs_target, int64_t op, int64_t dl,
                 int64_t dr, int64_t dout) {
    if (gsddmm_host(uids, vids, lhs, rhs, dst, num_edges, lhs_target, rhs_target, op, dl, dr,
                    dout) == BGL_OK)
        clear_error();
}

void mdgl_gspmm(int64_t indptr, int64_t indices, int64_t eid, int64_t lhs, int64_t rhs,
                int64_t dst, int64_t num_dst, int64_t op, int64_t dl, int64_t dr, int64_t dout,
                int64_t reduce_op, int64_t deg) {
    if (gspmm_host(indptr, indices, eid, lhs, rhs, dst, num_dst, op, dl, dr, dout, reduce_op,
                   deg) == BGL_OK)
        clear_error();
}

void mdgl_segment_reduce(int64_t offsets, int64_t value, int64_t dst, int64_t num_seg, int64_t d,
                         int64_t reduce_op, int64_t n) {
    if (segment_reduce_host(offsets, value, dst, num_seg, d, reduce_op, n) == BGL_OK)
        clear_error();
}

void mdgl_segment_softmax(int64_t offsets, int64_t value, int64_t dst, int64_t scratch,
                          int64_t num_seg, int64_t d, int64_t n) {
    (void)scratch;  // the device kernel keeps its running max/sum in registers
    if (segment_softmax_host(offsets, value, dst, num_seg, d, n) == BGL_OK) clear_error();
}

void mdgl_segment_mm(int64_t a, int64_t b, int64_t dst, int64_t seglen_a, int64_t n, int64_t d1,
                     int64_t r, int64_t d2) {
    if (segment_mm_host(a, b, dst, seglen_a, n, d1, r, d2) == BGL_OK) clear_error();
}

void mdgl_edge_softmax_(int64_t indptr, int64_t indices, int64_t eid, int64_t mask,
                        int64_t logits, int64_t dst, int64_t scratch, int64_t num_nodes,
                        int64_t all_ones, int64_t d) {
    (void)indices;
    (void)scratch;
    if (edge_softmax_host(indptr, eid, mask, logits, dst, num_nodes, all_ones, d) == BGL_OK)
        clear_error();
}

void mdgl_gather_mm(int64_t a, int64_t b, int64_t idx_b, int64_t dst, int64_t n, int64_t d1,
                    int64_t d2) {
    if (gather_mm_host(a, b, idx_b, dst, n, d1, d2) == BGL_OK) clear_error();
}

}  // extern "C"
