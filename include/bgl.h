/*
 * bgl.h -- C ABI of libbgl.so, the B200 (sm_100a) kernels behind mojodgl's
 * message-passing hot path.
 *
 * Two layers, both plain C (pointers and sizes, no framework types):
 *
 *  1. The reference-compatible layer: the eleven `mdgl_*` symbols of
 *     lee101/mojo-dgl's src/capi.mojo, same names, same all-int64 argument
 *     lists, same host float64 buffers, same `void` return.  Each call stages
 *     its host arrays to the current CUDA device, runs the float64 kernels and
 *     copies the result back before returning, so the reference's own Python
 *     package (python/mojodgl/_lib.py, MOJODGL_LIB=libbgl.so) runs on the GPU
 *     unchanged.  As in the reference these have no error channel; a failure
 *     is recorded for bgl_last_error() and the destination is left unwritten.
 *
 *  2. The native layer: `bgl_*` entry points taking DEVICE pointers, a dtype
 *     code, an explicit workspace the caller allocates (the library never
 *     allocates on this layer, as the reference never does:
 *     src/capi.mojo:5-7) and a cudaStream_t passed as `void*`.  Each returns
 *     an int status (BGL_OK = 0) and never synchronises the device.  Device
 *     graph arrays use int64 row pointers and int32 column/edge ids.
 *
 *     Precondition on the native layer, as on the reference's (whose kernels
 *     do no bounds checks either: python/mojodgl validates before each call):
 *     every id a kernel gathers through must be in range -- gspmm/gat
 *     `indices` below the lhs operand's row count and `eid` below the rhs
 *     operand's, gsddmm `u`/`v` below their operands' row counts, row
 *     pointers non-decreasing from 0 to num_edges.  The kernels read device
 *     arrays and do not check ids against sizes they are not given; an id out
 *     of range reads outside the operand.  The Python layer (mojodgl) checks
 *     node ids when a graph is built, bgl_csr_build only produces ids in
 *     range, and bgl_check_csr checks a CSR from elsewhere on the device.
 *
 * Op, reduce and target codes are the reference's (src/ported.mojo:44-65,
 * python/mojodgl/_lib.py:66-73).
 */
#ifndef BGL_H
#define BGL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* every declaration below is an exported symbol of libbgl.so */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ------------------------------------------------------------------ codes */
enum {
    BGL_OK = 0,
    BGL_E_INVALID = 1,     /* bad argument (shape, code, alignment, size) */
    BGL_E_CUDA = 2,        /* a CUDA runtime call failed */
    BGL_E_UNSUPPORTED = 3, /* valid request this build does not implement */
    BGL_E_WORKSPACE = 4    /* workspace smaller than the *_workspace_size query */
};
enum { BGL_F32 = 0, BGL_F64 = 1, BGL_BF16 = 2 };
enum { BGL_SRC = 0, BGL_DST = 1, BGL_EDGE = 2 };
enum {
    BGL_OP_ADD = 0, BGL_OP_SUB = 1, BGL_OP_MUL = 2, BGL_OP_DIV = 3, BGL_OP_DOT = 4,
    BGL_OP_COPY_LHS = 5, BGL_OP_COPY_RHS = 6
};
enum { BGL_RED_SUM = 0, BGL_RED_MAX = 1, BGL_RED_MIN = 2, BGL_RED_MEAN = 3 };
/* gspmm flags */
enum {
    BGL_ZERO_INF = 1,  /* replace +-inf results with 0 (the max/min post-pass of
                          python/mojodgl/heterograph.py:232-239 and
                          python/mojodgl/ops/segment.py:106-110, fused) */
    BGL_ACCUMULATE = 2 /* fold each row into what out (and arg_e) already hold:
                          sums add; max/min keep the better value, a tie going
                          to the smaller edge id.  Lets one aggregation run as
                          several passes over disjoint edge subsets (e.g. per
                          source-owner block as blocks arrive); the mean divide
                          and ZERO_INF belong on the last pass only */
};

/* ------------------------------------------------------------- utilities */
/* Message of the last failed call on this host thread ("" if none). */
const char *bgl_last_error(void);
/* ABI revision of this header. */
int bgl_abi_version(void);
/* Tuning knobs for tests and benchmarks: "spmm_min_items" (merge-path chunk
 * floor), "spmm_max_chunks" (cap on merge-path chunks; 0 = automatic),
 * "spmm_split_min" (rows with at most this many edges are never split across
 * chunks; default 512), "softmax_segment_warp" (bgl_edge_softmax with eid =
 * NULL, i.e. segment_softmax: 1 = one warp per segment, each segment read
 * once from DRAM, 0 = the merge-path passes; default 1).
 * Returns BGL_OK or BGL_E_INVALID for an unknown name. */
int bgl_set_param(const char *name, int64_t value);

/* ------------------------------------------------------------- CSR build */
/* Replaces python/mojodgl/heterograph.py:69-86 (_build_csr): for the in-CSR
 * pass key = v, other = u; for the out-CSR key = u, other = v.  Produces
 *   deg[n]        = bincount(key)               (int64)
 *   indptr[n + 1] = [0, cumsum(deg)]            (int64)
 *   order[e]      = argsort(key, kind="stable") (int32, the CSR's edge ids)
 *   indices[e]    = other[order]                (int32)
 * bit-identical to numpy.  key/other are int64 node ids in [0, n). */
size_t bgl_csr_build_workspace_size(int64_t num_edges, int64_t num_nodes);
int bgl_csr_build(const int64_t *key, const int64_t *other, int64_t num_edges,
                  int64_t num_nodes, int64_t *indptr, int64_t *deg, int32_t *order,
                  int32_t *indices, void *workspace, size_t workspace_bytes, void *stream);
/* Checks a CSR against the precondition of the native layer (no counterpart
 * in the reference, whose Python layer validates before each call): on the
 * stream, result[0] = the number of bad row pointers (indptr[0] != 0, a
 * decrease, indptr[num_rows] != num_edges), result[1] = the number of bad ids
 * (indices outside [0, num_src), eid outside [0, num_eid); either array may be
 * NULL), result[2] = the smallest CSR position holding a bad id, -1 if none.
 * `result` is a DEVICE int64[3]; read it after the stream reaches this call.
 * Only the given arrays are read, within the sizes given. */
int bgl_check_csr(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
                  int64_t num_rows, int64_t num_edges, int64_t num_src, int64_t num_eid,
                  int64_t *result, void *stream);
/* int64 -> int32 narrowing copy (edge endpoint arrays for gsddmm). */
int bgl_narrow_i64(const int64_t *src, int32_t *dst, int64_t n, void *stream);

/* ---------------------------------------------------------------- gspmm */
/* Replaces mdgl_gspmm (src/capi.mojo:95-115 -> src/ported.mojo:352-548):
 *   out[v, k] = RED_{i in [indptr[v], indptr[v+1])} op(lhs[indices[i], .], rhs[eid[i], .])
 * with the reference's identities for empty rows (0, -inf, +inf), `mean` =
 * sum / max(deg, 1), and per-column sequential CSR-order accumulation for
 * every row no longer than the merge-path chunk (longer rows are split and
 * their pieces folded in CSR order).
 * Operand broadcast: output column k reads column (k / div) % width of its
 * operand row, whose stride is `width` (full: width = dout, div = 1; a (n, 1)
 * column: width = 1; DGL's head broadcast (n, H, 1) against (.., H, D):
 * width = H, div = D).
 * eid == NULL means the identity (eid[i] = i); indices may be NULL for
 * copy_rhs; deg == NULL means indptr differences.  arg_u/arg_e (nullable,
 * int64, num_rows x dout) receive, for max/min, the source node id / edge id
 * of the first strictly-best message in CSR order, -1 for empty rows. */
size_t bgl_gspmm_workspace_size(int64_t num_rows, int64_t num_edges, int64_t dout, int dtype,
                                int reduce);
int bgl_gspmm(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
              const int64_t *deg, int64_t num_rows, int64_t num_edges, const void *lhs,
              int64_t lhs_width, int64_t lhs_div, const void *rhs, int64_t rhs_width,
              int64_t rhs_div, void *out, int64_t dout, int64_t *arg_u, int64_t *arg_e,
              int dtype, int op, int reduce, int flags, void *workspace, size_t workspace_bytes,
              void *stream);

/* gSpMM without a caller workspace.  No counterpart in the reference: it is
 * for callers that cannot allocate device memory (a plugin or serving runtime
 * that hands the library only its input and output buffers, or a request path
 * where cudaMalloc, which may synchronise the device, is not allowed).  Same
 * arguments and results as bgl_gspmm; the scratch is a fixed 64 MiB device
 * array inside the library (bgl_static_scratch_bytes()), held by every GPU
 * that loads it until exit.  Calls needing more than that fail with
 * BGL_E_INVALID.  All calls on a device share the array, so calls that may
 * overlap on the GPU race and must be serialised by the caller.  The array's
 * address is resolved (cudaGetSymbolAddress) for each CUDA context the first
 * time a call runs in it -- the device's primary context or one the caller
 * made current -- so make that first call before any stream capture.
 * Allocates nothing. */
size_t bgl_static_scratch_bytes(void);
int bgl_gspmm_static_scratch(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
                             const int64_t *deg, int64_t num_rows, int64_t num_edges,
                             const void *lhs, int64_t lhs_width, int64_t lhs_div, const void *rhs,
                             int64_t rhs_width, int64_t rhs_div, void *out, int64_t dout,
                             int64_t *arg_u, int64_t *arg_e, int dtype, int op, int reduce,
                             int flags, void *stream);

/* --------------------------------------------------------------- gsddmm */
/* Replaces mdgl_gsddmm (src/capi.mojo:70-91 -> src/ported.mojo:204-329):
 *   out[e, k] = op(lhs[T_l(e), .], rhs[T_r(e), .]),  T = u[e] | v[e] | e
 * Broadcast descriptors as for gspmm.  For op == DOT: lhs and rhs rows are
 * `red_len` wide (no broadcast) and out[e] = sum_k lhs * rhs (dout = 1). */
int bgl_gsddmm(const int32_t *u, const int32_t *v, int64_t num_edges, const void *lhs,
               int64_t lhs_width, int64_t lhs_div, int lhs_target, const void *rhs,
               int64_t rhs_width, int64_t rhs_div, int rhs_target, void *out, int64_t dout,
               int64_t red_len, int dtype, int op, void *stream);

/* -------------------------------------------------------- fused softmax */
/* Replaces mdgl_edge_softmax_ (src/capi.mojo:149-165 -> src/ported.mojo:876-1080)
 * and mdgl_segment_softmax (src/capi.mojo:132-138 -> src/ported.mojo:660-768):
 * per CSR row and per column h < d, over the row's edges e = eid[i] (eid NULL:
 * e = i) that `mask` selects (mask NULL: all),
 *   out[e, h] = exp(logits[e, h] - max) / sum exp(logits[., h] - max).
 * Rows with no selected edge write nothing.  indptr must be non-decreasing
 * with indptr[0] = 0 and indptr[num_rows] = num_items (the compat layer turns
 * the reference's clamped offsets, src/ported.mojo:694-699, into such a CSR).
 * Heavy rows are split over merge-path chunks; the workspace holds the chunk
 * boundaries, the split rows' per-column (max, sum) pieces, every row's
 * (max, 1 / sum) and every item's row. */
size_t bgl_softmax_workspace_size(int64_t num_rows, int64_t num_items, int64_t d, int dtype);
int bgl_edge_softmax(const int64_t *indptr, const int32_t *eid, const int8_t *mask,
                     int64_t num_rows, int64_t num_items, const void *logits, void *out,
                     int64_t d, int dtype, void *workspace, size_t workspace_bytes,
                     void *stream);
/* bgl_edge_softmax over every edge (no mask), given the row of every edge by
 * edge id (edge_row[e]: the destination of edge e for norm_by "dst", its
 * source for "src"; eid must permute [0, num_items)).  With it the output
 * pass runs in edge order -- logits read and outputs written contiguously --
 * for rows of up to 8 column vectors.  Same workspace as bgl_edge_softmax. */
int bgl_edge_softmax_by_edge(const int64_t *indptr, const int32_t *eid, const int32_t *edge_row,
                             int64_t num_rows, int64_t num_items, const void *logits, void *out,
                             int64_t d, int dtype, void *workspace, size_t workspace_bytes,
                             void *stream);

/* ------------------------------------------------ fused GAT aggregation */
/* One pass for the chain the reference runs as four operators on a GAT layer
 * (python/mojodgl/ops/sddmm.py u_add_v -> the caller's leaky_relu ->
 * ops/edge_softmax.py norm_by="dst" -> ops/spmm.py u_mul_e_sum; kernels at
 * src/ported.mojo:204-329, 876-1080, 352-423):
 *   s_e = leaky_relu(el[u_e, h] + er[v, h], negative_slope)
 *   out[v, h, :] = sum_{e -> v} softmax_{e -> v}(s_e) * feat[u_e, h, :]
 * over the in-CSR (indptr, indices = source ids).  feat is (sources, heads *
 * head_dim), el (sources, heads), er (num_rows, heads), out (num_rows, heads *
 * head_dim), all C-contiguous; rows without in-edges get 0.  No per-edge
 * score or attention array is written.  Rounding differs from the unfused
 * chain (rescaled running sums, one divide). */
size_t bgl_gat_workspace_size(int64_t num_rows, int64_t num_edges, int64_t heads, int64_t head_dim,
                              int dtype);
int bgl_gat_aggregate(const int64_t *indptr, const int32_t *indices, int64_t num_rows,
                      int64_t num_edges, const void *feat, const void *el, const void *er,
                      int64_t heads, int64_t head_dim, double negative_slope, void *out, int dtype,
                      void *workspace, size_t workspace_bytes, void *stream);

/* --------------------------------------------------------- segment_mm */
/* Replaces mdgl_segment_mm (src/capi.mojo:141-145 -> src/ported.mojo:773-804):
 * out[rows of segment r] = a[rows] @ b[r]; rows past sum(seglen) are zeroed.
 * seglen is a DEVICE int64 array of r entries.  fp32 runs on the tcgen05
 * tensor cores in TF32 (kind::tf32), bf16 in kind::f16 with fp32
 * accumulation, fp64 on a SIMT kernel. */
size_t bgl_segment_mm_workspace_size(int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype);
int bgl_segment_mm(const void *a, const void *b, void *out, const int64_t *seglen, int64_t n,
                   int64_t d1, int64_t r, int64_t d2, int dtype, void *workspace,
                   size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------- gather_mm */
/* Replaces mdgl_gather_mm (src/capi.mojo:169-173 -> src/ported.mojo:1089-1130)
 * and the sort -> segment_mm -> unsort route of python/mojodgl/ops/gather_mm.py:79-87:
 * out[i] = a[i] @ b[idx_b[i]].  Rows are grouped by a stable sort on idx_b
 * on the device and fed to the grouped GEMM with gathered A rows and
 * scattered output rows; both of the reference's routes give this result. */
size_t bgl_gather_mm_workspace_size(int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype);
int bgl_gather_mm(const void *a, const void *b, const int64_t *idx_b, void *out, int64_t n,
                  int64_t d1, int64_t r, int64_t d2, int dtype, void *workspace,
                  size_t workspace_bytes, void *stream);

/* Device-side status of the tensor-core grouped GEMM: 0, or the code of the
 * first bounded wait that expired (1-4) since the last call; synchronises
 * the device and clears the word. */
int bgl_tc_error(void);

/* ------------------------------------------------ multi-GPU halo buffers */
/* Device buffers shared between the processes of one node (one process per
 * GPU) through CUDA IPC, and copies between them run by the copy engines:
 * the multi-GPU gSpMM pulls its peers' feature blocks over NVLink this way,
 * so the transfer overlaps the aggregation without taking SMs.  Not part of
 * the reference's interface (its gSpMM runs in one process,
 * src/ported.mojo:442-443).  Every entry point checks its byte range against
 * the allocation that holds it and rejects a range that leaves it. */
enum { BGL_IPC_HANDLE_BYTES = 64 };
/* handle (BGL_IPC_HANDLE_BYTES) and offset of [ptr, ptr + bytes) within its
 * allocation, for bgl_ipc_open in another process */
int bgl_ipc_export(const void *ptr, int64_t bytes, void *handle, int64_t *offset);
/* maps another process's exported allocation into the current device's
 * context (peer access enabled on demand); *ptr = mapping + offset */
int bgl_ipc_open(const void *handle, int64_t offset, int64_t bytes, void **ptr);
/* unmaps what bgl_ipc_open mapped (any pointer inside the mapping) */
int bgl_ipc_close(void *ptr);
/* queues a copy-engine copy of `bytes` from src to dst on `stream`; either
 * side may be a peer mapping */
int bgl_peer_copy(void *dst, const void *src, int64_t bytes, void *stream);

/* ------------------------------------------------------- array primitives */
/* src/ported.mojo:145-190 */
size_t bgl_cumsum_workspace_size(int64_t n);
int bgl_cumsum_i64(const int64_t *src, int64_t *dst, int64_t n, void *workspace,
                   size_t workspace_bytes, void *stream);
int bgl_clamp_i64(const int64_t *src, int64_t *dst, int64_t n, int64_t lo, int64_t hi,
                  void *stream);
int bgl_replace_inf_with_zero(const void *src, void *dst, int64_t n, int dtype, void *stream);

/* ------------------------------------------- reference-compatible layer */
/* src/capi.mojo:48-173, one for one. */
int64_t mdgl_workers(void);
void mdgl_cumsum(int64_t src, int64_t dst, int64_t n);
void mdgl_replace_inf_with_zero(int64_t src, int64_t dst, int64_t n);
void mdgl_clamp_i64(int64_t src, int64_t dst, int64_t n, int64_t lo, int64_t hi);
void mdgl_gsddmm(int64_t uids, int64_t vids, int64_t lhs, int64_t rhs, int64_t dst,
                 int64_t num_edges, int64_t lhs_target, int64_t rhs_target, int64_t op,
                 int64_t dl, int64_t dr, int64_t dout);
void mdgl_gspmm(int64_t indptr, int64_t indices, int64_t eid, int64_t lhs, int64_t rhs,
                int64_t dst, int64_t num_dst, int64_t op, int64_t dl, int64_t dr, int64_t dout,
                int64_t reduce_op, int64_t deg);
void mdgl_segment_reduce(int64_t offsets, int64_t value, int64_t dst, int64_t num_seg, int64_t d,
                         int64_t reduce_op, int64_t n);
void mdgl_segment_softmax(int64_t offsets, int64_t value, int64_t dst, int64_t scratch,
                          int64_t num_seg, int64_t d, int64_t n);
void mdgl_segment_mm(int64_t a, int64_t b, int64_t dst, int64_t seglen_a, int64_t n, int64_t d1,
                     int64_t r, int64_t d2);
void mdgl_edge_softmax_(int64_t indptr, int64_t indices, int64_t eid, int64_t mask,
                        int64_t logits, int64_t dst, int64_t scratch, int64_t num_nodes,
                        int64_t all_ones, int64_t d);
void mdgl_gather_mm(int64_t a, int64_t b, int64_t idx_b, int64_t dst, int64_t n, int64_t d1,
                    int64_t d2);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* BGL_H */
