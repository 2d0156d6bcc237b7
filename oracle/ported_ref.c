/*
 * TEST INFRASTRUCTURE -- the CPU oracle.  Nothing in the product path links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use it, as the checker and
 * as the timed CPU baseline.
 *
 * A plain-C restatement of the reference's Mojo kernels (src/ported.mojo of
 * lee101/mojo-dgl) exported under the reference's own C ABI (src/capi.mojo:
 * eleven `mdgl_*` symbols, every argument int64, void return).  Because the
 * symbols and signatures are identical, the reference's own Python package can
 * load this library through its MOJODGL_LIB override, which is how the golden
 * fixtures under tests/golden/ are produced.
 *
 * Semantics kept from the reference, with the line each one follows:
 *   - fp64 throughout (ported.mojo:27-32);
 *   - WORKERS = 32 static output-axis split above PARALLEL_MIN = 4096 output
 *     elements (ported.mojo:40-42, 159-167, 221-235, 444-458, 571-581, ...);
 *   - the `vec` flag decided by the ABI layer from the row widths
 *     (capi.mojo:85-87, 111, 129, 137, 145) -- it only changes the summation
 *     order of gsddmm's `dot`, which accumulates W lane partials and then does
 *     one horizontal add (ported.mojo:273-293).  Every other kernel is per
 *     column sequential in either form, so the scalar loops below reproduce the
 *     vector path exactly;
 *   - `acc + x * y` is two roundings, never a fused multiply-add: build with
 *     -ffp-contract=off (oracle/Makefile does).
 *
 * Extension (no counterpart in the reference): oref_gspmm_arg additionally
 * writes, for max/min, the CSR position's edge id and source node id of the
 * winning message, using the reference's own update rule -- the accumulator
 * changes only on a strict improvement (ported.mojo:106-109) -- so the first
 * winner in CSR (ascending edge id) order is reported; -1 for empty rows.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define WORKERS 32      /* ported.mojo:40 */
#define PARALLEL_MIN 4096 /* ported.mojo:42 */
#define W 4             /* simd_width_of[float64] on the reference's AVX2 box */

enum { SRC = 0, DST = 1, EDGE = 2 };                             /* ported.mojo:45-47 */
enum { OP_ADD = 0, OP_SUB, OP_MUL, OP_DIV, OP_DOT, OP_COPY_LHS, OP_COPY_RHS }; /* :50-57 */
enum { RED_SUM = 0, RED_MAX, RED_MIN, RED_MEAN };                 /* ported.mojo:62-65 */

typedef double f64;
typedef int64_t i64;

#define FP(a) ((f64 *)(uintptr_t)(a))
#define IP(a) ((i64 *)(uintptr_t)(a))
#define BP(a) ((int8_t *)(uintptr_t)(a))

/* The 32-worker split of ported.mojo: task t owns [n*t/32, n*(t+1)/32). */
#define SPLIT(n, body)                                                        \
    do {                                                                      \
        if ((n) >= PARALLEL_MIN) {                                            \
            _Pragma("omp parallel for schedule(static)")                      \
            for (int task = 0; task < WORKERS; ++task) {                      \
                i64 lo = (i64)(n) * task / WORKERS;                           \
                i64 hi = (i64)(n) * (task + 1) / WORKERS;                     \
                body;                                                         \
            }                                                                 \
        } else {                                                              \
            int task = 0;                                                     \
            i64 lo = 0, hi = (n);                                             \
            (void)task;                                                       \
            body;                                                             \
        }                                                                     \
    } while (0)

static inline f64 seed_of(int red) {                       /* ported.mojo:76-81 */
    if (red == RED_MAX) return -INFINITY;
    if (red == RED_MIN) return INFINITY;
    return 0.0;
}

static inline f64 message(int op, f64 x, f64 y) {          /* ported.mojo:92-105 */
    switch (op) {
    case OP_ADD: return x + y;
    case OP_SUB: return x - y;
    case OP_MUL: return x * y;
    case OP_DIV: return x / y;
    case OP_COPY_LHS: return x;
    default: return y;
    }
}

/* Mojo's max/min on Float64 (ported.mojo:106-109): the accumulator moves only
 * when the new value is strictly better. */
static inline f64 fmax_ref(f64 a, f64 b) { return b > a ? b : a; }
static inline f64 fmin_ref(f64 a, f64 b) { return b < a ? b : a; }

/* ------------------------------------------------------------ array prims */
/* ported.mojo:145-151 */
void mdgl_cumsum(i64 src, i64 dst, i64 n) {
    i64 acc = 0;
    for (i64 i = 0; i < n; ++i) {
        acc += IP(src)[i];
        IP(dst)[i] = acc;
    }
}

/* ported.mojo:157-177 */
void mdgl_replace_inf_with_zero(i64 src, i64 dst, i64 n) {
    const f64 *s = FP(src);
    f64 *d = FP(dst);
    SPLIT(n, {
        for (i64 i = lo; i < hi; ++i) {
            f64 v = s[i];
            if (v == INFINITY || v == -INFINITY) v = 0.0;
            d[i] = v;
        }
    });
}

/* ported.mojo:181-190 */
void mdgl_clamp_i64(i64 src, i64 dst, i64 n, i64 lo, i64 hi) {
    for (i64 i = 0; i < n; ++i) {
        i64 v = IP(src)[i];
        if (v < lo) v = lo;
        else if (v > hi) v = hi;
        IP(dst)[i] = v;
    }
}

/* ------------------------------------------------------------------ gsddmm */
/* ported.mojo:238-329 */
static void gsddmm_range(const i64 *uids, const i64 *vids, const f64 *lhs, const f64 *rhs,
                         f64 *dst, i64 e0, i64 e1, i64 lt, i64 rt, i64 op, i64 dl,
                         i64 dr, i64 dout, int vec) {
    for (i64 e = e0; e < e1; ++e) {
        i64 li = lt == SRC ? uids[e] * dl : lt == DST ? vids[e] * dl : e * dl;
        i64 ri = rt == SRC ? uids[e] * dr : rt == DST ? vids[e] * dr : e * dr;
        if (op == OP_DOT) {
            /* W lane partials over the vector body, one horizontal add, then
             * the scalar tail (ported.mojo:273-293). */
            f64 p[W] = {0.0, 0.0, 0.0, 0.0};
            i64 k = 0;
            if (vec) {
                for (; k + W <= dl; k += W)
                    for (int j = 0; j < W; ++j) p[j] += lhs[li + k + j] * rhs[ri + k + j];
            }
            f64 acc = 0.0;
            if (vec) acc = (p[0] + p[2]) + (p[1] + p[3]); /* SIMD reduce_add: halves */
            for (; k < dl; ++k) acc += lhs[li + k] * rhs[ri + k];
            dst[e] = acc;
            continue;
        }
        for (i64 d = 0; d < dout; ++d) {
            f64 x = op == OP_COPY_RHS ? 0.0 : lhs[li + d];
            f64 y = op == OP_COPY_LHS ? 0.0 : rhs[ri + d];
            dst[e * dout + d] = message((int)op, x, y);
        }
    }
}

/* capi.mojo:70-91 + ported.mojo:204-235 */
void mdgl_gsddmm(i64 uids, i64 vids, i64 lhs, i64 rhs, i64 dst, i64 num_edges, i64 lhs_target,
                 i64 rhs_target, i64 op, i64 dl, i64 dr, i64 dout) {
    int vec = dl % W == 0 && dr % W == 0;
    if (op != OP_DOT) vec = vec && dout % W == 0;
    SPLIT(num_edges, gsddmm_range(IP(uids), IP(vids), FP(lhs), FP(rhs), FP(dst), lo, hi,
                                  lhs_target, rhs_target, op, dl, dr, dout, vec));
}

/* ------------------------------------------------------------------- gspmm */
/* ported.mojo:352-423.  Per destination row, per column, the messages are
 * folded in CSR order; `mean` divides the sum by max(deg, 1) in the kernel;
 * an empty row keeps the reduce identity. */
static void gspmm_range(const i64 *indptr, const i64 *indices, const i64 *eid, const f64 *lhs,
                        const f64 *rhs, f64 *dst, i64 v0, i64 v1, i64 dl, i64 dr, i64 dout,
                        int op, int red, const i64 *deg, i64 *arg_u, i64 *arg_e) {
    int mean = red == RED_MEAN;
    int kred = mean ? RED_SUM : red;
    for (i64 v = v0; v < v1; ++v) {
        i64 start = indptr[v], stop = indptr[v + 1];
        f64 scale = 1.0;
        if (mean) {
            scale = (f64)deg[v];
            if (scale < 1.0) scale = 1.0;
        }
        for (i64 k = 0; k < dout; ++k) {
            f64 acc = seed_of(kred);
            i64 best = -1;
            for (i64 i = start; i < stop; ++i) {
                /* the operand a copy op does not use is never read: with
                 * copy_lhs the reference passes rhs = lhs (spmm.py:64-66) and
                 * eid can exceed its row count, a load its specialised
                 * kernel drops at compile time */
                f64 x = op == OP_COPY_RHS ? 0.0 : lhs[indices[i] * dl + k];
                f64 y = op == OP_COPY_LHS ? 0.0 : rhs[eid[i] * dr + k];
                f64 m = message(op, x, y);
                if (kred == RED_MAX) {
                    if (m > acc) best = i;
                    acc = fmax_ref(acc, m);
                } else if (kred == RED_MIN) {
                    if (m < acc) best = i;
                    acc = fmin_ref(acc, m);
                } else {
                    acc = acc + m;
                }
            }
            if (mean) acc = acc / scale;
            dst[v * dout + k] = acc;
            if (arg_u) arg_u[v * dout + k] = best < 0 ? -1 : indices[best];
            if (arg_e) arg_e[v * dout + k] = best < 0 ? -1 : eid[best];
        }
    }
}

/* capi.mojo:95-115 + ported.mojo:426-548 */
void mdgl_gspmm(i64 indptr, i64 indices, i64 eid, i64 lhs, i64 rhs, i64 dst, i64 num_dst, i64 op,
                i64 dl, i64 dr, i64 dout, i64 reduce_op, i64 deg) {
    SPLIT(num_dst, gspmm_range(IP(indptr), IP(indices), IP(eid), FP(lhs), FP(rhs), FP(dst), lo,
                               hi, dl, dr, dout, (int)op, (int)reduce_op, IP(deg), 0, 0));
}

/* Extension: the same kernel plus the arg-index outputs (see header). */
void oref_gspmm_arg(i64 indptr, i64 indices, i64 eid, i64 lhs, i64 rhs, i64 dst, i64 num_dst,
                    i64 op, i64 dl, i64 dr, i64 dout, i64 reduce_op, i64 deg, i64 arg_u,
                    i64 arg_e) {
    SPLIT(num_dst, gspmm_range(IP(indptr), IP(indices), IP(eid), FP(lhs), FP(rhs), FP(dst), lo,
                               hi, dl, dr, dout, (int)op, (int)reduce_op, IP(deg), IP(arg_u),
                               IP(arg_e)));
}

/* ---------------------------------------------------------- segment_reduce */
/* ported.mojo:584-647: offsets clamped into [0, n], per column sequential. */
static void seg_reduce_range(const i64 *offsets, const f64 *value, f64 *dst, i64 s0, i64 s1,
                             i64 d, i64 red, i64 n) {
    for (i64 s = s0; s < s1; ++s) {
        i64 start = offsets[s], stop = offsets[s + 1];
        if (start < 0) start = 0;
        if (stop > n) stop = n;
        if (stop < start) stop = start;
        for (i64 k = 0; k < d; ++k) {
            f64 acc = seed_of((int)red);
            for (i64 i = start; i < stop; ++i) {
                f64 x = value[i * d + k];
                if (red == RED_MAX) acc = fmax_ref(acc, x);
                else if (red == RED_MIN) acc = fmin_ref(acc, x);
                else acc += x;
            }
            dst[s * d + k] = acc;
        }
    }
}

/* capi.mojo:119-129 + ported.mojo:559-581 */
void mdgl_segment_reduce(i64 offsets, i64 value, i64 dst, i64 num_seg, i64 d, i64 reduce_op,
                         i64 n) {
    SPLIT(num_seg,
          seg_reduce_range(IP(offsets), FP(value), FP(dst), lo, hi, d, reduce_op, n));
}

/* --------------------------------------------------------- segment_softmax */
/* ported.mojo:679-768: max pass, exp(x - max) written while summing, divide. */
static void seg_softmax_range(const i64 *offsets, const f64 *value, f64 *dst, f64 *scratch,
                              i64 s0, i64 s1, i64 d, i64 n) {
    for (i64 s = s0; s < s1; ++s) {
        i64 start = offsets[s], stop = offsets[s + 1];
        if (start < 0) start = 0;
        if (stop > n) stop = n;
        if (stop < start) stop = start;
        f64 *mx = scratch, *sm = scratch + d;
        for (i64 k = 0; k < d; ++k) mx[k] = -INFINITY;
        for (i64 i = start; i < stop; ++i)
            for (i64 k = 0; k < d; ++k) mx[k] = fmax_ref(mx[k], value[i * d + k]);
        for (i64 k = 0; k < d; ++k) sm[k] = start == stop ? 1.0 : 0.0;
        for (i64 i = start; i < stop; ++i)
            for (i64 k = 0; k < d; ++k) {
                f64 e = exp(value[i * d + k] - mx[k]);
                dst[i * d + k] = e;
                sm[k] = sm[k] + e;
            }
        for (i64 i = start; i < stop; ++i)
            for (i64 k = 0; k < d; ++k) dst[i * d + k] = dst[i * d + k] / sm[k];
    }
}

/* capi.mojo:132-138 + ported.mojo:660-676 (per-worker scratch rows) */
void mdgl_segment_softmax(i64 offsets, i64 value, i64 dst, i64 scratch, i64 num_seg, i64 d,
                          i64 n) {
    SPLIT(num_seg, seg_softmax_range(IP(offsets), FP(value), FP(dst), FP(scratch) + task * 2 * d,
                                     lo, hi, d, n));
}

/* -------------------------------------------------------------- segment_mm */
/* ported.mojo:773-804: serial; out[row] = a[row] @ b[seg], per column the
 * contraction runs k = 0..d1-1 in order. */
void mdgl_segment_mm(i64 a_, i64 b_, i64 dst_, i64 seglen_a, i64 n, i64 d1, i64 r, i64 d2) {
    const f64 *a = FP(a_), *b = FP(b_);
    f64 *dst = FP(dst_);
    const i64 *seglen = IP(seglen_a);
    (void)n;
    i64 row = 0;
    for (i64 seg = 0; seg < r; ++seg) {
        i64 end = row + seglen[seg];
        for (; row < end; ++row)
            for (i64 j = 0; j < d2; ++j) {
                f64 acc = 0.0;
                for (i64 k = 0; k < d1; ++k) acc += a[row * d1 + k] * b[(seg * d1 + k) * d2 + j];
                dst[row * d2 + j] = acc;
            }
    }
}

/* ------------------------------------------------------------ edge_softmax */
/* ported.mojo:918-987 (d > 1) and :1014-1080 (d == 1): the same arithmetic;
 * rows whose selection is empty write zeros to the selected edges. */
static void es_range(const i64 *indptr, const i64 *eid, const int8_t *mask, const f64 *logits,
                     f64 *dst, f64 *scratch, i64 i0, i64 i1, i64 all_ones, i64 d) {
    f64 *mx = scratch, *sm = scratch + d;
    for (i64 i = i0; i < i1; ++i) {
        i64 start = indptr[i], stop = indptr[i + 1];
        if (start >= stop) continue;
        for (i64 h = 0; h < d; ++h) mx[h] = -INFINITY;
        int any = 0;
        for (i64 j = start; j < stop; ++j) {
            i64 e = eid[j];
            if (all_ones == 1 || mask[e] == 1) {
                for (i64 h = 0; h < d; ++h) mx[h] = fmax_ref(mx[h], logits[e * d + h]);
                any = 1;
            }
        }
        if (!any) {
            for (i64 j = start; j < stop; ++j) {
                i64 e = eid[j];
                if (all_ones == 1 || mask[e] == 1)
                    for (i64 h = 0; h < d; ++h) dst[e * d + h] = 0.0;
            }
            continue;
        }
        for (i64 h = 0; h < d; ++h) sm[h] = 0.0;
        for (i64 j = start; j < stop; ++j) {
            i64 e = eid[j];
            if (all_ones == 1 || mask[e] == 1)
                for (i64 h = 0; h < d; ++h) {
                    f64 v = exp(logits[e * d + h] - mx[h]);
                    dst[e * d + h] = v;
                    sm[h] = sm[h] + v;
                }
        }
        for (i64 j = start; j < stop; ++j) {
            i64 e = eid[j];
            if (all_ones == 1 || mask[e] == 1)
                for (i64 h = 0; h < d; ++h) dst[e * d + h] = dst[e * d + h] / sm[h];
        }
    }
}

/* capi.mojo:149-165 + ported.mojo:876-915 */
void mdgl_edge_softmax_(i64 indptr, i64 indices, i64 eid, i64 mask, i64 logits, i64 dst,
                        i64 scratch, i64 num_nodes, i64 all_ones, i64 d) {
    (void)indices;
    /* the d == 1 path keeps max/sum in registers; give it a private pair */
    if (d == 1) {
        SPLIT(num_nodes, {
            f64 pair[2];
            es_range(IP(indptr), IP(eid), BP(mask), FP(logits), FP(dst), pair, lo, hi, all_ones,
                     1);
        });
        return;
    }
    SPLIT(num_nodes, es_range(IP(indptr), IP(eid), BP(mask), FP(logits), FP(dst),
                              FP(scratch) + task * 2 * d, lo, hi, all_ones, d));
}

/* --------------------------------------------------------------- gather_mm */
/* ported.mojo:1089-1130 */
void mdgl_gather_mm(i64 a_, i64 b_, i64 idx_b_, i64 dst_, i64 n, i64 d1, i64 d2) {
    const f64 *a = FP(a_), *b = FP(b_);
    const i64 *idx_b = IP(idx_b_);
    f64 *dst = FP(dst_);
    SPLIT(n, {
        for (i64 i = lo; i < hi; ++i) {
            i64 o = idx_b[i] * d1 * d2;
            for (i64 j = 0; j < d2; ++j) {
                f64 acc = 0.0;
                for (i64 k = 0; k < d1; ++k) acc += a[i * d1 + k] * b[o + k * d2 + j];
                dst[i * d2 + j] = acc;
            }
        }
    });
}

/* capi.mojo:48-50 */
i64 mdgl_workers(void) { return WORKERS; }

/* Threads the OpenMP runtime will use for the 32-task split. */
i64 oref_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* The reference's in-CSR build (python/mojodgl/heterograph.py:69-86):
 * deg = bincount(key), indptr = [0, cumsum(deg)], order = argsort(key,
 * kind="stable"), indices = other[order].  A counting sort is a stable
 * argsort of integer keys, so this is the same arrays in O(E) (the timed CPU
 * arm builds config 3's 125M-edge CSR with it; it is not timed itself). */
void oref_csr_build(i64 key_, i64 other_, i64 num_edges, i64 num_nodes, i64 indptr_, i64 deg_,
                    i64 order_, i64 indices_) {
    const i64 *key = IP(key_), *other = IP(other_);
    i64 *indptr = IP(indptr_), *deg = IP(deg_), *order = IP(order_), *indices = IP(indices_);
    memset(deg, 0, (size_t)num_nodes * sizeof(i64));
    for (i64 e = 0; e < num_edges; ++e) deg[key[e]] += 1;
    indptr[0] = 0;
    for (i64 v = 0; v < num_nodes; ++v) indptr[v + 1] = indptr[v] + deg[v];
    i64 *next = (i64 *)malloc((size_t)(num_nodes > 0 ? num_nodes : 1) * sizeof(i64));
    memcpy(next, indptr, (size_t)num_nodes * sizeof(i64));
    for (i64 e = 0; e < num_edges; ++e) {
        i64 p = next[key[e]]++;
        order[p] = e;
        indices[p] = other[e];
    }
    free(next);
}
