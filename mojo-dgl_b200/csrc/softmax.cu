// Fused per-row softmax over a CSR (replaces mdgl_edge_softmax_,
// src/ported.mojo:876-1080, and mdgl_segment_softmax, src/ported.mojo:660-768).
//
// Both reference kernels compute, for each CSR row and each column h, over the
// row's selected items e,
//     out[e, h] = exp(z[e, h] - max) / sum exp(z[., h] - max).
// edge_softmax reaches the items through the CSR's edge ids; segment_softmax's
// items are the consecutive rows of `value` (eid = identity).
//
// Pass 1 computes each row's (max, 1 / sum) over merge-path chunks of (row
// ends, items), one warp per chunk, so a warp gets the same number of items
// whatever the degrees are and a 50,000-edge attention hub is spread over
// many warps.  Three forms by row width:
//  * k_softmax_lane_stats, items of at most 64 bytes (8 float32 heads): each
//    lane walks its own run of consecutive items with all columns in
//    registers; split rows are joined by one warp scan per chunk;
//  * k_softmax_stats, other narrow rows (up to 8 column vectors): a step of
//    the warp covers 32 / CV items, finds each item's row among 32 row ends
//    held across the warp and reduces every row's items with segmented scans;
//  * k_softmax_walk_stats, wide rows: a team of lanes walks the chunk in CSR
//    order, gSpMM-style.
// Logits reach shared memory through per-lane cp.async rings.  A row split
// over chunks leaves a (max, sum) piece per chunk, folded by k_softmax_fixup.
// Pass 2 writes out = exp(z - max) * (1 / sum): in edge order when the caller
// gives every edge's row (logits read and outputs written contiguously), else
// item-parallel with the row the first pass recorded per item, or along the
// same walk for wide rows.
// The rounding differs from the reference's max-then-sum loops (a tree of
// partial sums, a multiply by the reciprocal, CUDA's exp), so results are
// compared with a relative tolerance (1e-12 in float64).
#include "spmm_impl.cuh"

namespace bgl {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kSoftBlock = 256;
#ifndef BGL_SOFTMAX_DEPTH
#define BGL_SOFTMAX_DEPTH 4  // steps whose logits are in flight ahead of the fold
#endif

template <typename T>
struct SoftArgs {
    const int64_t *indptr;
    const int32_t *eid;
    const int8_t *mask;
    int32_t num_rows;
    int32_t num_items;
    const T *logits;
    T *out;
    int32_t d;
    int64_t num_chunks;
    const Coord *coords;
    int32_t *head_row;
    int32_t *tail_row;
    T *head_m, *head_s, *tail_m, *tail_s;  // per chunk x d: the split rows' (max, sum) pieces
    T *row_m, *row_r;                      // per row: its d maxima and d values of 1 / sum
    int32_t *item_row;                     // per item: its row
    const int32_t *edge_row;               // optional: the row of every edge, by edge id
    int64_t rstride;                       // row_m / row_r elements between rows (2 d:
                                           // a row's maxima and reciprocals side by side)
    const int *gate;                       // optional: run only if *gate != 0 (the
                                           // fallback of the segment-per-warp pass)
};

// (m, s) <- the softmax statistics of the items of (m, s) followed by those of
// (m2, s2): the larger max wins and the other sum is rescaled to it.
// One exponential and no branch: the smaller max's sum is scaled by
// exp(-|m - m2|), which is 0 against an empty piece (max -inf) and taken as 1
// for equal maxima (two empty pieces included).
template <typename T>
__device__ __forceinline__ void combine(T &m, T &s, T m2, T s2) {
    const T dm = Arith<T>::sub(m, m2);
    const T e = m == m2 ? T(1) : Arith<T>::ex(dm > T(0) ? -dm : dm);
    const bool keep = m >= m2;
    s = keep ? Arith<T>::add(s, Arith<T>::mul(s2, e)) : Arith<T>::add(Arith<T>::mul(s, e), s2);
    m = keep ? m : m2;
}

template <typename T, int V>
__device__ __forceinline__ void put2(T *pa, T *pb, int64_t off, const T (&va)[V], const T (&vb)[V]) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
        pa[off + v] = va[v];
        pb[off + v] = vb[v];
    }
}

// Pass 1: per-row (max, 1 / sum) for rows that start and end in the chunk,
// (max, sum) pieces for the others, and every item's row.
template <typename T, int V, int CV>
__global__ void __launch_bounds__(kSoftBlock) k_softmax_stats(const SoftArgs<T> a) {
    if (a.gate && *a.gate == 0) return;
    constexpr int W = 32 / CV;  // items per step
    constexpr int P = BGL_SOFTMAX_DEPTH, R = P + 1;
    constexpr int SLOT = V * (int)sizeof(T);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // ring stage s: this thread's logits at [s][thread], its item's edge id
    // (for the mask) at [R][...]
    const uint32_t sbase = smem_addr(smem_raw) + threadIdx.x * SLOT;
    const T *pbase = reinterpret_cast<const T *>(smem_raw + threadIdx.x * SLOT);
    int32_t *ebase = reinterpret_cast<int32_t *>(smem_raw + R * kSoftBlock * SLOT) + threadIdx.x;

    const int lane = threadIdx.x & 31;
    const int k = lane / CV, c = lane % CV;
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;  // warp-uniform
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t x1 = (int32_t)a.coords[chunk + 1].x, ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t nrows = a.num_rows;
    const int64_t d = a.d;
    // row x0 began in an earlier chunk and ends in this one: its items here
    // are a head piece; row x1 has items here and goes on: a tail piece
    const bool x0_before = x0 < nrows && (int32_t)a.indptr[x0] < y0;
    const bool has_head = x0_before && x0 < x1;
    const bool has_tail = x1 < nrows && max((int32_t)a.indptr[x1], y0) < ye;
    const int32_t cvn = a.d / V;

    for (int32_t cb = 0; cb < cvn && y0 < ye; cb += CV) {
        const int32_t cv = cb + c;
        const bool live = cv < cvn;
        const int64_t col = (int64_t)cv * V;

        // the copy side of the ring: step w_copy, this lane's item id fetched
        // one step ahead of its copy
        int32_t w_copy = y0, e_next = 0;
        auto fetch = [&]() {
            const int32_t i = w_copy + k;
            if (i < ye) e_next = a.eid ? __ldg(a.eid + i) : i;
        };
        auto copy_step = [&](int stage) {
            const int32_t i = w_copy + k;
            if (i < ye) {
                if (live)
                    cp_async<SLOT>(sbase + stage * kSoftBlock * SLOT,
                                   a.logits + (int64_t)e_next * d + col);
                if (a.mask) ebase[stage * kSoftBlock] = e_next;
            }
            cp_async_commit();  // an empty group past the chunk end keeps the count
            w_copy += W;
            fetch();
        };
        fetch();
#pragma unroll
        for (int q = 0; q < P; ++q) copy_step(q);

        int32_t x = x0;             // the row holding the step's first item
        int32_t carry_row = -1;     // the row left open by the previous step
        T cm[V], cs[V];             // its (max, sum) so far in this chunk
#pragma unroll
        for (int v = 0; v < V; ++v) {
            cm[v] = Arith<T>::ninf();
            cs[v] = T(0);
        }
        int fstage = 0, cstage = P;
        for (int32_t w0 = y0; w0 < ye; w0 += W) {
            copy_step(cstage);
            cp_async_wait<P>();  // the step at w0 has landed
            const int32_t wend = min(w0 + W, ye);
            const int32_t i = w0 + k;
            const bool valid = i < wend;

            // the row of item i: lane j holds the end of row x + j (rows from
            // x1 on do not end in this chunk)
            const int32_t endj = (x + lane < x1) ? (int32_t)a.indptr[x + lane + 1] : INT32_MAX;
            int32_t cnt = 0;
#pragma unroll
            for (int step = 16; step > 0; step >>= 1) {
                const int32_t v = __shfl_sync(kFull, endj, cnt + step - 1);
                if (v <= i) cnt += step;
            }
            int32_t row = x + cnt;
            int32_t rend = __shfl_sync(kFull, endj, cnt);
            if (valid && rend <= i) {
                // past the 32 rows held (a run of empty rows): search the rest
                int32_t lo = x + 32, hi = x1;
                while (lo < hi) {
                    const int32_t mid = lo + ((hi - lo) >> 1);
                    if ((int32_t)a.indptr[mid + 1] <= i)
                        lo = mid + 1;
                    else
                        hi = mid;
                }
                row = lo;
                rend = lo < x1 ? (int32_t)a.indptr[lo + 1] : INT32_MAX;
            }
            if (!valid) row = INT32_MAX;  // joins no item's segment

            T z[V];
#pragma unroll
            for (int v = 0; v < V; ++v) z[v] = Arith<T>::ninf();
            if (valid && live) {
                bool sel = true;
                if (a.mask) sel = a.mask[ebase[fstage * kSoftBlock]] == 1;
                if (sel) {
                    using VT = typename VecT<T, V>::type;
                    const VT vv = *reinterpret_cast<const VT *>(pbase + fstage * kSoftBlock * V);
                    const T *sv = reinterpret_cast<const T *>(&vv);
#pragma unroll
                    for (int v = 0; v < V; ++v) z[v] = sv[v];
                }
            }

            // segmented max over the step's items of each row
            T mx[V];
#pragma unroll
            for (int v = 0; v < V; ++v) mx[v] = z[v];
#pragma unroll
            for (int off = 1; off < W; off <<= 1) {
                const int32_t orow = __shfl_up_sync(kFull, row, off * CV);
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const T om = __shfl_up_sync(kFull, mx[v], off * CV);
                    if (k >= off && orow == row && om > mx[v]) mx[v] = om;
                }
            }
            // the row's max over the step sits at its last item of the step;
            // the row left open by the previous step takes its running max
            // into account here, so its sum needs rescaling only when the max
            // grows
            const int32_t seg_last = valid ? min(rend, wend) - 1 - w0 : k;
            const int src = seg_last * CV + c;
            const bool carried = row == carry_row;
            T ev[V], M[V];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                M[v] = __shfl_sync(kFull, mx[v], src);
                if (carried && cm[v] > M[v]) M[v] = cm[v];
                ev[v] = (valid && M[v] != Arith<T>::ninf())
                            ? Arith<T>::ex(Arith<T>::sub(z[v], M[v]))
                            : T(0);
            }
            // segmented sum of exp(z - max)
#pragma unroll
            for (int off = 1; off < W; off <<= 1) {
                const int32_t orow = __shfl_up_sync(kFull, row, off * CV);
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const T oe = __shfl_up_sync(kFull, ev[v], off * CV);
                    if (k >= off && orow == row) ev[v] = Arith<T>::add(ev[v], oe);
                }
            }

            // each row's last item of the step folds in the open row's
            // statistics and stores the row, its head or tail piece
            T rm[V], rs[V];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                rm[v] = M[v];
                rs[v] = ev[v];
            }
            if (valid && k == seg_last) {
                if (carried) {
#pragma unroll
                    for (int v = 0; v < V; ++v) {
                        T prev = cs[v];
                        if (cm[v] != rm[v])  // the max grew: rescale the earlier sum
                            prev = cm[v] == Arith<T>::ninf()
                                       ? T(0)
                                       : Arith<T>::mul(prev, Arith<T>::ex(Arith<T>::sub(cm[v], rm[v])));
                        rs[v] = Arith<T>::add(prev, rs[v]);
                    }
                }
                if (live) {
                    if (rend <= wend) {
                        if (row == x0 && x0_before) {
                            put2<T, V>(a.head_m, a.head_s, chunk * d + col, rm, rs);
                        } else {
                            T r[V];
#pragma unroll
                            for (int v = 0; v < V; ++v) r[v] = Arith<T>::div(T(1), rs[v]);
                            put2<T, V>(a.row_m, a.row_r, (int64_t)row * a.rstride + col, rm, r);
                        }
                    } else if (wend == ye) {
                        put2<T, V>(a.tail_m, a.tail_s, chunk * d + col, rm, rs);
                    }
                }
            }
            // the row holding the step's last item stays open if it goes on
            const int ll = (wend - 1 - w0) * CV + c;
            const int32_t lrow = __shfl_sync(kFull, row, ll);
            const int32_t lrend = __shfl_sync(kFull, rend, ll);
#pragma unroll
            for (int v = 0; v < V; ++v) {
                const T nm = __shfl_sync(kFull, rm[v], ll);
                const T ns = __shfl_sync(kFull, rs[v], ll);
                cm[v] = nm;
                cs[v] = ns;
            }
            carry_row = lrend > wend ? lrow : -1;
            x = lrow;
            if (cb == 0 && valid && c == 0) __stcs(a.item_row + i, row);
            fstage = fstage + 1 == R ? 0 : fstage + 1;
            cstage = cstage + 1 == R ? 0 : cstage + 1;
        }
        cp_async_wait<0>();
    }
    // row x0 ends here without an item in this chunk: an empty head piece
    if (has_head && (int32_t)a.indptr[x0 + 1] <= y0) {
        for (int64_t h = lane; h < d; h += 32) {
            a.head_m[chunk * d + h] = Arith<T>::ninf();
            a.head_s[chunk * d + h] = T(0);
        }
    }
    if (lane == 0) {
        a.head_row[chunk] = has_head ? x0 : -1;
        a.tail_row[chunk] = has_tail ? x1 : -1;
    }
}

// ---------------------------------------------------------------- wide rows
// With 16 or more lanes per item a step of the warp-wide kernel above covers
// one or two items and its per-step row search and scans dominate.  Wide rows
// instead give each chunk to a team of `ts` lanes that walks the chunk's items
// in CSR order, the gSpMM way: logits come through the same per-lane cp.async
// ring (groups of UN items, P groups ahead) and every value takes one online
// (max, sum) update -- a larger value rescales the running sum.
// Both cases need exp(-|z - m|): a larger z rescales the running sum by
// exp(m - z) and adds 1, a smaller one adds exp(z - m).  One exponential per
// value and a select, no divergent branch.
template <typename T>
__device__ __forceinline__ void online(T &m, T &s, T z) {
    const T dz = Arith<T>::sub(z, m);
    const T e = Arith<T>::ex(dz > T(0) ? -dz : dz);
    const bool up = z > m;
    s = up ? Arith<T>::add(Arith<T>::mul(s, e), T(1)) : Arith<T>::add(s, e);
    m = up ? z : m;
}

constexpr int kWalkUN = 4;     // items per group
constexpr int kWalkDepth = 2;  // groups in flight ahead of the fold (60 KB: 3 blocks per SM)

template <typename T, int V>
struct WalkRing {
    static constexpr int R = kWalkDepth + 1;
    static constexpr int SLOT = V * (int)sizeof(T);
    // logits slots, then the items' edge ids (int32) for the mask and the stores
    static constexpr int smem = R * kWalkUN * kSoftBlock * (SLOT + 4);
};

// The walk shared by both wide-row passes: `on_item(e, i, z)` for every item
// i (edge id e) of the team's chunk in CSR order, `close_row()` whenever the
// walk passes a row end (the caller tracks rows).  z is the lane's V logits.
template <typename T, int V, bool NEED_E, typename OnItem>
__device__ __forceinline__ void walk_items(const SoftArgs<T> &a, int32_t y0, int32_t ye, int t,
                                           bool live, int64_t col, OnItem on_item) {
    using Ring = WalkRing<T, V>;
    constexpr int UN = kWalkUN, P = kWalkDepth, R = Ring::R, SLOT = Ring::SLOT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t sbase = smem_addr(smem_raw) + threadIdx.x * SLOT;
    const T *pbase = reinterpret_cast<const T *>(smem_raw + threadIdx.x * SLOT);
    int32_t *ebase =
        reinterpret_cast<int32_t *>(smem_raw + R * UN * kSoftBlock * SLOT) + threadIdx.x;
    auto slot = [](int stage, int u) { return (stage * UN + u) * kSoftBlock; };
    (void)t;

    int32_t ids[UN];
    int32_t e_copy = y0;
    auto fetch_one = [&](int u) { ids[u] = a.eid ? __ldg(a.eid + e_copy + u) : e_copy + u; };
    auto fetch = [&]() {
        if (e_copy + UN <= ye) {
#pragma unroll
            for (int u = 0; u < UN; ++u) fetch_one(u);
        } else {
#pragma unroll
            for (int u = 0; u < UN; ++u)
                if (e_copy + u < ye) fetch_one(u);
        }
    };
    auto copy_one = [&](int stage, int u) {
        if (live) cp_async<SLOT>(sbase + slot(stage, u) * SLOT, a.logits + (int64_t)ids[u] * a.d + col);
        if (NEED_E || a.mask) ebase[slot(stage, u)] = ids[u];
    };
    auto copy_group = [&](int stage) {
        if (e_copy + UN <= ye) {
#pragma unroll
            for (int u = 0; u < UN; ++u) copy_one(stage, u);
        } else {
#pragma unroll
            for (int u = 0; u < UN; ++u)
                if (e_copy + u < ye) copy_one(stage, u);
        }
        cp_async_commit();
        e_copy += UN;
        fetch();
    };
    auto fold_one = [&](int stage, int u, int32_t i) {
        const int32_t e = (NEED_E || a.mask) ? ebase[slot(stage, u)] : i;
        T z[V];
        using VT = typename VecT<T, V>::type;
        const VT vv = *reinterpret_cast<const VT *>(pbase + slot(stage, u) * V);
        const T *sv = reinterpret_cast<const T *>(&vv);
#pragma unroll
        for (int v = 0; v < V; ++v) z[v] = sv[v];
        on_item(e, i, z);
    };
    fetch();
#pragma unroll
    for (int g = 0; g < P; ++g) copy_group(g);
    int fstage = 0, cstage = P;
    for (int32_t i0 = y0; i0 < ye; i0 += UN) {
        copy_group(cstage);
        cp_async_wait<P>();
        if (i0 + UN <= ye) {
#pragma unroll
            for (int u = 0; u < UN; ++u) fold_one(fstage, u, i0 + u);
        } else {
#pragma unroll
            for (int u = 0; u < UN; ++u)
                if (i0 + u < ye) fold_one(fstage, u, i0 + u);
        }
        fstage = fstage + 1 == R ? 0 : fstage + 1;
        cstage = cstage + 1 == R ? 0 : cstage + 1;
    }
    cp_async_wait<0>();
}

// Wide rows, pass 1: (max, 1 / sum) of rows that start and end in the chunk,
// (max, sum) pieces of the others.
template <typename T, int V>
__global__ void __launch_bounds__(kSoftBlock, 3) k_softmax_walk_stats(const SoftArgs<T> a, int ts) {
    if (a.gate && *a.gate == 0) return;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t x1 = (int32_t)a.coords[chunk + 1].x, ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t nrows = a.num_rows;
    const int64_t d = a.d;
    const int32_t cvn = a.d / V;
    int32_t head_row = -1, tail_row = -1;
    for (int32_t cb = 0; cb < cvn; cb += ts) {
        int32_t x = x0;
        if (x >= nrows) break;
        const int32_t cv = cb + t;
        const bool live = cv < cvn;
        const int64_t col = (int64_t)cv * V;
        int32_t rs = (int32_t)a.indptr[x];
        int32_t re = (x < x1) ? (int32_t)a.indptr[x + 1] : ye;
        int32_t row_begin = y0;
        T m[V], s[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            m[v] = Arith<T>::ninf();
            s[v] = T(0);
        }
        auto close_row = [&]() {
            if (live) {
                if (row_begin == rs) {
                    T r[V];
#pragma unroll
                    for (int v = 0; v < V; ++v) r[v] = Arith<T>::div(T(1), s[v]);
                    put2<T, V>(a.row_m, a.row_r, (int64_t)x * a.rstride + col, m, r);
                } else {
                    put2<T, V>(a.head_m, a.head_s, chunk * d + col, m, s);
                }
            }
            if (row_begin != rs) head_row = x;
            row_begin = re;
            rs = re;
            ++x;
            re = (x < x1) ? (int32_t)a.indptr[x + 1] : ye;
#pragma unroll
            for (int v = 0; v < V; ++v) {
                m[v] = Arith<T>::ninf();
                s[v] = T(0);
            }
        };
        walk_items<T, V, false>(a, y0, ye, t, live, col, [&](int32_t e, int32_t i, const T(&z)[V]) {
            while (i >= re) close_row();
            if (a.mask && a.mask[e] != 1) return;
#pragma unroll
            for (int v = 0; v < V; ++v) online(m[v], s[v], z[v]);
        });
        while (x < x1) close_row();  // rows ending at the chunk end, empty rows
        if (x < nrows && ye > row_begin) {
            if (live) put2<T, V>(a.tail_m, a.tail_s, chunk * d + col, m, s);
            tail_row = x;
        }
    }
    if (t == 0) {
        a.head_row[chunk] = head_row;
        a.tail_row[chunk] = tail_row;
    }
}

// Wide rows, pass 2: out = exp(z - max) * (1 / sum) along the same walk; a
// row's statistics are loaded when the walk enters it, the next row's ahead.
template <typename T, int V>
__global__ void __launch_bounds__(kSoftBlock, 3) k_softmax_walk_apply(const SoftArgs<T> a, int ts) {
    if (a.gate && *a.gate == 0) return;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t nrows = a.num_rows;
    const int64_t d = a.d;
    const int32_t cvn = a.d / V;
    for (int32_t cb = 0; cb < cvn; cb += ts) {
        int32_t x = x0;
        if (x >= nrows || y0 >= ye) break;
        const int32_t cv = cb + t;
        const bool live = cv < cvn;
        const int64_t col = (int64_t)cv * V;
        // the row holding the chunk's first item (skipping rows that end first)
        int32_t re = (int32_t)a.indptr[x + 1];
        while (y0 >= re) re = (int32_t)a.indptr[++x + 1];
        T m[V], r[V], nm[V], nr[V];
        auto load_stats = [&](int32_t row, T(&mm)[V], T(&rr)[V]) {
            if (live && row < nrows) {
                load_vec<T, V>(a.row_m + (int64_t)row * a.rstride + col, mm);
                load_vec<T, V>(a.row_r + (int64_t)row * a.rstride + col, rr);
            }
        };
        load_stats(x, m, r);
        load_stats(x + 1, nm, nr);
        walk_items<T, V, true>(a, y0, ye, t, live, col, [&](int32_t e, int32_t i, const T(&z)[V]) {
            if (i >= re) {
                const int32_t prev = x;
                do {
                    re = (int32_t)a.indptr[++x + 1];
                } while (i >= re);
                if (x == prev + 1) {  // the prefetched row
#pragma unroll
                    for (int v = 0; v < V; ++v) {
                        m[v] = nm[v];
                        r[v] = nr[v];
                    }
                } else {
                    load_stats(x, m, r);
                }
                load_stats(x + 1, nm, nr);
            }
            if (!live || (a.mask && a.mask[e] != 1)) return;
            T o[V];
#pragma unroll
            for (int v = 0; v < V; ++v)
                o[v] = Arith<T>::mul(Arith<T>::ex(Arith<T>::sub(z[v], m[v])), r[v]);
            store_stream<T, V>(a.out + (int64_t)e * d + col, o);
        });
    }
}

// ------------------------------------------------------------- narrow rows
// Rows of at most kLaneBytes per item (8 heads of float32, say).  The warp's
// lanes form 32 / L runs of L lanes, L = the item's column vectors, so a lane
// holds one vector of V columns and the L lanes of a run read an item's row
// with one instruction (one request per row: random rows cost requests, not
// bytes).  Run j takes the j-th stretch of K = ceil(items / runs) consecutive
// items of the chunk and walks it in CSR order, one online (max, sum) update
// per value -- no per-step row search, no scans.  The logits come through a
// per-lane cp.async ring, P groups of U items ahead of the fold; the edge ids
// through shared-memory tiles the warp copies with instructions that cover
// whole segments of a run's ids.  A row that starts and ends inside a run is
// stored as it closes.  A run's first row, if it began in an earlier run, is
// a head piece; its last row, if it goes on past the run, a tail piece.  After
// the walk one segmented scan of the tails over the runs joins every row split
// between runs: a head takes the scanned tail of the run before it.  The
// chunk's own head and tail pieces (rows split between chunks) are left for
// k_softmax_fixup as in the other passes.
#ifndef BGL_SOFTMAX_LANE_BYTES
#define BGL_SOFTMAX_LANE_BYTES 64  // widest item (d * sizeof(T)) the lane walk takes
#endif
#ifndef BGL_SOFTMAX_LANE_WAVES
// waves of 24 resident warps per SM the lane walk's chunks make (config 2: one
// wave 5 % slower, four within 2 %)
#define BGL_SOFTMAX_LANE_WAVES 2
#endif
constexpr int kLaneBytes = BGL_SOFTMAX_LANE_BYTES;

template <typename T, int V, int L>
struct LaneRing {
    static constexpr int VB = V * (int)sizeof(T);  // one cp.async per lane and item
    static constexpr int RUNS = 32 / L;            // runs per warp
    static constexpr int U = VB >= 16 ? 2 : 4;     // items per group
    static constexpr int P = VB >= 16 ? 4 : 3;     // groups in flight ahead of the fold
    static constexpr int R = P + 1;
    // logits [R * U][thread], then the item ids [R * U][thread]
    static constexpr int ring_bytes = R * U * kSoftBlock * (VB + 4);
    // then each warp's edge ids in tiles of W per run, two buffers, rows padded
    // to S words; a tile holds GPT ring groups and is loaded one tile ahead of
    // the copies that use it
    static constexpr int W = 16;
    static constexpr int GPT = W / U;
    static constexpr int S = W + 1;
    static constexpr int smem = ring_bytes + (kSoftBlock / 32) * 2 * RUNS * S * 4;
    static_assert(GPT >= P + 1, "a tile must land before the copies that read it");
    static_assert(RUNS * W % 32 == 0, "a tile is copied by whole warp instructions");
};

template <typename T, int V, int L>
__global__ void __launch_bounds__(kSoftBlock, 3) k_softmax_lane_stats(const SoftArgs<T> a) {
    if (a.gate && *a.gate == 0) return;
    using Ring = LaneRing<T, V, L>;
    constexpr int U = Ring::U, P = Ring::P, R = Ring::R, VB = Ring::VB, RUNS = Ring::RUNS;
    constexpr int W = Ring::W, S = Ring::S, GPT = Ring::GPT;
    using VT = typename VecT<T, V>::type;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    auto slot = [](int stage, int u) { return (stage * U + u) * kSoftBlock; };
    const uint32_t sbase = smem_addr(smem_raw) + threadIdx.x * VB;
    const VT *pbase = reinterpret_cast<const VT *>(smem_raw) + threadIdx.x;
    int32_t *ebase = reinterpret_cast<int32_t *>(smem_raw + R * U * kSoftBlock * VB) + threadIdx.x;

    const int lane = threadIdx.x & 31;
    const int run = lane / L, c = lane % L;  // the lane's run and column vector
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;  // warp-uniform
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t x1 = (int32_t)a.coords[chunk + 1].x, ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t nrows = a.num_rows;
    const int64_t d = a.d;
    const bool live = c < a.d / V;
    const int64_t col = (int64_t)c * V;
    const bool x0_before = x0 < nrows && (int32_t)a.indptr[x0] < y0;
    const bool has_head = x0_before && x0 < x1;
    const bool has_tail = x1 < nrows && max((int32_t)a.indptr[x1], y0) < ye;

    const int32_t K = (ye - y0 + RUNS - 1) / RUNS;
    const int32_t i0 = min(y0 + run * K, ye), i1 = min(i0 + K, ye);

    // Edge ids: the warp copies tile q -- ids [q W, q W + W) of every run --
    // with instructions that each cover 32 / W runs x W consecutive ids.
    int32_t *tiles = reinterpret_cast<int32_t *>(smem_raw + Ring::ring_bytes) +
                     (threadIdx.x >> 5) * 2 * RUNS * S;
    const bool staged = a.eid != nullptr;  // warp-uniform
    auto load_tile = [&](int32_t q) {
        int32_t *t = tiles + (q & 1) * RUNS * S;
#pragma unroll
        for (int k = 0; k < RUNS * W / 32; ++k) {
            const int r = k * (32 / W) + lane / W, o = lane % W;
            const int32_t rs = min(y0 + r * K, ye), p = rs + q * W + o;
            if (p < min(rs + K, ye)) cp_async<4>(smem_addr(t + r * S + o), a.eid + p);
        }
    };
    // the copy side of the ring
    int32_t c_next = i0;
    auto copy_group = [&](int stage) {
        const int32_t off = c_next - i0;  // a multiple of U, so the group is in one tile
        const int32_t *t = tiles + ((off / W) & 1) * RUNS * S + run * S + off % W;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (c_next + u < i1) {
                const int32_t id = staged ? t[u] : c_next + u;
                if (live) cp_async<VB>(sbase + slot(stage, u) * VB, a.logits + (int64_t)id * d + col);
                ebase[slot(stage, u)] = id;
            }
        }
        cp_async_commit();  // an empty group past the run's end keeps the count
        c_next += U;
    };
    if (staged) {
        load_tile(0);
        load_tile(1);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
#pragma unroll
    for (int g = 0; g < P; ++g) copy_group(g);

    T m[V], s[V], hm[V], hs[V];
    auto reset = [&]() {
#pragma unroll
        for (int v = 0; v < V; ++v) {
            m[v] = Arith<T>::ninf();
            s[v] = T(0);
        }
    };
    auto put_row = [&](int32_t row, const T (&mm)[V], const T (&ss)[V]) {
        if (!live) return;
        T r[V];
#pragma unroll
        for (int v = 0; v < V; ++v) r[v] = Arith<T>::div(T(1), ss[v]);
        store_vec<T, V>(a.row_m + (int64_t)row * a.rstride + col, mm);
        store_vec<T, V>(a.row_r + (int64_t)row * a.rstride + col, r);
    };
    reset();
#pragma unroll
    for (int v = 0; v < V; ++v) {
        hm[v] = Arith<T>::ninf();
        hs[v] = T(0);
    }
    int32_t x = x0, rb = 0, re = 0, hrow = -1, trow = -1;
    if (i0 < i1) {
        // the row holding item i0: the first row from x0 on that ends after it
        int32_t lo = x0, hi = min(x1, nrows - 1);
        while (lo < hi) {
            const int32_t mid = lo + ((hi - lo) >> 1);
            if ((int32_t)a.indptr[mid + 1] <= i0)
                lo = mid + 1;
            else
                hi = mid;
        }
        x = lo;
        rb = (int32_t)a.indptr[x];
        re = (int32_t)a.indptr[x + 1];
    }
    // a row ends: stored if it began in this run, else it is the head piece
    auto close_row = [&]() {
        if (rb >= i0) {
            put_row(x, m, s);
        } else {
            hrow = x;
#pragma unroll
            for (int v = 0; v < V; ++v) {
                hm[v] = m[v];
                hs[v] = s[v];
            }
        }
        reset();
    };
    int fstage = 0, cstage = P;
    // the same number of steps on every lane (the tiles are the warp's)
    const int32_t steps = (K + U - 1) / U;
    for (int32_t step = 0; step < steps; ++step) {
        // the copies of this step start a tile: the next one is loaded now,
        // with this step's group, and has landed P steps later, before its
        // first use GPT steps later
        if (staged && (step + P) % GPT == 0) load_tile((step + P) / GPT + 1);
        copy_group(cstage);
        cp_async_wait<P>();  // the group of this step has landed
        __syncwarp();        // and so have the other lanes' tile copies
        const int32_t g0 = i0 + step * U;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int32_t i = g0 + u;
            if (i >= i1) break;
            if (i >= re) {
                close_row();
                do {
                    ++x;
                    rb = re;
                    re = (int32_t)a.indptr[x + 1];
                } while (i >= re);
            }
            if (!a.edge_row && c == 0) __stcs(a.item_row + i, x);
            if (!live || (a.mask && a.mask[ebase[slot(fstage, u)]] != 1)) continue;
            const VT vv = pbase[slot(fstage, u)];
            const T *z = reinterpret_cast<const T *>(&vv);
#pragma unroll
            for (int v = 0; v < V; ++v) online(m[v], s[v], z[v]);
        }
        fstage = fstage + 1 == R ? 0 : fstage + 1;
        cstage = cstage + 1 == R ? 0 : cstage + 1;
    }
    cp_async_wait<0>();
    // the run's last row: a tail piece if it goes on past the run (the chunk's
    // last row always counts as going on: the next chunk closes it), else it
    // closes here
    if (i0 < i1) {
        if (re > i1 || x == x1)
            trow = x;
        else
            close_row();
    }
    // segmented inclusive scan of the tail pieces over the runs, in order
#pragma unroll
    for (int off = 1; off < RUNS; off <<= 1) {
        const int32_t orow = __shfl_up_sync(kFull, trow, off * L);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const T om = __shfl_up_sync(kFull, m[v], off * L);
            const T os = __shfl_up_sync(kFull, s[v], off * L);
            if (run >= off && trow >= 0 && orow == trow) combine(m[v], s[v], om, os);
        }
    }
    // a head piece takes the scanned tail of the run before it when that run
    // ends in the same row
    const int32_t prow = __shfl_up_sync(kFull, trow, L);
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const T pm = __shfl_up_sync(kFull, m[v], L);
        const T ps = __shfl_up_sync(kFull, s[v], L);
        if (hrow >= 0 && run > 0 && prow == hrow) combine(hm[v], hs[v], pm, ps);
    }
    if (hrow >= 0) {
        if (hrow == x0 && x0_before) {
            if (live) {
                store_vec<T, V>(a.head_m + chunk * d + col, hm);
                store_vec<T, V>(a.head_s + chunk * d + col, hs);
            }
        } else {
            put_row(hrow, hm, hs);
        }
    }
    // the chunk's tail piece: the scanned tail of the last run with items
    const int32_t last = ye > y0 ? (ye - y0 - 1) / K : -1;
    if (run == last && trow >= 0 && live) {
        store_vec<T, V>(a.tail_m + chunk * d + col, m);
        store_vec<T, V>(a.tail_s + chunk * d + col, s);
    }
    // row x0 ends here without an item in this chunk: an empty head piece
    if (has_head && (int32_t)a.indptr[x0 + 1] <= y0) {
        for (int64_t h = lane; h < d; h += 32) {
            a.head_m[chunk * d + h] = Arith<T>::ninf();
            a.head_s[chunk * d + h] = T(0);
        }
    }
    if (lane == 0) {
        a.head_row[chunk] = has_head ? x0 : -1;
        a.tail_row[chunk] = has_tail ? x1 : -1;
    }
}

// Folds every split row's pieces in CSR order into its (max, 1 / sum): one
// warp per chunk in which a split row ends.  A row of few pieces is folded
// with a lane per column, piece after piece; a row of many (an attention hub
// over a hundred chunks or more) with a lane per piece and a warp reduction
// per column -- whichever takes fewer dependent loads.
template <typename T>
__global__ void __launch_bounds__(kSoftBlock) k_softmax_fixup(const SoftArgs<T> a) {
    if (a.gate && *a.gate == 0) return;
    const int lane = threadIdx.x & 31;
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (chunk >= a.num_chunks) return;
    const int32_t row = a.head_row[chunk];
    if (row < 0) return;
    const int64_t first = first_piece(a.tail_row, chunk, row, lane, 32);
    const int64_t d = a.d, np = chunk - first + 1;
    auto piece = [&](int64_t q, int64_t h, T &m, T &s) {
        const bool head = q == chunk;
        m = (head ? a.head_m : a.tail_m)[q * d + h];
        s = (head ? a.head_s : a.tail_s)[q * d + h];
    };
    auto put = [&](int64_t h, T m, T s) {
        a.row_m[(int64_t)row * a.rstride + h] = m;
        a.row_r[(int64_t)row * a.rstride + h] = Arith<T>::div(T(1), s);
    };
    if ((d + 31) / 32 * np <= d * ((np + 31) / 32)) {
        for (int64_t h = lane; h < d; h += 32) {
            T m = Arith<T>::ninf(), s = T(0);
#pragma unroll 4
            for (int64_t q = first; q <= chunk; ++q) {
                T m2, s2;
                piece(q, h, m2, s2);
                combine(m, s, m2, s2);
            }
            put(h, m, s);
        }
    } else {
        for (int64_t h = 0; h < d; ++h) {
            T m = Arith<T>::ninf(), s = T(0);
            for (int64_t q = first + lane; q <= chunk; q += 32) {
                T m2, s2;
                piece(q, h, m2, s2);
                combine(m, s, m2, s2);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const T m2 = __shfl_xor_sync(kFull, m, off), s2 = __shfl_xor_sync(kFull, s, off);
                combine(m, s, m2, s2);
            }
            if (lane == 0) put(h, m, s);
        }
    }
}

// Pass 2: out = exp(z - max) * (1 / sum) for every selected item, a team of CV
// lanes per item, UN items of a team in flight.
template <typename T, int V, int CV>
__global__ void __launch_bounds__(kSoftBlock) k_softmax_apply(const SoftArgs<T> a) {
    if (a.gate && *a.gate == 0) return;
    constexpr int UN = 4;
    const int c = (threadIdx.x & 31) % CV;
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / CV;
    const int64_t teams = ((int64_t)gridDim.x * blockDim.x) / CV;
    const int32_t cvn = a.d / V;
    const int64_t d = a.d;
    for (int32_t cb = 0; cb < cvn; cb += CV) {
        const int32_t cv = cb + c;
        if (cv >= cvn) break;
        const int64_t col = (int64_t)cv * V;
        for (int64_t i0 = team; i0 < a.num_items; i0 += teams * UN) {
            int64_t e[UN];
            int32_t r[UN];
            bool ok[UN];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                const int64_t i = i0 + u * teams;
                ok[u] = i < a.num_items;
                if (ok[u]) {
                    e[u] = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                    r[u] = __ldg(a.item_row + i);
                }
            }
            if (a.mask) {
#pragma unroll
                for (int u = 0; u < UN; ++u)
                    if (ok[u]) ok[u] = a.mask[e[u]] == 1;
            }
            T z[UN][V], m[UN][V], rr[UN][V];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (ok[u]) {
                    ld_stream(a.logits + e[u] * d + col, z[u]);
                    load_vec<T, V>(a.row_m + (int64_t)r[u] * a.rstride + col, m[u]);
                    load_vec<T, V>(a.row_r + (int64_t)r[u] * a.rstride + col, rr[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (ok[u]) {
                    T o[V];
#pragma unroll
                    for (int v = 0; v < V; ++v)
                        o[v] = Arith<T>::mul(Arith<T>::ex(Arith<T>::sub(z[u][v], m[u][v])), rr[u][v]);
                    store_stream<T, V>(a.out + e[u] * d + col, o);
                }
            }
        }
    }
}

// Pass 2 in edge order, when the caller supplies every edge's row
// (edge_row, indexed by edge id; eid then permutes [0, num_items)): logits
// are read and outputs written contiguously, and the rows' statistics --
// small for narrow rows -- are the gathered side.
#ifndef BGL_SOFTMAX_APPLY_MINB
// blocks per SM the edge-order pass's registers are sized for: 1 lets it keep
// two groups' rows and values in registers (128 a thread, 2 blocks per SM);
// sized for 3 or 4 blocks it ran 2-6 % slower on config 2
#define BGL_SOFTMAX_APPLY_MINB 1
#endif
template <typename T, int V, int CV>
__global__ void __launch_bounds__(kSoftBlock, BGL_SOFTMAX_APPLY_MINB) k_softmax_apply_edges(const SoftArgs<T> a) {
    if (a.gate && *a.gate == 0) return;
    constexpr int UN = 4;
    const int c = (threadIdx.x & 31) % CV;
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / CV;
    const int64_t teams = ((int64_t)gridDim.x * blockDim.x) / CV;
    const int32_t cvn = a.d / V;
    const int64_t d = a.d;
    const int64_t step = teams * UN;
    for (int32_t cb = 0; cb < cvn; cb += CV) {
        const int32_t cv = cb + c;
        if (cv >= cvn) break;
        const int64_t col = (int64_t)cv * V;
        // the rows of the group after this one are read one iteration ahead,
        // so a group's statistics and logits loads wait on nothing
        int32_t r[UN], rn[UN];
        auto rows_of = [&](int64_t e0, int32_t(&rr)[UN]) {
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                const int64_t e = e0 + u * teams;
                rr[u] = e < a.num_items ? __ldg(a.edge_row + e) : -1;
            }
        };
        rows_of(team, rn);
        for (int64_t e0 = team; e0 < a.num_items; e0 += step) {
#pragma unroll
            for (int u = 0; u < UN; ++u) r[u] = rn[u];
            rows_of(e0 + step, rn);
            T z[UN][V], m[UN][V], rr[UN][V];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (r[u] >= 0) {
                    load_once<T, V>(a.logits + (e0 + u * teams) * d + col, z[u]);
                    load_vec<T, V>(a.row_m + (int64_t)r[u] * a.rstride + col, m[u]);
                    load_vec<T, V>(a.row_r + (int64_t)r[u] * a.rstride + col, rr[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (r[u] >= 0) {
                    T o[V];
#pragma unroll
                    for (int v = 0; v < V; ++v)
                        o[v] = Arith<T>::mul(Arith<T>::ex(Arith<T>::sub(z[u][v], m[u][v])), rr[u][v]);
                    store_stream<T, V>(a.out + (e0 + u * teams) * d + col, o);
                }
            }
        }
    }
}

// ------------------------------------------------ contiguous segments
// segment_softmax (items are the consecutive rows of `logits`, eid the
// identity): a warp takes whole segments.  It reads a segment's rows once for
// the per-column (max, sum) -- one online update per value, the lanes of a
// column joined by shuffles -- and straight after reads them again for the
// output, so the second read is served by L2: DRAM sees every value read once
// and written once, where the merge-path passes (statistics over all chunks,
// then the output) read it twice.  The lanes cover RPS = 32 / CV rows at a
// time, CV 16-byte vectors a row.  A segment longer than kSegLong rows would
// hold its warp far longer than the others: the kernel leaves it and sets the
// gate, and the merge-path passes (gated on it) compute every row.
constexpr int64_t kSegLong = 4096;
#ifndef BGL_SEG_UN
#define BGL_SEG_UN 6  // rows a lane loads before folding them (4: 6.04 ms, 6: 5.79, 8: 6.62 on config 5)
#endif
#ifndef BGL_SEG_MINB
#define BGL_SEG_MINB 2  // resident blocks per SM the register budget allows
#endif

template <typename T, int CV>
__global__ void __launch_bounds__(kSoftBlock, BGL_SEG_MINB) k_seg_softmax(const SoftArgs<T> a,
                                                                          int *gate) {
    constexpr int V = 16 / (int)sizeof(T);
    constexpr int RPS = 32 / CV;
    constexpr int UN = BGL_SEG_UN;
    const int lane = threadIdx.x & 31;
    const int c = lane % CV, r0 = lane / CV;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t d = a.d;
    for (int64_t seg = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; seg < a.num_rows;
         seg += nwarps) {
        const int64_t i0 = a.indptr[seg], len = a.indptr[seg + 1] - i0;
        if (len <= 0) continue;
        if (len > kSegLong) {
            if (lane == 0) *gate = 1;
            continue;
        }
        const T *zin = a.logits + i0 * d + c * V;
        T m[V], sm[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            m[v] = Arith<T>::ninf();
            sm[v] = T(0);
        }
        int64_t r = r0;
        for (; r + (UN - 1) * RPS < len; r += UN * RPS) {
            T z[UN][V];
#pragma unroll
            for (int u = 0; u < UN; ++u) load_vec<T, V>(zin + (r + u * RPS) * d, z[u]);
#pragma unroll
            for (int u = 0; u < UN; ++u)
#pragma unroll
                for (int v = 0; v < V; ++v) online<T>(m[v], sm[v], z[u][v]);
        }
        for (; r < len; r += RPS) {
            T z[V];
            load_vec<T, V>(zin + r * d, z);
#pragma unroll
            for (int v = 0; v < V; ++v) online<T>(m[v], sm[v], z[v]);
        }
        // the lanes holding the same column vector (lane ^ k CV) join their pieces
#pragma unroll
        for (int off = CV; off < 32; off <<= 1)
#pragma unroll
            for (int v = 0; v < V; ++v) {
                const T m2 = __shfl_xor_sync(kFull, m[v], off);
                const T s2 = __shfl_xor_sync(kFull, sm[v], off);
                combine<T>(m[v], sm[v], m2, s2);
            }
        T rr[V];
#pragma unroll
        for (int v = 0; v < V; ++v) rr[v] = Arith<T>::div(T(1), sm[v]);
        T *zout = a.out + i0 * d + c * V;
        r = r0;
        for (; r + (UN - 1) * RPS < len; r += UN * RPS) {
            T z[UN][V];
#pragma unroll
            for (int u = 0; u < UN; ++u) load_vec<T, V>(zin + (r + u * RPS) * d, z[u]);
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                T o[V];
#pragma unroll
                for (int v = 0; v < V; ++v)
                    o[v] = Arith<T>::mul(Arith<T>::ex(Arith<T>::sub(z[u][v], m[v])), rr[v]);
                store_stream<T, V>(zout + (r + u * RPS) * d, o);
            }
        }
        for (; r < len; r += RPS) {
            T z[V], o[V];
            load_vec<T, V>(zin + r * d, z);
#pragma unroll
            for (int v = 0; v < V; ++v)
                o[v] = Arith<T>::mul(Arith<T>::ex(Arith<T>::sub(z[v], m[v])), rr[v]);
            store_stream<T, V>(zout + r * d, o);
        }
    }
}

// One wave of resident blocks (the SM count times the blocks an SM holds at
// this kernel's register count), the warps striding over the segments: a
// fixed cap of eight blocks an SM ran 2.7 waves at three resident, the last
// one partly empty (28.6 % of the SM's warps active in a config-5 capture).
template <typename T, int CV>
int launch_seg_cv(const SoftArgs<T> &a, int *gate, cudaStream_t s) {
    auto k = k_seg_softmax<T, CV>;
    int per_sm = 0;
    BGL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kSoftBlock, 0));
    if (per_sm < 1) per_sm = 1;
    const int64_t blocks = (a.num_rows * 32 + kSoftBlock - 1) / kSoftBlock;
    const int64_t cap = int64_t(num_sms()) * per_sm;
    const int grid = (int)(blocks < 1 ? 1 : blocks > cap ? cap : blocks);
    k<<<grid, kSoftBlock, 0, s>>>(a, gate);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

template <typename T>
int launch_seg(const SoftArgs<T> &a, int cv, int *gate, cudaStream_t s) {
    switch (cv) {
    case 1: return launch_seg_cv<T, 1>(a, gate, s);
    case 2: return launch_seg_cv<T, 2>(a, gate, s);
    case 4: return launch_seg_cv<T, 4>(a, gate, s);
    case 8: return launch_seg_cv<T, 8>(a, gate, s);
    case 16: return launch_seg_cv<T, 16>(a, gate, s);
    case 32: return launch_seg_cv<T, 32>(a, gate, s);
    }
    return fail(BGL_E_INVALID, "softmax: no segment pass for %d vectors", cv);
}

struct SoftPlan {
    int vmax;  // widest vector the row width allows
    int64_t num_chunks, items, split_min;
};

SoftPlan softmax_plan(int64_t rows, int64_t items, int64_t d, int dtype) {
    SoftPlan p;
    const int vm = dtype == BGL_F32 ? 4 : 2;
    p.vmax = (d % vm == 0) ? vm : 1;
    const int64_t total = rows + items;
    // one warp per chunk, about four chunks per resident warp; the lane walk
    // (items of at most kLaneBytes) takes two waves of 24 warps per SM, so
    // each lane's run is long against the warp scan that ends it
    const bool lane = d * (dtype == BGL_F32 ? 4 : 8) <= kLaneBytes;
    int64_t target = int64_t(num_sms()) * (lane ? 24 * BGL_SOFTMAX_LANE_WAVES : 64 * 4);
    const int64_t per_chunk = 4 * (d > 0 ? d : 1) * (dtype == BGL_F32 ? 4 : 8);
    const int64_t cap = (int64_t(256) << 20) / per_chunk;
    if (target > cap) target = cap;
    int64_t by_items = (total + params().spmm_min_items - 1) / params().spmm_min_items;
    p.num_chunks = by_items < target ? by_items : target;
    if (p.num_chunks < 1) p.num_chunks = 1;
    p.items = (total + p.num_chunks - 1) / p.num_chunks;
    if (p.items < 1) p.items = 1;
    p.split_min = p.items > params().spmm_split_min ? p.items : params().spmm_split_min;
    return p;
}

template <typename T>
struct SoftLayout {
    Coord *coords;
    int32_t *head_row, *tail_row;
    T *head_m, *head_s, *tail_m, *tail_s;
    T *row_m, *row_r;
    int32_t *item_row;
    int *flag;  // segment-per-warp pass: set when the merge-path passes must run
    size_t bytes;
};

template <typename T>
SoftLayout<T> softmax_layout(void *ws, const SoftPlan &p, int64_t rows, int64_t items, int64_t d) {
    Carver c(ws);
    SoftLayout<T> l;
    l.coords = c.take<Coord>(p.num_chunks + 1);
    l.head_row = c.take<int32_t>(p.num_chunks);
    l.tail_row = c.take<int32_t>(p.num_chunks);
    l.head_m = c.take<T>(p.num_chunks * d);
    l.head_s = c.take<T>(p.num_chunks * d);
    l.tail_m = c.take<T>(p.num_chunks * d);
    l.tail_s = c.take<T>(p.num_chunks * d);
    l.row_m = c.take<T>(rows * 2 * d);
    l.row_r = l.row_m + d;
    l.item_row = c.take<int32_t>(items);
    l.flag = c.take<int>(4);
    l.bytes = c.used + 256;
    return l;
}

size_t softmax_ws(int64_t rows, int64_t items, int64_t d, int dtype) {
    SoftPlan p = softmax_plan(rows, items, d, dtype);
    if (dtype == BGL_F32) return softmax_layout<float>(nullptr, p, rows, items, d).bytes;
    return softmax_layout<double>(nullptr, p, rows, items, d).bytes;
}

// After a warp-per-chunk statistics pass: the split rows' fixup, then the
// item pass.
template <typename T, int V, int CV>
int launch_finish(const SoftArgs<T> &a, int grid, cudaStream_t s) {
    k_softmax_fixup<T><<<grid, kSoftBlock, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    // the item pass: enough teams to fill the GPU a few times over
    int64_t teams = (int64_t)a.num_items;
    const int64_t cap = int64_t(num_sms()) * 2048 / CV * 2;
    if (teams > cap) teams = cap;
    const int agrid = (int)((teams * CV + kSoftBlock - 1) / kSoftBlock);
    if (a.edge_row)
        k_softmax_apply_edges<T, V, CV><<<agrid < 1 ? 1 : agrid, kSoftBlock, 0, s>>>(a);
    else
        k_softmax_apply<T, V, CV><<<agrid < 1 ? 1 : agrid, kSoftBlock, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

template <typename T, int V, int CV>
int launch_softmax(const SoftArgs<T> &a, cudaStream_t s) {
    constexpr int R = BGL_SOFTMAX_DEPTH + 1;
    constexpr int smem = R * kSoftBlock * (V * (int)sizeof(T) + 4);
    auto ks = k_softmax_stats<T, V, CV>;
    BGL_CUDA(cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int grid = (int)((a.num_chunks * 32 + kSoftBlock - 1) / kSoftBlock);
    ks<<<grid, kSoftBlock, smem, s>>>(a);
    BGL_LAUNCH_CHECK();
    return launch_finish<T, V, CV>(a, grid, s);
}

template <typename T, int V, int L>
int launch_lane(const SoftArgs<T> &a, cudaStream_t s) {
    constexpr int smem = LaneRing<T, V, L>::smem;
    auto ks = k_softmax_lane_stats<T, V, L>;
    BGL_CUDA(cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    BGL_CUDA(cudaFuncSetAttribute(ks, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  cudaSharedmemCarveoutMaxShared));
    const int grid = (int)((a.num_chunks * 32 + kSoftBlock - 1) / kSoftBlock);
    ks<<<grid, kSoftBlock, smem, s>>>(a);
    BGL_LAUNCH_CHECK();
    return launch_finish<T, V, L>(a, grid, s);
}

template <typename T, int V>
int launch_walk(const SoftArgs<T> &a, int ts, cudaStream_t s) {
    constexpr int smem = WalkRing<T, V>::smem;
    auto ks = k_softmax_walk_stats<T, V>;
    auto ka = k_softmax_walk_apply<T, V>;
    BGL_CUDA(cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    BGL_CUDA(cudaFuncSetAttribute(ks, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  cudaSharedmemCarveoutMaxShared));
    BGL_CUDA(cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    BGL_CUDA(cudaFuncSetAttribute(ka, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  cudaSharedmemCarveoutMaxShared));
    const int grid = (int)((a.num_chunks * ts + kSoftBlock - 1) / kSoftBlock);
    ks<<<grid, kSoftBlock, smem, s>>>(a, ts);
    BGL_LAUNCH_CHECK();
    const int fgrid = (int)((a.num_chunks * 32 + kSoftBlock - 1) / kSoftBlock);
    k_softmax_fixup<T><<<fgrid, kSoftBlock, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    ka<<<grid, kSoftBlock, smem, s>>>(a, ts);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

// Items of at most kLaneBytes: the lane walk, nv = the item's column vectors
// (lanes per run).
template <typename T, int V>
int launch_by_nv(const SoftArgs<T> &a, int nv, cudaStream_t s) {
    switch (nv) {
    case 1: return launch_lane<T, V, 1>(a, s);
    case 2: return launch_lane<T, V, 2>(a, s);
    case 4: return launch_lane<T, V, 4>(a, s);
    case 8:
        if constexpr (V * 8 * sizeof(T) <= kLaneBytes) return launch_lane<T, V, 8>(a, s);
        break;
    case 16:
        if constexpr (V * 16 * sizeof(T) <= kLaneBytes) return launch_lane<T, V, 16>(a, s);
        break;
    default: break;
    }
    return fail(BGL_E_INVALID, "softmax: no lane walk for %d vectors", nv);
}

template <typename T, int V>
int launch_by_cv(const SoftArgs<T> &a, int cv, cudaStream_t s) {
    // 16 or more lanes per item: the team walk; fewer: the warp-wide steps
    switch (cv) {
    case 1: return launch_softmax<T, V, 1>(a, s);
    case 2: return launch_softmax<T, V, 2>(a, s);
    case 4: return launch_softmax<T, V, 4>(a, s);
    case 8: return launch_softmax<T, V, 8>(a, s);
    default: return launch_walk<T, V>(a, cv, s);
    }
}

template <typename T>
int run_softmax(const int64_t *indptr, const int32_t *eid, const int8_t *mask, int64_t rows,
                int64_t items, const void *logits, void *out, int64_t d, int dtype, void *ws,
                cudaStream_t s, const int32_t *edge_row = nullptr) {
    SoftPlan p = softmax_plan(rows, items, d, dtype);
    SoftLayout<T> l = softmax_layout<T>(ws, p, rows, items, d);
    constexpr int VM = sizeof(T) == 4 ? 4 : 2;
    int V = p.vmax;
    if (V > 1 && (!aligned(logits, V * sizeof(T)) || !aligned(out, V * sizeof(T)))) V = 1;
    const int64_t cvn = d / V;
    const int cv = next_pow2(cvn > 32 ? 32 : (int)cvn);
    SoftArgs<T> a{indptr,   eid,        mask,       (int32_t)rows, (int32_t)items,
                  (const T *)logits, (T *)out, (int32_t)d, p.num_chunks, l.coords,
                  l.head_row, l.tail_row, l.head_m, l.head_s,      l.tail_m,
                  l.tail_s, l.row_m,    l.row_r,    l.item_row, edge_row, 2 * d, nullptr};
    // segment_softmax with rows of whole 16-byte vectors: the segment-per-warp
    // pass; the merge-path passes below then run only if it left a segment
    const int64_t rvec = d * (int64_t)sizeof(T) / 16;
    if (!eid && !mask && !edge_row && params().softmax_segment_warp &&
        (d * (int64_t)sizeof(T)) % 16 == 0 && rvec <= 32 && (rvec & (rvec - 1)) == 0 &&
        aligned(logits, 16) && aligned(out, 16)) {
        BGL_CUDA(cudaMemsetAsync(l.flag, 0, sizeof(int), s));
        int rc = launch_seg<T>(a, (int)rvec, l.flag, s);
        if (rc) return rc;
        a.gate = l.flag;
    }
    int cg = (int)((p.num_chunks + 1 + 255) / 256);
    k_spmm_coords<<<cg, 256, 0, s>>>(indptr, rows, items, p.items, p.split_min, p.num_chunks,
                                     l.coords);
    BGL_LAUNCH_CHECK();
    if (d * (int64_t)sizeof(T) <= kLaneBytes) {
        if (V == 1) return launch_by_nv<T, 1>(a, cv, s);
        return launch_by_nv<T, VM>(a, cv, s);
    }
    if (V == 1) return launch_by_cv<T, 1>(a, cv, s);
    return launch_by_cv<T, VM>(a, cv, s);
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_softmax_workspace_size(int64_t num_rows, int64_t num_items, int64_t d, int dtype) {
    if (num_rows < 0 || num_items < 0 || d < 0) return 0;
    if (dtype != BGL_F32 && dtype != BGL_F64) return 0;
    return softmax_ws(num_rows, num_items, d, dtype);
}

int bgl_edge_softmax(const int64_t *indptr, const int32_t *eid, const int8_t *mask,
                     int64_t num_rows, int64_t num_items, const void *logits, void *out,
                     int64_t d, int dtype, void *workspace, size_t workspace_bytes,
                     void *stream) {
    if (dtype != BGL_F32 && dtype != BGL_F64)
        return fail(BGL_E_UNSUPPORTED, "bgl_edge_softmax: dtype %d (f32 and f64 only)", dtype);
    if (num_rows < 0 || num_items < 0 || d < 0)
        return fail(BGL_E_INVALID, "bgl_edge_softmax: negative size");
    if (num_rows >= (int64_t(1) << 31) || num_items >= (int64_t(1) << 31) || d >= (int64_t(1) << 31))
        return fail(BGL_E_UNSUPPORTED, "bgl_edge_softmax: sizes must be below 2^31");
    if (num_rows == 0 || num_items == 0 || d == 0) return BGL_OK;
    if (!indptr || !logits || !out) return fail(BGL_E_INVALID, "bgl_edge_softmax: null buffer");
    const size_t need = softmax_ws(num_rows, num_items, d, dtype);
    if (workspace_bytes < need || !workspace)
        return fail(BGL_E_WORKSPACE, "bgl_edge_softmax: workspace %zu < %zu bytes", workspace_bytes,
                    need);
    cudaStream_t s = as_stream(stream);
    if (dtype == BGL_F32)
        return run_softmax<float>(indptr, eid, mask, num_rows, num_items, logits, out, d, dtype,
                                  workspace, s);
    return run_softmax<double>(indptr, eid, mask, num_rows, num_items, logits, out, d, dtype,
                               workspace, s);
}

int bgl_edge_softmax_by_edge(const int64_t *indptr, const int32_t *eid, const int32_t *edge_row,
                             int64_t num_rows, int64_t num_items, const void *logits, void *out,
                             int64_t d, int dtype, void *workspace, size_t workspace_bytes,
                             void *stream) {
    if (!edge_row) return fail(BGL_E_INVALID, "bgl_edge_softmax_by_edge: null edge_row");
    if (dtype != BGL_F32 && dtype != BGL_F64)
        return fail(BGL_E_UNSUPPORTED, "bgl_edge_softmax_by_edge: dtype %d (f32 and f64 only)", dtype);
    if (num_rows < 0 || num_items < 0 || d < 0)
        return fail(BGL_E_INVALID, "bgl_edge_softmax_by_edge: negative size");
    if (num_rows >= (int64_t(1) << 31) || num_items >= (int64_t(1) << 31) || d >= (int64_t(1) << 31))
        return fail(BGL_E_UNSUPPORTED, "bgl_edge_softmax_by_edge: sizes must be below 2^31");
    if (num_rows == 0 || num_items == 0 || d == 0) return BGL_OK;
    if (!indptr || !logits || !out) return fail(BGL_E_INVALID, "bgl_edge_softmax_by_edge: null buffer");
    const size_t need = softmax_ws(num_rows, num_items, d, dtype);
    if (workspace_bytes < need || !workspace)
        return fail(BGL_E_WORKSPACE, "bgl_edge_softmax_by_edge: workspace %zu < %zu bytes",
                    workspace_bytes, need);
    cudaStream_t s = as_stream(stream);
    if (dtype == BGL_F32)
        return run_softmax<float>(indptr, eid, nullptr, num_rows, num_items, logits, out, d, dtype,
                                  workspace, s, edge_row);
    return run_softmax<double>(indptr, eid, nullptr, num_rows, num_items, logits, out, d, dtype,
                               workspace, s, edge_row);
}

}  // extern "C"
