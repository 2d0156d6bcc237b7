// Fused per-row softmax over a CSR (replaces mdgl_edge_softmax_,
// src/ported.mojo:876-1080, and mdgl_segment_softmax, src/ported.mojo:660-768).
//
// Both reference kernels compute, for each CSR row and each column h, over the
// row's selected items e,
//     out[e, h] = exp(z[e, h] - max) / sum exp(z[., h] - max).
// edge_softmax reaches the items through the CSR's edge ids; segment_softmax's
// items are the consecutive rows of `value` (eid = identity).
//
// Work split: the gSpMM engine's merge path over (row ends, items), so a team
// of lanes gets the same number of items whatever the degrees are -- a
// 50,000-edge attention hub is spread over many teams.  Lanes own V adjacent
// columns; a team streams its chunk's items in groups of UN across row ends and
// folds, per column, an online (max, sum of exp(z - max)) pair: a larger z
// rescales the running sum by exp(old max - z).  A row that closes inside the
// chunk stores its (max, sum) in a per-row buffer; a row split over chunks
// leaves one (max, sum) piece per chunk and the fixup kernel folds the pieces
// in CSR order into the row's entry.  The write pass then streams the same
// chunks again and writes exp(z - max) / sum, reloading the stats only when
// it crosses a row end -- no team ever runs a per-row loop the other teams of
// its warp would have to wait for.
// The online sum rounds differently from the reference's max-then-sum passes
// (and CUDA's exp is not the Mojo stdlib's), so results are compared with a
// relative tolerance (1e-12 in float64).
#include "spmm_impl.cuh"

#ifndef BGL_SOFTMAX_MINB
#define BGL_SOFTMAX_MINB 1  // resident 256-thread blocks per SM the registers must allow
#endif

namespace bgl {
namespace {

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
    int32_t ts;
    int64_t num_chunks;
    const Coord *coords;
    int32_t *head_row;
    int32_t *tail_row;
    T *head_m, *head_s, *tail_m, *tail_s;  // per chunk x d: the split rows' pieces
    T *row_m, *row_s;                      // per row x d: each row's final (max, sum)
};

template <typename T>
__device__ __forceinline__ void online(T &m, T &s, T z) {
    if (z > m) {
        s = Arith<T>::add(Arith<T>::mul(s, Arith<T>::ex(Arith<T>::sub(m, z))), T(1));
        m = z;
    } else {
        s = Arith<T>::add(s, Arith<T>::ex(Arith<T>::sub(z, m)));
    }
}

template <typename T>
__device__ __forceinline__ void combine(T &m, T &s, T m2, T s2) {
    if (m2 == Arith<T>::ninf()) return;
    if (m == Arith<T>::ninf()) {
        m = m2;
        s = s2;
    } else if (m2 > m) {
        s = Arith<T>::add(Arith<T>::mul(s, Arith<T>::ex(Arith<T>::sub(m, m2))), s2);
        m = m2;
    } else {
        s = Arith<T>::add(s, Arith<T>::mul(s2, Arith<T>::ex(Arith<T>::sub(m2, m))));
    }
}

template <typename T>
__device__ __forceinline__ int64_t item_id(const SoftArgs<T> &a, int32_t i) {
    return a.eid ? (int64_t)__ldg(a.eid + i) : (int64_t)i;
}

// One group of UN consecutive items of a lane's column vector.
template <typename T, int V, int UN>
struct Group {
    int64_t e[UN];
    bool sel[UN];
    T z[UN][V];
};

template <typename T, int V, int UN>
__device__ __forceinline__ void load_group(const SoftArgs<T> &a, int32_t i0, int32_t ye, int32_t cv,
                                           Group<T, V, UN> &g) {
#pragma unroll
    for (int u = 0; u < UN; ++u) {
        g.sel[u] = false;
        if (i0 + u < ye) {
            g.e[u] = item_id(a, i0 + u);
            g.sel[u] = !a.mask || a.mask[g.e[u]] == 1;
            if (g.sel[u]) ld_stream(a.logits + g.e[u] * a.d + (int64_t)cv * V, g.z[u]);
        }
    }
}

template <typename T, int V>
__device__ __forceinline__ void put_stats(T *pm, T *ps, int64_t slot, int32_t d, int32_t cv,
                                          const T (&m)[V], const T (&s)[V]) {
#pragma unroll
    for (int k = 0; k < V; ++k) {
        pm[slot * d + (int64_t)cv * V + k] = m[k];
        ps[slot * d + (int64_t)cv * V + k] = s[k];
    }
}

// Pass 1: per-row (max, sum) for every row, pieces for split rows.
template <typename T, int V>
__global__ void __launch_bounds__(256, BGL_SOFTMAX_MINB) k_softmax_stats(const SoftArgs<T> a) {
    constexpr int UN = V == 1 ? 8 : 4;
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t x1 = (int32_t)a.coords[chunk + 1].x, ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t cvn = a.d / V;
    int32_t head_row = -1, tail_row = -1;
    for (int32_t cv = t; cv < cvn; cv += ts) {
        int32_t x = x0;
        if (x >= a.num_rows) break;
        int32_t rs = (int32_t)a.indptr[x];
        int32_t re = (x < x1) ? (int32_t)a.indptr[x + 1] : ye;
        int32_t row_begin = y0;
        T m[V], s[V];
#pragma unroll
        for (int k = 0; k < V; ++k) {
            m[k] = Arith<T>::ninf();
            s[k] = T(0);
        }
        auto close_row = [&]() {
            if (row_begin == rs) {
                put_stats<T, V>(a.row_m, a.row_s, x, a.d, cv, m, s);
            } else {
                put_stats<T, V>(a.head_m, a.head_s, chunk, a.d, cv, m, s);
                head_row = x;
            }
            row_begin = re;
            rs = re;
            ++x;
            re = (x < x1) ? (int32_t)a.indptr[x + 1] : ye;
#pragma unroll
            for (int k = 0; k < V; ++k) {
                m[k] = Arith<T>::ninf();
                s[k] = T(0);
            }
        };
        for (int32_t i0 = y0; i0 < ye; i0 += UN) {
            Group<T, V, UN> g;
            load_group<T, V, UN>(a, i0, ye, cv, g);
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (i0 + u < ye) {
                    while (i0 + u >= re) close_row();
                    if (g.sel[u]) {
#pragma unroll
                        for (int k = 0; k < V; ++k) online(m[k], s[k], g.z[u][k]);
                    }
                }
            }
        }
        while (x < x1) close_row();
        if (x < a.num_rows && ye > row_begin) {
            put_stats<T, V>(a.tail_m, a.tail_s, chunk, a.d, cv, m, s);
            tail_row = x;
        }
    }
    if (t == 0) {
        a.head_row[chunk] = head_row;
        a.tail_row[chunk] = tail_row;
    }
}

// Pass 2: fold every split row's pieces in CSR order into its row entry.
template <typename T>
__global__ void k_softmax_fixup(const SoftArgs<T> a) {
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int32_t row = a.head_row[chunk];
    if (row < 0) return;
    int64_t first = chunk;
    while (first > 0 && a.tail_row[first - 1] == row) --first;
    for (int32_t h = t; h < a.d; h += ts) {
        T m = Arith<T>::ninf(), s = T(0);
        for (int64_t q = first; q < chunk; ++q) combine(m, s, a.tail_m[q * a.d + h], a.tail_s[q * a.d + h]);
        combine(m, s, a.head_m[chunk * a.d + h], a.head_s[chunk * a.d + h]);
        a.row_m[(int64_t)row * a.d + h] = m;
        a.row_s[(int64_t)row * a.d + h] = s;
    }
}

// Pass 3: out = exp(z - max) * (1 / sum) over the same chunks; a row's stats
// are loaded (and its sum inverted) when the walk enters it.
template <typename T, int V>
__global__ void __launch_bounds__(256, BGL_SOFTMAX_MINB) k_softmax_write(const SoftArgs<T> a) {
    constexpr int UN = V == 1 ? 8 : 4;
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t cvn = a.d / V;
    for (int32_t cv = t; cv < cvn; cv += ts) {
        int32_t x = x0;
        if (x >= a.num_rows || y0 >= ye) break;
        int32_t re = (int32_t)a.indptr[x + 1];
        T m[V], r[V];  // the row's max and the reciprocal of its sum
        auto load_stats = [&]() {
            T sum[V];
            load_vec<T, V>(a.row_m + (int64_t)x * a.d + (int64_t)cv * V, m);
            load_vec<T, V>(a.row_s + (int64_t)x * a.d + (int64_t)cv * V, sum);
#pragma unroll
            for (int k = 0; k < V; ++k) r[k] = Arith<T>::div(T(1), sum[k]);
        };
        while (y0 >= re) {  // rows that end before the first item (empty rows)
            ++x;
            re = (int32_t)a.indptr[x + 1];
        }
        load_stats();
        for (int32_t i0 = y0; i0 < ye; i0 += UN) {
            Group<T, V, UN> g;
            load_group<T, V, UN>(a, i0, ye, cv, g);
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (i0 + u < ye) {
                    if (i0 + u >= re) {
                        do {
                            ++x;
                            re = (int32_t)a.indptr[x + 1];
                        } while (i0 + u >= re);
                        load_stats();
                    }
                    if (g.sel[u]) {
                        T o[V];
#pragma unroll
                        for (int k = 0; k < V; ++k)
                            o[k] = Arith<T>::mul(Arith<T>::ex(Arith<T>::sub(g.z[u][k], m[k])), r[k]);
                        store_vec<T, V>(a.out + g.e[u] * a.d + (int64_t)cv * V, o);
                    }
                }
            }
        }
    }
}

struct SoftPlan {
    int vmax;
    int ts;
    int64_t num_chunks, items, split_min;
};

SoftPlan softmax_plan(int64_t rows, int64_t items, int64_t d, int dtype) {
    SoftPlan p;
    const int vm = dtype == BGL_F32 ? 4 : 2;
    p.vmax = (d % vm == 0) ? vm : 1;
    const int64_t cvn = d / p.vmax;
    p.ts = next_pow2(cvn < 1 ? 1 : cvn);
    const int64_t total = rows + items;
    int64_t target = int64_t(num_sms()) * 48 * (32 / p.ts) * 3;
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
    T *row_m, *row_s;
    size_t bytes;
};

template <typename T>
SoftLayout<T> softmax_layout(void *ws, const SoftPlan &p, int64_t rows, int64_t d) {
    Carver c(ws);
    SoftLayout<T> l;
    l.coords = c.take<Coord>(p.num_chunks + 1);
    l.head_row = c.take<int32_t>(p.num_chunks);
    l.tail_row = c.take<int32_t>(p.num_chunks);
    l.head_m = c.take<T>(p.num_chunks * d);
    l.head_s = c.take<T>(p.num_chunks * d);
    l.tail_m = c.take<T>(p.num_chunks * d);
    l.tail_s = c.take<T>(p.num_chunks * d);
    l.row_m = c.take<T>(rows * d);
    l.row_s = c.take<T>(rows * d);
    l.bytes = c.used + 256;
    return l;
}

size_t softmax_ws(int64_t rows, int64_t items, int64_t d, int dtype) {
    SoftPlan p = softmax_plan(rows, items, d, dtype);
    if (dtype == BGL_F32) return softmax_layout<float>(nullptr, p, rows, d).bytes;
    return softmax_layout<double>(nullptr, p, rows, d).bytes;
}

template <typename T>
int run_softmax(const int64_t *indptr, const int32_t *eid, const int8_t *mask, int64_t rows,
                int64_t items, const void *logits, void *out, int64_t d, int dtype, void *ws,
                cudaStream_t s) {
    SoftPlan p = softmax_plan(rows, items, d, dtype);
    SoftLayout<T> l = softmax_layout<T>(ws, p, rows, d);
    constexpr int VM = sizeof(T) == 4 ? 4 : 2;
    int V = p.vmax;
    if (V > 1 && (!aligned(logits, V * sizeof(T)) || !aligned(out, V * sizeof(T)))) V = 1;
    SoftArgs<T> a{indptr,   eid,          mask,       (int32_t)rows, (int32_t)items,
                  (const T *)logits, (T *)out, (int32_t)d, p.ts,      p.num_chunks,
                  l.coords, l.head_row,   l.tail_row, l.head_m,      l.head_s,
                  l.tail_m, l.tail_s,     l.row_m,    l.row_s};
    int cg = (int)((p.num_chunks + 1 + 255) / 256);
    k_spmm_coords<<<cg, 256, 0, s>>>(indptr, rows, items, p.items, p.split_min, p.num_chunks,
                                     l.coords);
    BGL_LAUNCH_CHECK();
    const int grid = (int)((p.num_chunks * p.ts + 255) / 256);
    if (V == 1)
        k_softmax_stats<T, 1><<<grid, 256, 0, s>>>(a);
    else
        k_softmax_stats<T, VM><<<grid, 256, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    k_softmax_fixup<T><<<grid, 256, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    if (V == 1)
        k_softmax_write<T, 1><<<grid, 256, 0, s>>>(a);
    else
        k_softmax_write<T, VM><<<grid, 256, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
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

}  // extern "C"
