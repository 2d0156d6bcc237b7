// gSpMM engine (replaces src/ported.mojo:352-548, _gspmm and its dispatch).
//
// Work split: merge-path over the (row ends, edges) sequence of the CSR.  The
// N + E items are cut into equal chunks, one per team of lanes; a boundary
// that falls inside a row no longer than `split_min` edges is moved back to
// that row's start, so only rows longer than a chunk are ever split.  That
// gives every team the same amount of work whatever the degree distribution
// (power-law hubs included) while keeping the reference's arithmetic for all
// ordinary rows: each lane owns V consecutive output columns and folds the
// row's messages in CSR order, one rounding per message and one per add,
// exactly as the reference's per-column loop does (src/ported.mojo:392-422).
//
// A split row leaves one piece per chunk it touches in the workspace; the
// fixup kernel folds the pieces in CSR order (a sum of partial sums, so the
// rounding differs from the sequential loop only for those rows; max/min and
// their arg indices stay exact because a later piece replaces the running
// winner only on a strict improvement, the reference's rule at
// src/ported.mojo:106-109).
#pragma once

#include "common.cuh"

namespace bgl {

struct Coord {
    int64_t x;  // rows finished
    int64_t y;  // edges consumed
};

template <typename T>
struct SpmmArgs {
    const int64_t *indptr;
    const int32_t *indices;
    const int32_t *eid;
    const int64_t *deg;
    int64_t num_rows;
    int64_t num_edges;
    Operand<T> lhs, rhs;
    T *out;
    int64_t dout;
    int64_t *arg_u;
    int64_t *arg_e;
    bool mean;
    bool zero_inf;
    bool accumulate;  // BGL_ACCUMULATE: selects the kernels compiled with ACC = true
    int ts;  // lanes per team (power of two <= 32)
    int32_t num_slices;  // column slices of ts * V columns; one team per (chunk, slice)
    int64_t num_chunks;
    const Coord *coords;  // num_chunks + 1 boundaries
    T *head_val;
    T *tail_val;
    int32_t *head_pos;
    int32_t *tail_pos;
    int64_t *head_row;
    int64_t *tail_row;
};

// Merge-path diagonal search (Merrill & Garland, "Merge-based parallel sparse
// matrix-vector multiplication", SC'16), with the small-row snap.
__device__ __forceinline__ Coord merge_coord(const int64_t *__restrict__ indptr, int64_t n,
                                             int64_t e, int64_t diag, int64_t split_min) {
    int64_t lo = diag - e > 0 ? diag - e : 0;
    int64_t hi = diag < n ? diag : n;
    while (lo < hi) {
        int64_t mid = (lo + hi) >> 1;
        if (indptr[mid + 1] <= diag - mid - 1)
            lo = mid + 1;
        else
            hi = mid;
    }
    Coord c{lo, diag - lo};
    if (c.x < n) {
        int64_t rs = indptr[c.x];
        if (c.y > rs && indptr[c.x + 1] - rs <= split_min) c.y = rs;
    }
    return c;
}

static __global__ void k_spmm_coords(const int64_t *__restrict__ indptr, int64_t n, int64_t e,
                              int64_t items, int64_t split_min, int64_t num_chunks,
                              Coord *__restrict__ coords) {
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c <= num_chunks;
         c += (int64_t)gridDim.x * blockDim.x) {
        int64_t diag = c * items;
        if (diag > n + e) diag = n + e;
        coords[c] = merge_coord(indptr, n, e, diag, split_min);
    }
}

template <int RED, typename T>
__device__ __forceinline__ T identity() {
    if (RED == BGL_RED_MAX) return Arith<T>::ninf();
    if (RED == BGL_RED_MIN) return Arith<T>::pinf();
    return T(0);
}

// Folds message m (at CSR position p) into the running value.
template <int RED, typename T>
__device__ __forceinline__ void fold(T &acc, int32_t &pos, T m, int32_t p) {
    if (RED == BGL_RED_MAX) {
        if (m > acc) { acc = m; pos = p; }
    } else if (RED == BGL_RED_MIN) {
        if (m < acc) { acc = m; pos = p; }
    } else {
        acc = Arith<T>::add(acc, m);
    }
}

// Writes one finished row: the mean divide, the inf->0 post-pass and the arg
// indices are all applied here, so the row is written once.  In accumulate
// mode the row is first folded into what `out` already holds (a partial result
// over other edges of the same rows): sums add, max/min keep the better value,
// and on a tie the smaller edge id -- the earlier message in CSR order -- wins.
template <typename T, int RED, int V, int J, bool ACC>
__device__ __forceinline__ void emit_row(const SpmmArgs<T> &a, int64_t row, int64_t cb, int t,
                                         int64_t cvn, const T (&acc)[J][V],
                                         const int32_t (&pos)[J][V]) {
    T scale = T(1);
    if (a.mean) {
        int64_t dg = a.deg ? a.deg[row] : a.indptr[row + 1] - a.indptr[row];
        scale = dg < 1 ? T(1) : T(dg);
    }
    constexpr bool ARG = RED == BGL_RED_MAX || RED == BGL_RED_MIN;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        int64_t cv = cb + t + (int64_t)j * a.ts;
        if (cv >= cvn) continue;
        int64_t off = row * a.dout + cv * V;
        T o[V];
        int64_t ae[V], au[V];
        bool take[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int32_t p = pos[j][i];
            ae[i] = p < 0 ? -1 : (a.eid ? (int64_t)a.eid[p] : (int64_t)p);
            au[i] = (ARG && a.arg_u && p >= 0) ? (int64_t)a.indices[p] : -1;
            take[i] = true;
        }
        if (ACC) {
            T old[V];
            load_vec<T, V>(a.out + off, old);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                if (ARG) {
                    const int64_t oe = a.arg_e ? a.arg_e[off + i] : -1;
                    const T v = acc[j][i];
                    const bool better = RED == BGL_RED_MAX ? v > old[i] : v < old[i];
                    take[i] = better || (v == old[i] && ae[i] >= 0 && (oe < 0 || ae[i] < oe));
                    o[i] = take[i] ? v : old[i];
                } else {
                    o[i] = Arith<T>::add(old[i], acc[j][i]);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < V; ++i) o[i] = acc[j][i];
        }
#pragma unroll
        for (int i = 0; i < V; ++i) {
            T v = o[i];
            if (a.mean) v = Arith<T>::div(v, scale);
            if (a.zero_inf && isinf(v)) v = T(0);
            o[i] = v;
        }
        store_vec<T, V>(a.out + off, o);
        if (ARG) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                if (!take[i]) continue;
                if (a.arg_u) a.arg_u[off + i] = au[i];
                if (a.arg_e) a.arg_e[off + i] = ae[i];
            }
        }
    }
}

template <typename T, int RED, int V, int J>
__device__ __forceinline__ void store_piece(const SpmmArgs<T> &a, T *val, int32_t *pz,
                                            int64_t chunk, int64_t cb, int t, int64_t cvn,
                                            const T (&acc)[J][V], const int32_t (&pos)[J][V]) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
        int64_t cv = cb + t + (int64_t)j * a.ts;
        if (cv >= cvn) continue;
        int64_t off = chunk * a.dout + cv * V;
        store_vec<T, V>(val + off, acc[j]);
        if (RED == BGL_RED_MAX || RED == BGL_RED_MIN) {
#pragma unroll
            for (int i = 0; i < V; ++i) pz[off + i] = pos[j][i];
        }
    }
}

// Edges a lane keeps in flight: about eight vector loads per lane whatever
// the row width, halved when both operands are gathered.
// Measured on config 3 (125M edges, 128 fp32 columns): 4 edges in flight per
// lane with 4 resident 256-thread blocks per SM (64 registers) ran copy_u sum
// in 10.0 ms and max in 14.9 ms; 8 edges with 3 blocks: 10.0 / 22.2 ms; 8 with
// 2 blocks: 11.2 / 31.7 ms -- occupancy beats per-lane depth once the walk
// streams across row ends.
#ifndef BGL_SPMM_UN
#define BGL_SPMM_UN 4  // edges in flight per lane for rows of <= 32 vectors
#endif
#ifndef BGL_SPMM_MINB
#define BGL_SPMM_MINB 4  // resident 256-thread blocks per SM the registers must allow
#endif
// Ops that gather two rows per edge (u_op_e) keep their own depth and
// occupancy: twice the loads per edge, twice the registers per edge.
#ifndef BGL_SPMM_UN_BIN
#define BGL_SPMM_UN_BIN 2
#endif
#ifndef BGL_SPMM_MINB_BIN
#define BGL_SPMM_MINB_BIN 4
#endif
template <int OP, int J>
struct InFlight {
    static constexpr bool both = OP != BGL_OP_COPY_LHS && OP != BGL_OP_COPY_RHS;
    static constexpr int value = both ? BGL_SPMM_UN_BIN : BGL_SPMM_UN;
    static constexpr int minb = both ? BGL_SPMM_MINB_BIN : BGL_SPMM_MINB;
};

// The main pass.  A team walks its chunk's edge range [c0.y, c1.y) in full
// groups of UN edges regardless of where rows end -- a group can close one
// row and open the next -- so each lane always has UN row loads in flight,
// and the next group's neighbour ids are fetched while the current group's
// rows are still arriving.  Row ends are handled as the group is folded, in
// CSR order, so the arithmetic is exactly the per-row sequential fold.
template <typename T, int OP, int RED, int V, int J, bool ACC>
__global__ void __launch_bounds__(256, (InFlight<OP, J>::minb)) k_spmm(const SpmmArgs<T> a) {
    constexpr int UN = InFlight<OP, J>::value;
    constexpr bool NEED_L = OP != BGL_OP_COPY_RHS;
    constexpr bool NEED_R = OP != BGL_OP_COPY_LHS;
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    // wide rows are cut into column slices, one team per (chunk, slice): the
    // slices of a chunk walk the same edges, and their id loads share L1/L2
    const int64_t chunk = team / a.num_slices;
    const int32_t slice = (int32_t)(team % a.num_slices);
    if (chunk >= a.num_chunks) return;
    // rows and edges are below 2^31 (checked by the host), so the walk
    // bookkeeping stays in 32-bit registers
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t x1 = (int32_t)a.coords[chunk + 1].x, ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t nrows = (int32_t)a.num_rows;
    const int32_t cvn = (int32_t)(a.dout / V);
    const int64_t *__restrict__ indptr = a.indptr;

    int32_t head_row = -1, tail_row = -1;
    for (int32_t cb = slice * ts * J; cb < cvn; cb += a.num_slices * ts * J) {
        int32_t x = x0;
        if (x >= nrows) break;  // an empty trailing chunk
        int32_t rs = (int32_t)indptr[x];
        int32_t re = (x < x1) ? (int32_t)indptr[x + 1] : ye;
        int32_t row_begin = y0;  // first edge of the current row in this chunk
        T acc[J][V];
        int32_t pos[J][V];
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < V; ++i) {
                acc[j][i] = identity<RED, T>();
                pos[j][i] = -1;
            }
        // closes row x (emitted, or stored as a head piece if it began in an
        // earlier chunk) and opens row x + 1
        auto close_row = [&]() {
            if (row_begin == rs) {
                emit_row<T, RED, V, J, ACC>(a, x, cb, t, cvn, acc, pos);
            } else {
                store_piece<T, RED, V, J>(a, a.head_val, a.head_pos, chunk, cb, t, cvn, acc, pos);
                head_row = x;
            }
            row_begin = re;
            rs = re;
            ++x;
            re = (x < x1) ? (int32_t)indptr[x + 1] : ye;
#pragma unroll
            for (int j = 0; j < J; ++j)
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    acc[j][i] = identity<RED, T>();
                    pos[j][i] = -1;
                }
        };

        // this lane's columns in each operand, fixed for the whole walk (J = 1)
        ColMap<V> lmap[J], rmap[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int64_t k0 = (int64_t)(cb + t + j * ts) * V;
            if (NEED_L) lmap[j] = col_map<T, V>(a.lhs, k0);
            if (NEED_R) rmap[j] = col_map<T, V>(a.rhs, k0);
        }
        int32_t src[UN], edg[UN];
        auto fetch_ids = [&](int32_t e0, int32_t(&s)[UN], int32_t(&d)[UN]) {
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (e0 + u < ye) {
                    if (NEED_L) s[u] = __ldg(a.indices + e0 + u);
                    if (NEED_R) d[u] = a.eid ? __ldg(a.eid + e0 + u) : e0 + u;
                }
            }
        };
        fetch_ids(y0, src, edg);
        for (int32_t e0 = y0; e0 < ye; e0 += UN) {
            const int n = (ye - e0) < UN ? (ye - e0) : UN;
            T lv[UN][J][V], rv[UN][J][V];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (u < n) {
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        const int32_t cv = cb + t + j * ts;
                        if (cv < cvn) {
                            if (NEED_L) load_mapped<T, V>(a.lhs, src[u], lmap[j], lv[u][j]);
                            if (NEED_R) load_mapped<T, V>(a.rhs, edg[u], rmap[j], rv[u][j]);
                        }
                    }
                }
            }
            int32_t nsrc[UN], nedg[UN];
            fetch_ids(e0 + UN, nsrc, nedg);
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (u < n) {
                    const int32_t e = e0 + u;
                    while (e >= re) close_row();
#pragma unroll
                    for (int j = 0; j < J; ++j)
#pragma unroll
                        for (int i = 0; i < V; ++i) {
                            T m = message<OP, T>(NEED_L ? lv[u][j][i] : T(0),
                                                 NEED_R ? rv[u][j][i] : T(0));
                            fold<RED, T>(acc[j][i], pos[j][i], m, e);
                        }
                }
            }
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                src[u] = nsrc[u];
                edg[u] = nedg[u];
            }
        }
        while (x < x1) close_row();  // rows ending at the chunk end, empty rows
        if (x < nrows && ye > row_begin) {
            // row x continues into the next chunk: its first (or middle) piece
            store_piece<T, RED, V, J>(a, a.tail_val, a.tail_pos, chunk, cb, t, cvn, acc, pos);
            tail_row = x;
        }
    }
    if (t == 0 && slice == 0) {
        a.head_row[chunk] = head_row;
        a.tail_row[chunk] = tail_row;
    }
}

// Folds the pieces of every split row in CSR order and writes the row.
template <typename T, int RED, int V, int J, bool ACC>
__global__ void __launch_bounds__(256) k_spmm_fixup(const SpmmArgs<T> a) {
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int64_t row = a.head_row[chunk];
    if (row < 0) return;
    int64_t first = chunk;
    while (first > 0 && a.tail_row[first - 1] == row) --first;
    const int64_t cvn = a.dout / V;
    for (int64_t cb = 0; cb < cvn; cb += (int64_t)ts * J) {
        T acc[J][V];
        int32_t pos[J][V];
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < V; ++i) {
                acc[j][i] = identity<RED, T>();
                pos[j][i] = -1;
            }
        for (int64_t q = first; q <= chunk; ++q) {
            const T *val = (q == chunk) ? a.head_val : a.tail_val;
            const int32_t *pz = (q == chunk) ? a.head_pos : a.tail_pos;
#pragma unroll
            for (int j = 0; j < J; ++j) {
                int64_t cv = cb + t + (int64_t)j * ts;
                if (cv >= cvn) continue;
                int64_t off = q * a.dout + cv * V;
                T pv[V];
                load_vec<T, V>(val + off, pv);
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    int32_t pp = (RED == BGL_RED_MAX || RED == BGL_RED_MIN) ? pz[off + i] : 0;
                    fold<RED, T>(acc[j][i], pos[j][i], pv[i], pp);
                }
            }
        }
        emit_row<T, RED, V, J, ACC>(a, row, cb, t, cvn, acc, pos);
    }
}

// Launches main + fixup for one (T, V, J) with runtime op/reduce dispatch.
template <typename T, int V, int J>
int launch_spmm_vj(const SpmmArgs<T> &a, int op, int red, cudaStream_t s);

}  // namespace bgl
