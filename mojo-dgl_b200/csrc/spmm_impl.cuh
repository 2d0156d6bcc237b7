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

// Max / min computed for their values only (no arg output asked for): the
// same comparisons without the winning position, one select per value.
constexpr int kRedMaxValue = 16, kRedMinValue = 17;

template <int RED, typename T>
__device__ __forceinline__ T identity() {
    if (RED == BGL_RED_MAX || RED == kRedMaxValue) return Arith<T>::ninf();
    if (RED == BGL_RED_MIN || RED == kRedMinValue) return Arith<T>::pinf();
    return T(0);
}

// Folds message m (at CSR position p) into the running value.
template <int RED, typename T>
__device__ __forceinline__ void fold(T &acc, int32_t &pos, T m, int32_t p) {
    if (RED == BGL_RED_MAX) {
        if (m > acc) { acc = m; pos = p; }
    } else if (RED == BGL_RED_MIN) {
        if (m < acc) { acc = m; pos = p; }
    } else if (RED == kRedMaxValue) {
        acc = m > acc ? m : acc;
    } else if (RED == kRedMinValue) {
        acc = m < acc ? m : acc;
    } else {
            acc = Arith<T>::add(acc, m);
    }
}

// A lane's V arg indices: 16-byte stores where the address allows (V even),
// so a warp's instruction covers whole sectors instead of one word in each.
template <int V>
__device__ __forceinline__ void store_i64(int64_t *p, const int64_t (&w)[V]) {
    if constexpr (V % 2 == 0) {
        if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < V; i += 2)
                *reinterpret_cast<longlong2 *>(p + i) = make_longlong2(w[i], w[i + 1]);
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = w[i];
}

// Writes one finished row: the mean divide, the inf->0 post-pass and the arg
// indices are all applied here, so the row is written once.  In accumulate
// mode the row is first folded into what `out` already holds (a partial result
// over other edges of the same rows): sums add, max/min keep the better value,
// and on a tie the smaller edge id -- the earlier message in CSR order -- wins.
// `row_len` is the row's CSR length when the caller already holds it (the
// main pass does), else -1.
template <typename T, int RED, int V, int J, bool ACC>
__device__ __forceinline__ void emit_row(const SpmmArgs<T> &a, int64_t row, int64_t cb, int t,
                                         int64_t cvn, const T (&acc)[J][V],
                                         const int32_t (&pos)[J][V], int64_t row_len) {
    T scale = T(1);
    constexpr bool MEAN = RED == BGL_RED_MEAN;  // a sum divided by the in-degree
    if (MEAN) {
        int64_t dg = a.deg                ? a.deg[row]
                     : row_len >= 0 ? row_len
                                    : a.indptr[row + 1] - a.indptr[row];
        scale = dg < 1 ? T(1) : T(dg);
    }
    constexpr bool ARG = RED == BGL_RED_MAX || RED == BGL_RED_MIN;
    if constexpr (!ACC) {
#pragma unroll
        for (int j = 0; j < J; ++j) {
            int64_t cv = cb + t + (int64_t)j * a.ts;
            if (cv >= cvn) continue;
            int64_t off = row * a.dout + cv * V;
            T o[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                T v = acc[j][i];
                if (MEAN) v = Arith<T>::div(v, scale);
                if (a.zero_inf && isinf(v)) v = T(0);
                o[i] = v;
            }
            store_vec<T, V>(a.out + off, o);
            if (ARG) {
                int64_t w[V];
                if (a.arg_u) {
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        const int32_t p = pos[j][i];
                        w[i] = p < 0 ? -1 : (int64_t)a.indices[p];
                    }
                    store_i64<V>(a.arg_u + off, w);
                }
                if (a.arg_e) {
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        const int32_t p = pos[j][i];
                        w[i] = p < 0 ? -1 : (a.eid ? (int64_t)a.eid[p] : (int64_t)p);
                    }
                    store_i64<V>(a.arg_e + off, w);
                }
            }
        }
    } else {
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
            {
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
                    } else if (RED == kRedMaxValue) {
                        o[i] = acc[j][i] > old[i] ? acc[j][i] : old[i];
                    } else if (RED == kRedMinValue) {
                        o[i] = acc[j][i] < old[i] ? acc[j][i] : old[i];
                    } else {
                        o[i] = Arith<T>::add(old[i], acc[j][i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < V; ++i) {
                T v = o[i];
                if (MEAN) v = Arith<T>::div(v, scale);
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

// The gather pipeline.  A team walks its chunk's edges in groups of UN; the
// rows of the next P groups are already being copied into the lane's shared
// slots (cp.async) while the current group is folded, so each lane keeps
// P * UN rows in flight without holding them in registers.  A ring of
// P + 1 stages lets the copy for group g + P go into the stage that group g - 1
// was folded from, whose values the fold has already consumed.
#ifndef BGL_SPMM_UN
#define BGL_SPMM_UN 4  // edges per group, copy ops (one gathered row per edge)
#endif
#ifndef BGL_SPMM_UN_BIN
#define BGL_SPMM_UN_BIN 1  // edges per group when both operands are gathered
#endif
#ifndef BGL_SPMM_DEPTH
#define BGL_SPMM_DEPTH 3  // groups in flight ahead of the one being folded
#endif
#ifndef BGL_SPMM_DEPTH_BIN
#define BGL_SPMM_DEPTH_BIN 4
#endif
#ifndef BGL_SPMM_MAXB
#define BGL_SPMM_MAXB 3  // resident blocks a launch asks for at most
#endif
#ifndef BGL_SPMM_DEPTH_NARROW
#define BGL_SPMM_DEPTH_NARROW 2  // the narrow ring (float copy ops, teams under a warp)
#endif
#ifndef BGL_SPMM_MAXB_NARROW
#define BGL_SPMM_MAXB_NARROW 4
#endif
// Measured on config 3 (125M edges, 128 fp32 columns) and config 2: copy ops
// run best with groups of 4 and 3 in flight at three blocks per SM (copy_u sum
// 9.5 ms; groups of 2 x 6, 3 x 4, 6 x 2, or any two-block ring: 10.2-10.9 ms);
// binary ops with single-edge groups 4 deep (u_mul_e 19.5 ms on config 3,
// 12.1 ms on config 2; 2 x 3: 21.1 / 14.0 ms).  Re-measured on the cp.async
// ring just before the operand modes became template constants (config 3's
// (E,128) edge feature / config 2's head broadcast):
// 1 x 4: 18.5 / 9.2 ms; 2 x 3: 18.4 / 9.4; 2 x 4: 19.3 / 10.1; 4 x 2: 18.8 /
// 9.8 ms -- the choice stands.
constexpr int kSpmmBlock = 256;
constexpr int kSmemPerSm = 228 * 1024;  // shared memory per SM, 1 KB of it reserved per block

template <typename T, int OP, int V, bool NARROW = false>
struct Stages {
    static constexpr bool both = OP != BGL_OP_COPY_LHS && OP != BGL_OP_COPY_RHS;
    static_assert(!(NARROW && both), "the narrow ring is for copy ops");
    static constexpr int un = both ? BGL_SPMM_UN_BIN : BGL_SPMM_UN;
    static constexpr int depth = both ? BGL_SPMM_DEPTH_BIN
                                 : NARROW ? BGL_SPMM_DEPTH_NARROW : BGL_SPMM_DEPTH;
    static constexpr int ring = depth + 1;
    static constexpr int nops = both ? 2 : 1;
    static constexpr int slot = V * (int)sizeof(T);  // bytes per lane per operand row
    static constexpr int smem = ring * un * nops * kSpmmBlock * slot;
    // resident blocks the ring allows, at most three (85 registers a
    // thread), four for the narrow ring (64 registers)
    static constexpr int maxb = NARROW ? BGL_SPMM_MAXB_NARROW : BGL_SPMM_MAXB;
    static constexpr int fit = kSmemPerSm / (smem + 1024);
    static constexpr int minb = fit < 1 ? 1 : fit > maxb ? maxb : fit;
    static_assert(smem <= 227 * 1024, "gather ring larger than a block's shared memory");
};

// The main pass.  A team walks its chunk's edge range [c0.y, c1.y) in full
// groups of UN edges regardless of where rows end -- a group can close one
// row and open the next -- so the copy pipeline never drains at a row end.
// Row ends are handled as the group is folded, in CSR order, so the
// arithmetic is exactly the per-row sequential fold.
// LM / RM: the operands' column modes (lane_cols: 0 full rows, 1 a uniform
// broadcast, 2 per element) when the launch knows them, -1 to read them at
// run time.  A known mode folds every mode branch and slot stride of the
// per-edge copy and read-back into constants.
template <typename T, int OP, int RED, int V, int J, bool ACC, int LM = -1, int RM = -1,
          bool NARROW = false>
__global__ void __launch_bounds__(kSpmmBlock, (Stages<T, OP, V, NARROW>::minb))
    k_spmm(const SpmmArgs<T> a) {
    static_assert(J == 1, "the staged gather keeps one column vector per lane");
    using S = Stages<T, OP, V, NARROW>;
    constexpr int UN = S::un, P = S::depth, R = S::ring;
    constexpr bool NEED_L = OP != BGL_OP_COPY_RHS;
    constexpr bool NEED_R = OP != BGL_OP_COPY_LHS;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // each operand has its own region of slots (stage, u, thread), packed at
    // the size the operand copies per lane -- V values, or one for a uniform
    // broadcast -- so the lanes of a warp touch adjacent words: the copies and
    // the read-backs are free of bank conflicts
    const uint32_t s0 = smem_addr(smem_raw);
    constexpr uint32_t region = (uint32_t)R * UN * kSpmmBlock * S::slot;
    auto slot_at = [](int stage, int u, int op, uint32_t stride) -> uint32_t {
        return op * region + ((uint32_t)(stage * UN + u) * kSpmmBlock + threadIdx.x) * stride;
    };

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
    for (int32_t cb = slice * ts; cb < cvn; cb += a.num_slices * ts) {
        int32_t x = x0;
        if (x >= nrows) break;  // an empty trailing chunk
        const int32_t cv = cb + t;  // this lane's column vector (may be past the row)
        const bool live = cv < cvn;
        const int64_t k0 = (int64_t)cv * V;
        int32_t rs = (int32_t)indptr[x];
        int32_t re = (x < x1) ? (int32_t)indptr[x + 1] : ye;
        int32_t row_begin = y0;  // first edge of the current row in this chunk
        T acc[J][V];
        int32_t pos[J][V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
            acc[0][i] = identity<RED, T>();
            pos[0][i] = -1;
        }
        // closes row x (emitted, or stored as a head piece if it began in an
        // earlier chunk) and opens row x + 1
        auto close_row = [&]() {
            if (row_begin == rs) {
                emit_row<T, RED, V, J, ACC>(a, x, cb, t, cvn, acc, pos, re - rs);
            } else {
                store_piece<T, RED, V, J>(a, a.head_val, a.head_pos, chunk, cb, t, cvn, acc, pos);
                head_row = x;
            }
            row_begin = re;
            rs = re;
            ++x;
            re = (x < x1) ? (int32_t)indptr[x + 1] : ye;
#pragma unroll
            for (int i = 0; i < V; ++i) {
                acc[0][i] = identity<RED, T>();
                pos[0][i] = -1;
            }
        };

        // the lane's columns of each operand, fixed for the walk
        LaneCols<T, V> lc, rc;
        uint32_t lstride = S::slot, rstride = S::slot;  // bytes per slot
        if (NEED_L) {
            lc = lane_cols<T, V>(a.lhs, k0);
            if (LM >= 0) lc.mode = LM;
            if (lc.mode == 1) lstride = sizeof(T);
        }
        if (NEED_R) {
            rc = lane_cols<T, V>(a.rhs, k0);
            if (RM >= 0) rc.mode = RM;
            if (rc.mode == 1) rstride = sizeof(T);
        }

        // ids of the next group to copy, fetched one group ahead of its copy;
        // only a chunk's last group needs a bound on every edge
        int32_t src[UN], edg[UN];
        int32_t e_copy = y0;
        auto fetch_one = [&](int u) {
            if (NEED_L) src[u] = __ldg(a.indices + e_copy + u);
            if (NEED_R) edg[u] = a.eid ? __ldg(a.eid + e_copy + u) : e_copy + u;
        };
        auto fetch_ids = [&]() {
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
            if (NEED_L) stage_row<T, V>(lc, a.lhs, src[u], s0 + slot_at(stage, u, 0, lstride));
            if (NEED_R)
                stage_row<T, V>(rc, a.rhs, edg[u], s0 + slot_at(stage, u, S::nops - 1, rstride));
        };
        auto copy_group = [&](int stage) {
            if (live) {  // a lane past the row's last column copies nothing
                if (e_copy + UN <= ye) {
#pragma unroll
                    for (int u = 0; u < UN; ++u) copy_one(stage, u);
                } else {
#pragma unroll
                    for (int u = 0; u < UN; ++u)
                        if (e_copy + u < ye) copy_one(stage, u);
                }
            }
            cp_async_commit();  // an empty group past the chunk end keeps the count
            e_copy += UN;
            fetch_ids();
        };
        // folds edge e from slot (stage, u); a lane past the row's last column
        // folds whatever its slot holds and never stores it
        auto fold_one = [&](int stage, int u, int32_t e) {
            while (e >= re) close_row();
            T lv[V], rv[V];
            if (NEED_L)
                read_row<T, V>(lc, reinterpret_cast<const T *>(smem_raw + slot_at(stage, u, 0, lstride)), lv);
            if (NEED_R)
                read_row<T, V>(rc, reinterpret_cast<const T *>(
                                       smem_raw + slot_at(stage, u, S::nops - 1, rstride)), rv);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                T m = message<OP, T>(NEED_L ? lv[i] : T(0), NEED_R ? rv[i] : T(0));
                fold<RED, T>(acc[0][i], pos[0][i], m, e);
            }
        };
        fetch_ids();
#pragma unroll
        for (int g = 0; g < P; ++g) copy_group(g);
        int fold_stage = 0, copy_stage = P;
        for (int32_t e0 = y0; e0 < ye; e0 += UN) {
            copy_group(copy_stage);
            cp_async_wait<P>();  // the group at e0 has landed
            if (e0 + UN <= ye) {
#pragma unroll
                for (int u = 0; u < UN; ++u) fold_one(fold_stage, u, e0 + u);
            } else {
#pragma unroll
                for (int u = 0; u < UN; ++u)
                    if (e0 + u < ye) fold_one(fold_stage, u, e0 + u);
            }
            fold_stage = fold_stage + 1 == R ? 0 : fold_stage + 1;
            copy_stage = copy_stage + 1 == R ? 0 : copy_stage + 1;
        }
        cp_async_wait<0>();
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

// The first of the chunks whose pieces make up split row `row`, which ends in
// `chunk`: the chunks before it whose tail piece belongs to the row.  The
// team (ts lanes, a power of two <= 32, all of them calling) probes ts chunks
// per step, so a hub spread over hundreds of chunks costs a few dependent
// loads rather than one per chunk.
template <typename R>
__device__ __forceinline__ int64_t first_piece(const R *__restrict__ tail_row, int64_t chunk,
                                               int64_t row, int t, int ts) {
    const int base = (threadIdx.x & 31) & ~(ts - 1);
    const unsigned team = ts == 32 ? 0xffffffffu : ((1u << ts) - 1) << base;
    int64_t first = chunk;
    while (first > 0) {
        const int64_t q = first - 1 - t;
        const bool same = q >= 0 && (int64_t)tail_row[q] == row;
        const unsigned brk = __ballot_sync(team, !same) >> base;
        if (brk) return first - (__ffs(brk) - 1);
        first -= ts;
    }
    return first;
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
    const int64_t first = first_piece(a.tail_row, chunk, row, t, ts);
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
        // unrolled so that several pieces' loads are in flight at once
#pragma unroll 4
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
        emit_row<T, RED, V, J, ACC>(a, row, cb, t, cvn, acc, pos, -1);
    }
}

// Launches main + fixup for one (T, V, J) with runtime op/reduce dispatch.
template <typename T, int V, int J>
int launch_spmm_vj(const SpmmArgs<T> &a, int op, int red, cudaStream_t s);

}  // namespace bgl
