// Fused GAT aggregation: the chain u_add_v -> leaky_relu -> edge_softmax(dst)
// -> u_mul_e_sum of the reference's operators (ops/sddmm.py, ops/edge_softmax.py,
// ops/spmm.py; src/ported.mojo:204-329, 876-1080, 352-423) in one pass over
// the in-CSR, with no per-edge score or attention array:
//     s_e     = leaky_relu(el[u_e, h] + er[v, h])
//     a_e     = exp(s_e - max_v) / sum_{e' -> v} exp(s_e' - max_v)
//     out[v, h, :] = sum_{e -> v} a_e feat[u_e, h, :]
// Each lane owns V columns of one head and keeps, for its destination row, a
// running maximum M, the sum S of exp(s - M) and the weighted feature sum A:
// an edge with a larger score rescales (S, A) by exp(M - s) and enters with
// weight 1, any other edge enters with weight exp(s - M) -- one exponential per
// edge and head.  The row is written as A / S when it closes.
//
// The walk is the gSpMM engine's: merge-path chunks over (row ends, edges),
// a team of lanes per chunk, the source's feature columns and its el value
// staged per lane through a cp.async ring.  A row split over chunks leaves
// one (M, S, A) piece per chunk, folded in CSR order by the fixup kernel.
// The rounding differs from the unfused chain (a sum of rescaled terms and
// one divide instead of per-edge attention weights), so results are compared
// with a relative tolerance.
#include "spmm_impl.cuh"

namespace bgl {
namespace {

constexpr int kGatBlock = 256;
constexpr int kGatDepth = 4;  // single-edge groups in flight ahead of the fold

template <typename T>
struct GatArgs {
    const int64_t *indptr;
    const int32_t *indices;
    int32_t num_rows;
    int32_t num_edges;
    const T *feat;  // (src nodes, heads * head_dim)
    const T *el;    // (src nodes, heads)
    const T *er;    // (rows, heads)
    T *out;         // (rows, heads * head_dim)
    int32_t heads, head_dim, dout;
    T slope;
    int ts;
    int32_t num_slices;
    int64_t num_chunks;
    const Coord *coords;
    int64_t *head_row, *tail_row;
    T *head_m, *head_s, *head_a, *tail_m, *tail_s, *tail_a;  // per chunk x dout
};

// (M, S, A) <- the statistics of (M, S, A)'s edges followed by (m2, s2, a2)'s.
template <typename T, int V>
__device__ __forceinline__ void gat_combine(T &M, T &S, T (&A)[V], T m2, T s2, const T (&a2)[V]) {
    if (m2 == Arith<T>::ninf()) return;
    if (M == Arith<T>::ninf()) {
        M = m2;
        S = s2;
#pragma unroll
        for (int i = 0; i < V; ++i) A[i] = a2[i];
        return;
    }
    const T mx = m2 > M ? m2 : M;
    const T c1 = Arith<T>::ex(Arith<T>::sub(M, mx)), c2 = Arith<T>::ex(Arith<T>::sub(m2, mx));
    S = Arith<T>::add(Arith<T>::mul(S, c1), Arith<T>::mul(s2, c2));
#pragma unroll
    for (int i = 0; i < V; ++i) A[i] = Arith<T>::add(Arith<T>::mul(A[i], c1), Arith<T>::mul(a2[i], c2));
    M = mx;
}

template <typename T, int V>
__device__ __forceinline__ void gat_write(const GatArgs<T> &a, int64_t row, int64_t col, T S,
                                          const T (&A)[V]) {
    T o[V];
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = S > T(0) ? Arith<T>::div(A[i], S) : T(0);
    store_vec<T, V>(a.out + row * a.dout + col, o);
}

template <typename T, int V>
__device__ __forceinline__ void gat_piece(T *pm, T *ps, T *pa, int64_t off, T M, T S, const T (&A)[V]) {
    T m[V], s[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        m[i] = M;
        s[i] = S;
    }
    store_vec<T, V>(pm + off, m);
    store_vec<T, V>(ps + off, s);
    store_vec<T, V>(pa + off, A);
}

template <typename T, int V>
__global__ void __launch_bounds__(kGatBlock, 3) k_gat(const GatArgs<T> a) {
    constexpr int P = kGatDepth, R = P + 1;
    constexpr uint32_t FSLOT = V * sizeof(T);  // feature bytes per lane per edge
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t s0 = smem_addr(smem_raw);
    constexpr uint32_t fregion = (uint32_t)R * kGatBlock * FSLOT;
    // slots: features [stage][thread] (V values), then el [stage][thread] (one value)
    auto fslot = [](int stage) { return ((uint32_t)stage * kGatBlock + threadIdx.x) * FSLOT; };
    auto eslot = [](int stage) {
        return fregion + ((uint32_t)stage * kGatBlock + threadIdx.x) * (uint32_t)sizeof(T);
    };

    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    const int64_t chunk = team / a.num_slices;
    const int32_t slice = (int32_t)(team % a.num_slices);
    if (chunk >= a.num_chunks) return;
    const int32_t x0 = (int32_t)a.coords[chunk].x, y0 = (int32_t)a.coords[chunk].y;
    const int32_t x1 = (int32_t)a.coords[chunk + 1].x, ye = (int32_t)a.coords[chunk + 1].y;
    const int32_t nrows = a.num_rows;
    const int32_t cvn = a.dout / V;
    const int64_t *__restrict__ indptr = a.indptr;

    int64_t head_row = -1, tail_row = -1;
    for (int32_t cb = slice * ts; cb < cvn; cb += a.num_slices * ts) {
        int32_t x = x0;
        if (x >= nrows) break;
        const int32_t cv = cb + t;
        const bool live = cv < cvn;
        const int32_t col = cv * V;
        const int32_t h = live ? col / a.head_dim : 0;  // the lane's head
        const char *fbase = reinterpret_cast<const char *>(a.feat + col);
        const char *ebase = reinterpret_cast<const char *>(a.el + h);
        const uint32_t frow = (uint32_t)a.dout * sizeof(T), erow = (uint32_t)a.heads * sizeof(T);

        int32_t rs = (int32_t)indptr[x];
        int32_t re = (x < x1) ? (int32_t)indptr[x + 1] : ye;
        int32_t row_begin = y0;
        T er_row = live && x < nrows ? __ldg(a.er + (int64_t)x * a.heads + h) : T(0);
        T M = Arith<T>::ninf(), S = T(0), A[V];
#pragma unroll
        for (int i = 0; i < V; ++i) A[i] = T(0);
        auto close_row = [&]() {
            if (live) {
                if (row_begin == rs)
                    gat_write<T, V>(a, x, col, S, A);
                else
                    gat_piece<T, V>(a.head_m, a.head_s, a.head_a, chunk * a.dout + col, M, S, A);
            }
            if (row_begin != rs) head_row = x;
            row_begin = re;
            rs = re;
            ++x;
            re = (x < x1) ? (int32_t)indptr[x + 1] : ye;
            if (live && x < nrows) er_row = __ldg(a.er + (int64_t)x * a.heads + h);
            M = Arith<T>::ninf();
            S = T(0);
#pragma unroll
            for (int i = 0; i < V; ++i) A[i] = T(0);
        };

        int32_t e_copy = y0, src = 0;
        auto fetch = [&]() {
            if (e_copy < ye) src = __ldg(a.indices + e_copy);
        };
        auto copy_edge = [&](int stage) {
            if (live && e_copy < ye) {
                cp_async<FSLOT>(s0 + fslot(stage), fbase + (uint64_t)(uint32_t)src * frow);
                cp_async<sizeof(T)>(s0 + eslot(stage), ebase + (uint64_t)(uint32_t)src * erow);
            }
            cp_async_commit();
            ++e_copy;
            fetch();
        };
        fetch();
#pragma unroll
        for (int g = 0; g < P; ++g) copy_edge(g);
        int fstage = 0, cstage = P;
        for (int32_t e = y0; e < ye; ++e) {
            copy_edge(cstage);
            cp_async_wait<P>();
            while (e >= re) close_row();
            // a lane past the row's last column folds whatever its slot holds
            // and never stores it
            T f[V], elv[1];
            lds_vec(s0 + fslot(fstage), f);
            lds_vec(s0 + eslot(fstage), elv);
            const T z = Arith<T>::add(elv[0], er_row);
            const T sc = z > T(0) ? z : Arith<T>::mul(z, a.slope);
            const T d = Arith<T>::sub(sc, M);
            const T w = Arith<T>::ex(d > T(0) ? -d : d);  // exp(-|s - M|)
            // a new maximum rescales what came before by w and enters with
            // weight 1; any other score enters with weight w -- selects, not
            // a branch (the two heads of a warp would diverge)
            const bool up = sc > M;
            const T c1 = up ? w : T(1), c2 = up ? T(1) : w;
            S = Arith<T>::fma(S, c1, c2);
#pragma unroll
            for (int i = 0; i < V; ++i) A[i] = Arith<T>::fma(A[i], c1, Arith<T>::mul(c2, f[i]));
            M = up ? sc : M;
            fstage = fstage + 1 == R ? 0 : fstage + 1;
            cstage = cstage + 1 == R ? 0 : cstage + 1;
        }
        cp_async_wait<0>();
        while (x < x1) close_row();
        if (x < nrows && ye > row_begin) {
            if (live) gat_piece<T, V>(a.tail_m, a.tail_s, a.tail_a, chunk * a.dout + col, M, S, A);
            tail_row = x;
        }
    }
    if (t == 0 && slice == 0) {
        a.head_row[chunk] = head_row;
        a.tail_row[chunk] = tail_row;
    }
}

// Folds every split row's pieces in CSR order and writes A / S.
template <typename T, int V>
__global__ void __launch_bounds__(kGatBlock) k_gat_fixup(const GatArgs<T> a) {
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t chunk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    if (chunk >= a.num_chunks) return;
    const int64_t row = a.head_row[chunk];
    if (row < 0) return;
    const int64_t first = first_piece(a.tail_row, chunk, row, t, ts);
    const int32_t cvn = a.dout / V;
    for (int32_t cv = t; cv < cvn; cv += ts) {
        const int64_t col = (int64_t)cv * V;
        T M = Arith<T>::ninf(), S = T(0), A[V];
#pragma unroll
        for (int i = 0; i < V; ++i) A[i] = T(0);
        // unrolled so that several pieces' loads are in flight at once
#pragma unroll 4
        for (int64_t q = first; q <= chunk; ++q) {
            const bool head = q == chunk;
            const int64_t off = q * a.dout + col;
            T m2[V], s2[V], a2[V];
            load_vec<T, V>((head ? a.head_m : a.tail_m) + off, m2);
            load_vec<T, V>((head ? a.head_s : a.tail_s) + off, s2);
            load_vec<T, V>((head ? a.head_a : a.tail_a) + off, a2);
            gat_combine<T, V>(M, S, A, m2[0], s2[0], a2);
        }
        gat_write<T, V>(a, row, col, S, A);
    }
}

struct GatPlan {
    int vmax, ts, slices;
    int64_t num_chunks, items, split_min;
};

GatPlan gat_plan(int64_t n, int64_t e, int64_t heads, int64_t head_dim, int dtype) {
    GatPlan p;
    const int vm = dtype == BGL_F32 ? 4 : 2;
    const int64_t dout = heads * head_dim;
    p.vmax = (head_dim % vm == 0) ? vm : 1;  // a lane's vector stays inside one head
    const int64_t cvn = dout / p.vmax;
    p.ts = next_pow2(cvn < 1 ? 1 : cvn);
    p.slices = (int)((cvn + p.ts - 1) / p.ts);
    if (p.slices < 1) p.slices = 1;
    int64_t target = int64_t(num_sms()) * 48 * (32 / p.ts) * 3 / p.slices;
    if (target < int64_t(num_sms()) * 8) target = int64_t(num_sms()) * 8;
    const int64_t per_chunk = 6 * (dout > 0 ? dout : 1) * (dtype == BGL_F32 ? 4 : 8);
    const int64_t cap = (int64_t(256) << 20) / per_chunk;
    if (target > cap) target = cap;
    if (params().spmm_max_chunks > 0 && target > params().spmm_max_chunks)
        target = params().spmm_max_chunks;
    const int64_t total = n + e;
    const int64_t by_items = (total + params().spmm_min_items - 1) / params().spmm_min_items;
    p.num_chunks = by_items < target ? by_items : target;
    if (p.num_chunks < 1) p.num_chunks = 1;
    p.items = (total + p.num_chunks - 1) / p.num_chunks;
    if (p.items < 1) p.items = 1;
    p.split_min = p.items > params().spmm_split_min ? p.items : params().spmm_split_min;
    return p;
}

template <typename T>
struct GatLayout {
    Coord *coords;
    int64_t *head_row, *tail_row;
    T *head_m, *head_s, *head_a, *tail_m, *tail_s, *tail_a;
    size_t bytes;
};

template <typename T>
GatLayout<T> gat_layout(void *ws, const GatPlan &p, int64_t dout) {
    Carver c(ws);
    GatLayout<T> l;
    l.coords = c.take<Coord>(p.num_chunks + 1);
    l.head_row = c.take<int64_t>(p.num_chunks);
    l.tail_row = c.take<int64_t>(p.num_chunks);
    T **arrays[6] = {&l.head_m, &l.head_s, &l.head_a, &l.tail_m, &l.tail_s, &l.tail_a};
    for (T **a : arrays) *a = c.take<T>(p.num_chunks * dout);
    l.bytes = c.used + 256;
    return l;
}

size_t gat_ws(int64_t n, int64_t e, int64_t heads, int64_t head_dim, int dtype) {
    GatPlan p = gat_plan(n, e, heads, head_dim, dtype);
    if (dtype == BGL_F32) return gat_layout<float>(nullptr, p, heads * head_dim).bytes;
    return gat_layout<double>(nullptr, p, heads * head_dim).bytes;
}

template <typename T, int V>
int launch_gat(const GatArgs<T> &a, cudaStream_t s) {
    constexpr int smem = (kGatDepth + 1) * kGatBlock * (V + 1) * (int)sizeof(T);
    auto k = k_gat<T, V>;
    BGL_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int64_t threads = a.num_chunks * a.num_slices * a.ts;
    int grid = (int)((threads + kGatBlock - 1) / kGatBlock);
    k<<<grid < 1 ? 1 : grid, kGatBlock, smem, s>>>(a);
    BGL_LAUNCH_CHECK();
    const int fgrid = (int)((a.num_chunks * a.ts + kGatBlock - 1) / kGatBlock);
    k_gat_fixup<T, V><<<fgrid < 1 ? 1 : fgrid, kGatBlock, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

template <typename T>
int run_gat(const int64_t *indptr, const int32_t *indices, int64_t n, int64_t e, const void *feat,
            const void *el, const void *er, int64_t heads, int64_t head_dim, double slope,
            void *out, int dtype, void *ws, cudaStream_t s) {
    GatPlan p = gat_plan(n, e, heads, head_dim, dtype);
    const int64_t dout = heads * head_dim;
    GatLayout<T> l = gat_layout<T>(ws, p, dout);
    constexpr int VM = sizeof(T) == 4 ? 4 : 2;
    int V = p.vmax;
    if (V > 1 && (!aligned(feat, V * sizeof(T)) || !aligned(out, V * sizeof(T)))) V = 1;
    const int64_t cvn = dout / V;
    GatArgs<T> a;
    a.indptr = indptr;
    a.indices = indices;
    a.num_rows = (int32_t)n;
    a.num_edges = (int32_t)e;
    a.feat = static_cast<const T *>(feat);
    a.el = static_cast<const T *>(el);
    a.er = static_cast<const T *>(er);
    a.out = static_cast<T *>(out);
    a.heads = (int32_t)heads;
    a.head_dim = (int32_t)head_dim;
    a.dout = (int32_t)dout;
    a.slope = (T)slope;
    a.ts = p.ts;
    a.num_slices = (int32_t)((cvn + p.ts - 1) / p.ts);
    a.num_chunks = p.num_chunks;
    a.coords = l.coords;
    a.head_row = l.head_row;
    a.tail_row = l.tail_row;
    a.head_m = l.head_m;
    a.head_s = l.head_s;
    a.head_a = l.head_a;
    a.tail_m = l.tail_m;
    a.tail_s = l.tail_s;
    a.tail_a = l.tail_a;
    const int cg = (int)((p.num_chunks + 1 + 255) / 256);
    k_spmm_coords<<<cg, 256, 0, s>>>(indptr, n, e, p.items, p.split_min, p.num_chunks, l.coords);
    BGL_LAUNCH_CHECK();
    if (V == 1) return launch_gat<T, 1>(a, s);
    return launch_gat<T, VM>(a, s);
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_gat_workspace_size(int64_t num_rows, int64_t num_edges, int64_t heads, int64_t head_dim,
                              int dtype) {
    if (num_rows < 0 || num_edges < 0 || heads < 0 || head_dim < 0) return 0;
    if (dtype != BGL_F32 && dtype != BGL_F64) return 0;
    return gat_ws(num_rows, num_edges, heads, head_dim, dtype);
}

int bgl_gat_aggregate(const int64_t *indptr, const int32_t *indices, int64_t num_rows,
                      int64_t num_edges, const void *feat, const void *el, const void *er,
                      int64_t heads, int64_t head_dim, double negative_slope, void *out, int dtype,
                      void *workspace, size_t workspace_bytes, void *stream) {
    if (dtype != BGL_F32 && dtype != BGL_F64)
        return fail(BGL_E_UNSUPPORTED, "bgl_gat_aggregate: dtype %d (f32 and f64 only)", dtype);
    if (num_rows < 0 || num_edges < 0 || heads < 0 || head_dim < 0)
        return fail(BGL_E_INVALID, "bgl_gat_aggregate: negative size");
    const int64_t lim = int64_t(1) << 31, elem = dtype == BGL_F32 ? 4 : 8;
    if (num_rows >= lim || num_edges >= lim || heads * head_dim * elem >= 2 * lim)
        return fail(BGL_E_UNSUPPORTED, "bgl_gat_aggregate: sizes beyond the 32-bit walk");
    if (num_rows == 0 || heads == 0 || head_dim == 0) return BGL_OK;
    if (!indptr || !out || !er || (num_edges > 0 && (!indices || !feat || !el)))
        return fail(BGL_E_INVALID, "bgl_gat_aggregate: null buffer");
    const size_t need = gat_ws(num_rows, num_edges, heads, head_dim, dtype);
    if (workspace_bytes < need || !workspace)
        return fail(BGL_E_WORKSPACE, "bgl_gat_aggregate: workspace %zu < %zu bytes",
                    workspace_bytes, need);
    cudaStream_t s = as_stream(stream);
    if (dtype == BGL_F32)
        return run_gat<float>(indptr, indices, num_rows, num_edges, feat, el, er, heads, head_dim,
                              negative_slope, out, dtype, workspace, s);
    return run_gat<double>(indptr, indices, num_rows, num_edges, feat, el, er, heads, head_dim,
                           negative_slope, out, dtype, workspace, s);
}

}  // extern "C"
