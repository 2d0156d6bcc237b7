// Host side of the gSpMM engine: planning, workspace layout, validation and
// dispatch of bgl_gspmm (the replacement for mdgl_gspmm, src/capi.mojo:95-115).
#include "spmm_impl.cuh"

namespace bgl {

struct SpmmPlan {
    int vmax;     // widest vector the row width allows
    int ts;       // lanes per team
    int slices;   // column slices of ts * vmax columns (one team each)
    int64_t num_chunks;
    int64_t items;
    int64_t split_min;
};

static int vec_limit(int dtype) { return dtype == BGL_F32 ? 4 : 2; }

// Deterministic in (rows, edges, dout, dtype, reduce) and the device's SM
// count, so the workspace query and the call agree and repeated calls split
// rows identically (bitwise-reproducible results).
static SpmmPlan spmm_plan(int64_t n, int64_t e, int64_t dout, int dtype, int reduce) {
    SpmmPlan p;
    int vm = vec_limit(dtype);
    p.vmax = (dout % vm == 0) ? vm : 1;
    int64_t cvn = p.vmax ? dout / p.vmax : dout;
    p.ts = next_pow2(cvn < 1 ? 1 : cvn);
    p.slices = (int)((cvn + p.ts - 1) / p.ts);
    if (p.slices < 1) p.slices = 1;
    int64_t total = n + e;
    int64_t teams_per_warp = 32 / p.ts;
    int64_t target = int64_t(num_sms()) * 48 * teams_per_warp * 3 / p.slices;
    if (target < int64_t(num_sms()) * 8) target = int64_t(num_sms()) * 8;
    // bound the split-row piece buffers to ~256 MB
    size_t elem = (dtype == BGL_F32 ? 4 : 8) + ((reduce == BGL_RED_MAX || reduce == BGL_RED_MIN) ? 4 : 0);
    int64_t per_chunk = 2 * (dout > 0 ? dout : 1) * (int64_t)elem;
    int64_t mem_cap = (int64_t(256) << 20) / per_chunk;
    if (target > mem_cap) target = mem_cap;
    if (params().spmm_max_chunks > 0 && target > params().spmm_max_chunks)
        target = params().spmm_max_chunks;
    int64_t by_items = (total + params().spmm_min_items - 1) / params().spmm_min_items;
    p.num_chunks = by_items < target ? by_items : target;
    if (p.num_chunks < 1) p.num_chunks = 1;
    p.items = (total + p.num_chunks - 1) / p.num_chunks;
    if (p.items < 1) p.items = 1;
    // a row is split only when it is longer than both a chunk and the
    // split floor, so every ordinary row keeps the sequential CSR-order sum
    p.split_min = p.items > params().spmm_split_min ? p.items : params().spmm_split_min;
    return p;
}

template <typename T>
struct SpmmLayout {
    Coord *coords;
    int64_t *head_row, *tail_row;
    T *head_val, *tail_val;
    int32_t *head_pos, *tail_pos;
    size_t bytes;
};

template <typename T>
static SpmmLayout<T> spmm_layout(void *ws, const SpmmPlan &p, int64_t dout, int reduce) {
    Carver c(ws);
    SpmmLayout<T> l;
    l.coords = c.take<Coord>(p.num_chunks + 1);
    l.head_row = c.take<int64_t>(p.num_chunks);
    l.tail_row = c.take<int64_t>(p.num_chunks);
    l.head_val = c.take<T>(p.num_chunks * dout);
    l.tail_val = c.take<T>(p.num_chunks * dout);
    bool arg = reduce == BGL_RED_MAX || reduce == BGL_RED_MIN;
    l.head_pos = arg ? c.take<int32_t>(p.num_chunks * dout) : nullptr;
    l.tail_pos = arg ? c.take<int32_t>(p.num_chunks * dout) : nullptr;
    l.bytes = c.used + 256;
    return l;
}

static size_t spmm_ws_bytes(int64_t n, int64_t e, int64_t dout, int dtype, int reduce) {
    SpmmPlan p = spmm_plan(n, e, dout, dtype, reduce);
    if (dtype == BGL_F32) return spmm_layout<float>(nullptr, p, dout, reduce).bytes;
    return spmm_layout<double>(nullptr, p, dout, reduce).bytes;
}

template <typename T>
static int run_spmm(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
                    const int64_t *deg, int64_t n, int64_t e, const void *lhs, int64_t lw,
                    int64_t ldiv, const void *rhs, int64_t rw, int64_t rdiv, void *out,
                    int64_t dout, int64_t *arg_u, int64_t *arg_e, int dtype, int op, int red,
                    int flags, void *ws, cudaStream_t s) {
    SpmmPlan p = spmm_plan(n, e, dout, dtype, red);
    SpmmLayout<T> l = spmm_layout<T>(ws, p, dout, red);
    const bool need_l = op != BGL_OP_COPY_RHS, need_r = op != BGL_OP_COPY_LHS;
    const bool lfull = ldiv == 1 && lw == dout, rfull = rdiv == 1 && rw == dout;

    // vector width: the plan's, unless an operand read as full rows or the
    // output is not aligned to it
    int V = p.vmax;
    const size_t vb = size_t(V) * sizeof(T);
    if (V > 1 && (!aligned(out, vb) || (need_l && lfull && !aligned(lhs, vb)) ||
                  (need_r && rfull && !aligned(rhs, vb))))
        V = 1;
    // the plan's slices assume its vector width; with V = 1 a team covers
    // ts columns, so the slice count grows accordingly
    const int64_t cvn = dout / V;
    const int slices = (int)((cvn + p.ts - 1) / p.ts);

    SpmmArgs<T> a;
    a.indptr = indptr;
    a.indices = indices;
    a.eid = eid;
    a.deg = deg;
    a.num_rows = n;
    a.num_edges = e;
    a.lhs = Operand<T>{static_cast<const T *>(lhs), lw, ldiv, lfull, (ldiv % V == 0) || lw == 1};
    a.rhs = Operand<T>{static_cast<const T *>(rhs), rw, rdiv, rfull, (rdiv % V == 0) || rw == 1};
    a.out = static_cast<T *>(out);
    a.dout = dout;
    a.arg_u = (red == BGL_RED_MAX || red == BGL_RED_MIN) ? arg_u : nullptr;
    a.arg_e = (red == BGL_RED_MAX || red == BGL_RED_MIN) ? arg_e : nullptr;
    a.zero_inf = (flags & BGL_ZERO_INF) != 0;
    a.accumulate = (flags & BGL_ACCUMULATE) != 0;
    a.ts = p.ts;
    a.num_slices = slices;
    a.num_chunks = p.num_chunks;
    a.coords = l.coords;
    a.head_val = l.head_val;
    a.tail_val = l.tail_val;
    a.head_pos = l.head_pos;
    a.tail_pos = l.tail_pos;
    a.head_row = l.head_row;
    a.tail_row = l.tail_row;

    int cg = (int)((p.num_chunks + 1 + 255) / 256);
    k_spmm_coords<<<cg, 256, 0, s>>>(indptr, n, e, p.items, p.split_min, p.num_chunks, l.coords);
    BGL_LAUNCH_CHECK();
    constexpr int VM = sizeof(T) == 4 ? 4 : 2;
    if (V == 1) return launch_spmm_vj<T, 1, 1>(a, op, red, s);
    return launch_spmm_vj<T, VM, 1>(a, op, red, s);
}

}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_gspmm_workspace_size(int64_t num_rows, int64_t num_edges, int64_t dout, int dtype,
                                int reduce) {
    if (num_rows < 0 || num_edges < 0 || dout < 0) return 0;
    if (dtype != BGL_F32 && dtype != BGL_F64) return 0;
    return spmm_ws_bytes(num_rows, num_edges, dout, dtype, reduce);
}

int bgl_gspmm(const int64_t *indptr, const int32_t *indices, const int32_t *eid,
              const int64_t *deg, int64_t num_rows, int64_t num_edges, const void *lhs,
              int64_t lhs_width, int64_t lhs_div, const void *rhs, int64_t rhs_width,
              int64_t rhs_div, void *out, int64_t dout, int64_t *arg_u, int64_t *arg_e,
              int dtype, int op, int reduce, int flags, void *workspace, size_t workspace_bytes,
              void *stream) {
    if (dtype != BGL_F32 && dtype != BGL_F64)
        return fail(BGL_E_UNSUPPORTED, "bgl_gspmm: dtype %d (f32 and f64 only)", dtype);
    if (op < BGL_OP_ADD || op > BGL_OP_COPY_RHS || op == BGL_OP_DOT)
        return fail(BGL_E_INVALID, "bgl_gspmm: op %d is not a gspmm operator", op);
    if (reduce < BGL_RED_SUM || reduce > BGL_RED_MEAN)
        return fail(BGL_E_INVALID, "bgl_gspmm: reduce %d not recognized", reduce);
    if (num_rows < 0 || num_edges < 0 || dout < 0)
        return fail(BGL_E_INVALID, "bgl_gspmm: negative size");
    if (num_rows >= (int64_t(1) << 31) || num_edges >= (int64_t(1) << 31))
        return fail(BGL_E_UNSUPPORTED, "bgl_gspmm: more than 2^31-1 rows or edges");
    const bool need_l = op != BGL_OP_COPY_RHS, need_r = op != BGL_OP_COPY_LHS;
    // the kernels address a row's columns in 32 bits: row strides below 4 GiB,
    // column indices and broadcast divisors below 2^31
    const int64_t elem = dtype == BGL_F32 ? 4 : 8, lim = int64_t(1) << 31;
    if (dout >= lim || (need_l && (lhs_width * elem >= 2 * lim || lhs_div >= lim)) ||
        (need_r && (rhs_width * elem >= 2 * lim || rhs_div >= lim)))
        return fail(BGL_E_UNSUPPORTED, "bgl_gspmm: a feature row of 4 GiB or more");
    if (need_l && (lhs_width < 1 || lhs_div < 1))
        return fail(BGL_E_INVALID, "bgl_gspmm: lhs width/div must be >= 1");
    if (need_r && (rhs_width < 1 || rhs_div < 1))
        return fail(BGL_E_INVALID, "bgl_gspmm: rhs width/div must be >= 1");
    if (num_rows == 0 || dout == 0) return BGL_OK;
    if (!indptr || !out) return fail(BGL_E_INVALID, "bgl_gspmm: null indptr/out");
    if (num_edges > 0) {
        if (need_l && (!lhs || !indices)) return fail(BGL_E_INVALID, "bgl_gspmm: null lhs/indices");
        if (need_r && !rhs) return fail(BGL_E_INVALID, "bgl_gspmm: null rhs");
    }
    if (arg_u && !indices) return fail(BGL_E_INVALID, "bgl_gspmm: arg_u needs indices");
    size_t need = spmm_ws_bytes(num_rows, num_edges, dout, dtype, reduce);
    if (workspace_bytes < need || (need && !workspace))
        return fail(BGL_E_WORKSPACE, "bgl_gspmm: workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t s = as_stream(stream);
    if (dtype == BGL_F32)
        return run_spmm<float>(indptr, indices, eid, deg, num_rows, num_edges, lhs, lhs_width,
                               lhs_div, rhs, rhs_width, rhs_div, out, dout, arg_u, arg_e, dtype,
                               op, reduce, flags, workspace, s);
    return run_spmm<double>(indptr, indices, eid, deg, num_rows, num_edges, lhs, lhs_width,
                            lhs_div, rhs, rhs_width, rhs_div, out, dout, arg_u, arg_e, dtype, op,
                            reduce, flags, workspace, s);
}

}  // extern "C"
