// gSDDMM (replaces mdgl_gsddmm, src/capi.mojo:70-91 -> src/ported.mojo:204-329).
//
// Edge-parallel: a team of lanes per edge, each lane owning V consecutive
// output columns; the two operand rows are gathered through the target code
// (u[e], v[e] or e itself, src/ported.mojo:256-271).  `dot` accumulates the
// lane's products and folds the team's partials with xor shuffles, so unlike
// the element-wise ops its rounding differs from the reference's lane-partial
// order (src/ported.mojo:273-293) -- it is compared with a tolerance.
#include "common.cuh"

namespace bgl {
namespace {

template <typename T>
struct SddmmArgs {
    const int32_t *u;
    const int32_t *v;
    int64_t num_edges;
    Operand<T> lhs, rhs;
    int lt, rt;
    T *out;
    int64_t dout;
    int64_t red_len;
    int ts;
};

__device__ __forceinline__ int64_t target_row(int tgt, const int32_t *u, const int32_t *v,
                                              int64_t e) {
    if (tgt == BGL_SRC) return __ldg(u + e);
    if (tgt == BGL_DST) return __ldg(v + e);
    return e;
}

template <typename T, int OP, int V>
__global__ void __launch_bounds__(256) k_sddmm(const SddmmArgs<T> a) {
    const int ts = a.ts;
    const int lane = threadIdx.x & 31;
    const int t = lane & (ts - 1);
    const unsigned mask = ts == 32 ? 0xffffffffu : (((1u << ts) - 1u) << (lane & ~(ts - 1)));
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    const int64_t teams = ((int64_t)gridDim.x * blockDim.x) / ts;
    constexpr bool NEED_L = OP != BGL_OP_COPY_RHS;
    constexpr bool NEED_R = OP != BGL_OP_COPY_LHS;
    ColMap<V> lmap, rmap;
    if (OP != BGL_OP_DOT) {
        if (NEED_L) lmap = col_map<T, V>(a.lhs, (int64_t)t * V);
        if (NEED_R) rmap = col_map<T, V>(a.rhs, (int64_t)t * V);
    }
    for (int64_t e = team; e < a.num_edges; e += teams) {
        const int64_t li = NEED_L ? target_row(a.lt, a.u, a.v, e) : 0;
        const int64_t ri = NEED_R ? target_row(a.rt, a.u, a.v, e) : 0;
        if (OP == BGL_OP_DOT) {
            T acc = T(0);
            const int64_t cvn = a.red_len / V;
            for (int64_t cv = t; cv < cvn; cv += ts) {
                T l[V], r[V];
                load_vec<T, V>(a.lhs.ptr + li * a.red_len + cv * V, l);
                load_vec<T, V>(a.rhs.ptr + ri * a.red_len + cv * V, r);
#pragma unroll
                for (int i = 0; i < V; ++i) acc = Arith<T>::add(acc, Arith<T>::mul(l[i], r[i]));
            }
            for (int off = ts >> 1; off > 0; off >>= 1)
                acc = Arith<T>::add(acc, __shfl_xor_sync(mask, acc, off, ts));
            if (t == 0) a.out[e] = acc;
        } else {
            const int64_t cvn = a.dout / V;
            for (int64_t cv = t; cv < cvn; cv += ts) {
                T l[V], r[V], o[V];
                if (cv == t) {  // the lane's first columns: the common, one-vector case
                    if (NEED_L) load_mapped<T, V>(a.lhs, li, (int64_t)t * V, lmap, l);
                    if (NEED_R) load_mapped<T, V>(a.rhs, ri, (int64_t)t * V, rmap, r);
                } else {
                    if (NEED_L) load_cols<T, V>(a.lhs, li, cv * V, l);
                    if (NEED_R) load_cols<T, V>(a.rhs, ri, cv * V, r);
                }
#pragma unroll
                for (int i = 0; i < V; ++i)
                    o[i] = message<OP, T>(NEED_L ? l[i] : T(0), NEED_R ? r[i] : T(0));
                store_vec<T, V>(a.out + e * a.dout + cv * V, o);
            }
        }
    }
}

template <typename T, int V>
int launch_sddmm(const SddmmArgs<T> &a, int op, cudaStream_t s) {
    int64_t teams = a.num_edges;
    int64_t cap = int64_t(num_sms()) * 2048 / a.ts;  // one full wave of resident teams
    if (teams > cap) teams = cap;
    int grid = (int)((teams * a.ts + 255) / 256);
    if (grid < 1) grid = 1;
    switch (op) {
    case BGL_OP_ADD: k_sddmm<T, BGL_OP_ADD, V><<<grid, 256, 0, s>>>(a); break;
    case BGL_OP_SUB: k_sddmm<T, BGL_OP_SUB, V><<<grid, 256, 0, s>>>(a); break;
    case BGL_OP_MUL: k_sddmm<T, BGL_OP_MUL, V><<<grid, 256, 0, s>>>(a); break;
    case BGL_OP_DIV: k_sddmm<T, BGL_OP_DIV, V><<<grid, 256, 0, s>>>(a); break;
    case BGL_OP_DOT: k_sddmm<T, BGL_OP_DOT, V><<<grid, 256, 0, s>>>(a); break;
    case BGL_OP_COPY_LHS: k_sddmm<T, BGL_OP_COPY_LHS, V><<<grid, 256, 0, s>>>(a); break;
    case BGL_OP_COPY_RHS: k_sddmm<T, BGL_OP_COPY_RHS, V><<<grid, 256, 0, s>>>(a); break;
    default: return fail(BGL_E_INVALID, "bgl_gsddmm: op %d", op);
    }
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

template <typename T>
int run_sddmm(const int32_t *u, const int32_t *v, int64_t ne, const void *lhs, int64_t lw,
              int64_t ldiv, int lt, const void *rhs, int64_t rw, int64_t rdiv, int rt, void *out,
              int64_t dout, int64_t red_len, int op, cudaStream_t s) {
    constexpr int VM = sizeof(T) == 4 ? 4 : 2;
    const bool need_l = op != BGL_OP_COPY_RHS, need_r = op != BGL_OP_COPY_LHS;
    const bool dot = op == BGL_OP_DOT;
    const int64_t width = dot ? red_len : dout;
    const bool lfull = dot || (ldiv == 1 && lw == dout);
    const bool rfull = dot || (rdiv == 1 && rw == dout);
    int V = (width % VM == 0) ? VM : 1;
    const size_t vb = size_t(V) * sizeof(T);
    if (V > 1 && ((!dot && !aligned(out, vb)) || (need_l && lfull && !aligned(lhs, vb)) ||
                  (need_r && rfull && !aligned(rhs, vb))))
        V = 1;
    SddmmArgs<T> a;
    a.u = u;
    a.v = v;
    a.num_edges = ne;
    a.lhs = Operand<T>{static_cast<const T *>(lhs), lw, ldiv, lfull, (ldiv % V == 0) || lw == 1};
    a.rhs = Operand<T>{static_cast<const T *>(rhs), rw, rdiv, rfull, (rdiv % V == 0) || rw == 1};
    a.lt = lt;
    a.rt = rt;
    a.out = static_cast<T *>(out);
    a.dout = dout;
    a.red_len = red_len;
    a.ts = next_pow2(width / V < 1 ? 1 : width / V);
    if (V == 1) return launch_sddmm<T, 1>(a, op, s);
    return launch_sddmm<T, VM>(a, op, s);
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" int bgl_gsddmm(const int32_t *u, const int32_t *v, int64_t num_edges, const void *lhs,
                          int64_t lhs_width, int64_t lhs_div, int lhs_target, const void *rhs,
                          int64_t rhs_width, int64_t rhs_div, int rhs_target, void *out,
                          int64_t dout, int64_t red_len, int dtype, int op, void *stream) {
    if (dtype != BGL_F32 && dtype != BGL_F64)
        return fail(BGL_E_UNSUPPORTED, "bgl_gsddmm: dtype %d (f32 and f64 only)", dtype);
    if (op < BGL_OP_ADD || op > BGL_OP_COPY_RHS)
        return fail(BGL_E_INVALID, "bgl_gsddmm: op %d not recognized", op);
    if (lhs_target < BGL_SRC || lhs_target > BGL_EDGE || rhs_target < BGL_SRC ||
        rhs_target > BGL_EDGE)
        return fail(BGL_E_INVALID, "bgl_gsddmm: target codes must be 0 (u), 1 (v) or 2 (e)");
    if (num_edges < 0 || dout < 0) return fail(BGL_E_INVALID, "bgl_gsddmm: negative size");
    if (op == BGL_OP_DOT && (dout != 1 || red_len < 0))
        return fail(BGL_E_INVALID, "bgl_gsddmm: dot writes one column (dout = 1) over red_len >= 0");
    const bool need_l = op != BGL_OP_COPY_RHS, need_r = op != BGL_OP_COPY_LHS;
    if (op != BGL_OP_DOT && ((need_l && (lhs_width < 1 || lhs_div < 1)) ||
                             (need_r && (rhs_width < 1 || rhs_div < 1))))
        return fail(BGL_E_INVALID, "bgl_gsddmm: operand width/div must be >= 1");
    if (num_edges == 0 || dout == 0) return BGL_OK;
    if (!out || (need_l && !lhs) || (need_r && !rhs))
        return fail(BGL_E_INVALID, "bgl_gsddmm: null buffer");
    const bool need_u = (need_l && lhs_target == BGL_SRC) || (need_r && rhs_target == BGL_SRC);
    const bool need_v = (need_l && lhs_target == BGL_DST) || (need_r && rhs_target == BGL_DST);
    if ((need_u && !u) || (need_v && !v)) return fail(BGL_E_INVALID, "bgl_gsddmm: null u/v");
    cudaStream_t s = as_stream(stream);
    if (op == BGL_OP_DOT && red_len == 0) {
        BGL_CUDA(cudaMemsetAsync(out, 0, size_t(num_edges) * (dtype == BGL_F32 ? 4 : 8), s));
        return BGL_OK;
    }
    if (dtype == BGL_F32)
        return run_sddmm<float>(u, v, num_edges, lhs, lhs_width, lhs_div, lhs_target, rhs,
                                rhs_width, rhs_div, rhs_target, out, dout, red_len, op, s);
    return run_sddmm<double>(u, v, num_edges, lhs, lhs_width, lhs_div, lhs_target, rhs, rhs_width,
                             rhs_div, rhs_target, out, dout, red_len, op, s);
}
