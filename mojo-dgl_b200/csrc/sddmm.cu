// gSDDMM (replaces mdgl_gsddmm, src/capi.mojo:70-91 -> src/ported.mojo:204-329).
//
// Edge-parallel: a team of lanes per edge, each lane owning V consecutive
// output columns; the two operand rows are gathered through the target code
// (u[e], v[e] or e itself, src/ported.mojo:256-271).  A team takes UN edges
// per iteration -- their ids first, then all their row loads, then the
// arithmetic and the stores -- so each lane keeps UN row pairs in flight.
// `dot` accumulates the lane's products and folds the team's partials with
// xor shuffles, so unlike the element-wise ops its rounding differs from the
// reference's lane-partial order (src/ported.mojo:273-293) -- it is compared
// with a tolerance.
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
    bool ids_once;  // endpoint ids loaded evict-first (teams of <= 8 lanes)
};

// With narrow rows a warp covers many edges (teams of <= 8 lanes), so an
// endpoint-id line is read by one or two warps and never again: those ids
// are loaded evict-first (ld.global.cs) and L2 keeps the node rows the edges
// gather (config 2's u_add_v, 32 MB tables: 0.51 -> 0.39 ms).  With wide rows
// (a warp per edge) 32 consecutive warps share each id line, and evict-first
// lines did not survive the row traffic between them (config 5's u_dot_v
// 15.7 -> 16.8 ms), so those ids keep the default policy.
__device__ __forceinline__ int64_t target_row(int tgt, const int32_t *u, const int32_t *v,
                                              int64_t e, bool ids_once) {
    if (tgt == BGL_SRC) return ids_once ? __ldcs(u + e) : __ldg(u + e);
    if (tgt == BGL_DST) return ids_once ? __ldcs(v + e) : __ldg(v + e);
    return e;
}

// Random whole-row gathers want resident warps more than per-warp depth.
// Measured on config 5 (u_dot_v, 50M edges, two 5 GB (N, 256) float32
// matrices): one edge per team at 8 blocks of 256 per SM (32 registers)
// 15.7 ms; 2 edges at 4 blocks 20.9 ms; 4 at 3 blocks 23.9 ms; 4 at 2 blocks
// 37.1 ms.  Config 2's u_add_v (8 columns): 0.567 / 0.576 / 0.604 / 0.726 ms.
#ifndef BGL_SDDMM_UN
#define BGL_SDDMM_UN 1  // edges a team has in flight
#endif
#ifndef BGL_SDDMM_MINB
#define BGL_SDDMM_MINB 8  // resident 256-thread blocks per SM the registers must allow
#endif
constexpr int kSddmmUN = BGL_SDDMM_UN;

template <typename T, int OP, int V>
__global__ void __launch_bounds__(256, BGL_SDDMM_MINB) k_sddmm(const SddmmArgs<T> a) {
    constexpr int UN = kSddmmUN;
    const int ts = a.ts;
    const int lane = threadIdx.x & 31;
    const int t = lane & (ts - 1);
    const unsigned mask = ts == 32 ? 0xffffffffu : (((1u << ts) - 1u) << (lane & ~(ts - 1)));
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    const int64_t teams = ((int64_t)gridDim.x * blockDim.x) / ts;
    constexpr bool NEED_L = OP != BGL_OP_COPY_RHS;
    constexpr bool NEED_R = OP != BGL_OP_COPY_LHS;
    if (OP == BGL_OP_DOT) {
        const int32_t cvn = (int32_t)(a.red_len / V);
        for (int64_t e0 = team; e0 < a.num_edges; e0 += teams * UN) {
            int64_t li[UN], ri[UN];
            bool ok[UN];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                const int64_t e = e0 + u * teams;
                ok[u] = e < a.num_edges;
                li[u] = ok[u] ? target_row(a.lt, a.u, a.v, e, a.ids_once) : 0;
                ri[u] = ok[u] ? target_row(a.rt, a.u, a.v, e, a.ids_once) : 0;
            }
            T acc[UN];
#pragma unroll
            for (int u = 0; u < UN; ++u) acc[u] = T(0);
            for (int32_t cv = t; cv < cvn; cv += ts) {
                T l[UN][V], r[UN][V];
#pragma unroll
                for (int u = 0; u < UN; ++u) {
                    if (ok[u]) {
                        ld_stream(a.lhs.ptr + li[u] * a.red_len + (int64_t)cv * V, l[u]);
                        ld_stream(a.rhs.ptr + ri[u] * a.red_len + (int64_t)cv * V, r[u]);
                    }
                }
#pragma unroll
                for (int u = 0; u < UN; ++u) {
                    if (ok[u]) {
#pragma unroll
                        for (int i = 0; i < V; ++i)
                            acc[u] = Arith<T>::add(acc[u], Arith<T>::mul(l[u][i], r[u][i]));
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                for (int off = ts >> 1; off > 0; off >>= 1)
                    acc[u] = Arith<T>::add(acc[u], __shfl_xor_sync(mask, acc[u], off, ts));
                if (ok[u] && t == 0) a.out[e0 + u * teams] = acc[u];
            }
        }
        return;
    }
    const int32_t cvn = (int32_t)(a.dout / V);
    for (int32_t cb = 0; cb < cvn; cb += ts) {
        const int32_t cv = cb + t;
        if (cv >= cvn) break;  // no shuffles below: lanes may leave
        const int64_t k0 = (int64_t)cv * V;
        LaneCols<T, V> lc, rc;
        if (NEED_L) lc = lane_cols<T, V>(a.lhs, k0);
        if (NEED_R) rc = lane_cols<T, V>(a.rhs, k0);
        for (int64_t e0 = team; e0 < a.num_edges; e0 += teams * UN) {
            int64_t li[UN], ri[UN];
            bool ok[UN];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                const int64_t e = e0 + u * teams;
                ok[u] = e < a.num_edges;
                if (ok[u]) {
                    if (NEED_L) li[u] = target_row(a.lt, a.u, a.v, e, a.ids_once);
                    if (NEED_R) ri[u] = target_row(a.rt, a.u, a.v, e, a.ids_once);
                }
            }
            T l[UN][V], r[UN][V];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (ok[u]) {
                    if (NEED_L) load_row<T, V>(lc, a.lhs, li[u], l[u]);
                    if (NEED_R) load_row<T, V>(rc, a.rhs, ri[u], r[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < UN; ++u) {
                if (ok[u]) {
                    T o[V];
#pragma unroll
                    for (int i = 0; i < V; ++i)
                        o[i] = message<OP, T>(NEED_L ? l[u][i] : T(0), NEED_R ? r[u][i] : T(0));
                    store_stream<T, V>(a.out + (e0 + u * teams) * a.dout + k0, o);
                }
            }
        }
    }
}

template <typename T, int V>
int launch_sddmm(const SddmmArgs<T> &a, int op, cudaStream_t s) {
    // two waves of resident teams (3 blocks of 256 per SM); each keeps UN
    // edges in flight
    int64_t teams = (a.num_edges + kSddmmUN - 1) / kSddmmUN;
    const int64_t cap = int64_t(num_sms()) * 256 * BGL_SDDMM_MINB * 2 / a.ts;
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
    a.ids_once = a.ts <= 8;
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
    // 32-bit row strides: feature rows below 4 GiB, broadcast arithmetic below 2^31
    const int64_t elem = dtype == BGL_F32 ? 4 : 8, lim = int64_t(1) << 31;
    if (dout >= lim || red_len >= lim || (need_l && (lhs_width * elem >= 2 * lim || lhs_div >= lim)) ||
        (need_r && (rhs_width * elem >= 2 * lim || rhs_div >= lim)))
        return fail(BGL_E_UNSUPPORTED, "bgl_gsddmm: a feature row of 4 GiB or more");
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
