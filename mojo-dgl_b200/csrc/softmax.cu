// Fused per-row softmax over a CSR (replaces mdgl_edge_softmax_,
// src/ported.mojo:876-1080, and mdgl_segment_softmax, src/ported.mojo:660-768).
//
// Both reference kernels are the same computation: for each row of a CSR and
// each column h, over the row's selected items e,
//     out[e, h] = exp(z[e, h] - max_e z[., h]) / sum_e exp(z[., h] - max).
// edge_softmax reaches the items through the CSR's edge ids; segment_softmax's
// items are the consecutive value rows of a segment (eid = identity).
//
// Two layouts:
//   * narrow rows (d <= 8, attention heads): a warp per row, lanes striding
//     over the row's edges, each lane holding every column of its edge; the
//     max and the exp-sum are folded across the warp with shuffles.
//   * wide rows (segment softmax over feature columns): a team of lanes per
//     row, each lane owning V consecutive columns and walking the rows in
//     order -- the reference's own per-column sequential order.
#include "common.cuh"

namespace bgl {
namespace {

template <typename T>
struct SoftArgs {
    const int64_t *indptr;
    const int32_t *eid;
    const int8_t *mask;
    int64_t num_rows;
    int64_t num_items;
    const T *logits;
    T *out;
    int64_t d;
    int ts;
};

__device__ __forceinline__ void row_bounds(const int64_t *indptr, int64_t r, int64_t n,
                                           int64_t &s, int64_t &e) {
    s = indptr[r];
    e = indptr[r + 1];
    if (s < 0) s = 0;  // src/ported.mojo:694-699
    if (e > n) e = n;
    if (e < s) e = s;
}

template <typename T, int DM>
__global__ void __launch_bounds__(256) k_softmax_narrow(const SoftArgs<T> a) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t d = a.d;
    for (int64_t row = warp; row < a.num_rows; row += warps) {
        int64_t s, t;
        row_bounds(a.indptr, row, a.num_items, s, t);
        if (s >= t) continue;
        for (int64_t h0 = 0; h0 < d; h0 += DM) {
            const int hn = (d - h0) < DM ? (int)(d - h0) : DM;
            T m[DM];
#pragma unroll
            for (int h = 0; h < DM; ++h) m[h] = Arith<T>::ninf();
            bool any = false;
            for (int64_t i = s + lane; i < t; i += 32) {
                const int64_t e = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                if (a.mask && a.mask[e] != 1) continue;
                any = true;
                const T *z = a.logits + e * d + h0;
#pragma unroll
                for (int h = 0; h < DM; ++h)
                    if (h < hn) {
                        T x = __ldg(z + h);
                        m[h] = x > m[h] ? x : m[h];
                    }
            }
            if (!__any_sync(0xffffffffu, any)) continue;
#pragma unroll
            for (int h = 0; h < DM; ++h)
                for (int off = 16; off > 0; off >>= 1) {
                    T o = __shfl_xor_sync(0xffffffffu, m[h], off);
                    m[h] = o > m[h] ? o : m[h];
                }
            T sm[DM];
#pragma unroll
            for (int h = 0; h < DM; ++h) sm[h] = T(0);
            for (int64_t i = s + lane; i < t; i += 32) {
                const int64_t e = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                if (a.mask && a.mask[e] != 1) continue;
                const T *z = a.logits + e * d + h0;
#pragma unroll
                for (int h = 0; h < DM; ++h)
                    if (h < hn) sm[h] = Arith<T>::add(sm[h], Arith<T>::ex(Arith<T>::sub(__ldg(z + h), m[h])));
            }
#pragma unroll
            for (int h = 0; h < DM; ++h)
                for (int off = 16; off > 0; off >>= 1)
                    sm[h] = Arith<T>::add(sm[h], __shfl_xor_sync(0xffffffffu, sm[h], off));
            for (int64_t i = s + lane; i < t; i += 32) {
                const int64_t e = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                if (a.mask && a.mask[e] != 1) continue;
                const T *z = a.logits + e * d + h0;
                T *o = a.out + e * d + h0;
#pragma unroll
                for (int h = 0; h < DM; ++h)
                    if (h < hn)
                        o[h] = Arith<T>::div(Arith<T>::ex(Arith<T>::sub(__ldg(z + h), m[h])), sm[h]);
            }
        }
    }
}

template <typename T, int V>
__global__ void __launch_bounds__(256) k_softmax_wide(const SoftArgs<T> a) {
    const int ts = a.ts;
    const int t = threadIdx.x & (ts - 1);
    const int64_t team = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / ts;
    const int64_t teams = ((int64_t)gridDim.x * blockDim.x) / ts;
    const int64_t d = a.d;
    const int64_t cvn = d / V;
    for (int64_t row = team; row < a.num_rows; row += teams) {
        int64_t s, t_end;
        row_bounds(a.indptr, row, a.num_items, s, t_end);
        if (s >= t_end) continue;
        for (int64_t cv = t; cv < cvn; cv += ts) {
            T m[V];
#pragma unroll
            for (int i = 0; i < V; ++i) m[i] = Arith<T>::ninf();
            bool any = false;
            for (int64_t i = s; i < t_end; ++i) {
                const int64_t e = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                if (a.mask && a.mask[e] != 1) continue;
                any = true;
                T z[V];
                load_vec<T, V>(a.logits + e * d + cv * V, z);
#pragma unroll
                for (int k = 0; k < V; ++k) m[k] = z[k] > m[k] ? z[k] : m[k];
            }
            if (!any) continue;
            T sm[V];
#pragma unroll
            for (int k = 0; k < V; ++k) sm[k] = T(0);
            for (int64_t i = s; i < t_end; ++i) {
                const int64_t e = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                if (a.mask && a.mask[e] != 1) continue;
                T z[V];
                load_vec<T, V>(a.logits + e * d + cv * V, z);
#pragma unroll
                for (int k = 0; k < V; ++k)
                    sm[k] = Arith<T>::add(sm[k], Arith<T>::ex(Arith<T>::sub(z[k], m[k])));
            }
            for (int64_t i = s; i < t_end; ++i) {
                const int64_t e = a.eid ? (int64_t)__ldg(a.eid + i) : i;
                if (a.mask && a.mask[e] != 1) continue;
                T z[V], o[V];
                load_vec<T, V>(a.logits + e * d + cv * V, z);
#pragma unroll
                for (int k = 0; k < V; ++k)
                    o[k] = Arith<T>::div(Arith<T>::ex(Arith<T>::sub(z[k], m[k])), sm[k]);
                store_vec<T, V>(a.out + e * d + cv * V, o);
            }
        }
    }
}

template <typename T>
int run_softmax(SoftArgs<T> a, cudaStream_t s) {
    const int64_t cap = int64_t(num_sms()) * 8;  // blocks of 256 in one resident wave
    if (a.d <= 8) {
        int64_t grid = (a.num_rows * 32 + 255) / 256;
        if (grid > cap) grid = cap;
        if (grid < 1) grid = 1;
        k_softmax_narrow<T, 8><<<(int)grid, 256, 0, s>>>(a);
        BGL_LAUNCH_CHECK();
        return BGL_OK;
    }
    constexpr int VM = sizeof(T) == 4 ? 4 : 2;
    int V = (a.d % VM == 0 && aligned(a.logits, VM * sizeof(T)) && aligned(a.out, VM * sizeof(T)))
                ? VM
                : 1;
    a.ts = next_pow2(a.d / V);
    int64_t grid = (a.num_rows * a.ts + 255) / 256;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    if (V == 1)
        k_softmax_wide<T, 1><<<(int)grid, 256, 0, s>>>(a);
    else
        k_softmax_wide<T, VM><<<(int)grid, 256, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

}  // namespace
}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_softmax_workspace_size(int64_t num_rows, int64_t num_items, int64_t d, int dtype) {
    (void)num_rows;
    (void)num_items;
    (void)d;
    (void)dtype;
    return 0;
}

int bgl_edge_softmax(const int64_t *indptr, const int32_t *eid, const int8_t *mask,
                     int64_t num_rows, int64_t num_items, const void *logits, void *out,
                     int64_t d, int dtype, void *workspace, size_t workspace_bytes,
                     void *stream) {
    (void)workspace;
    (void)workspace_bytes;
    if (dtype != BGL_F32 && dtype != BGL_F64)
        return fail(BGL_E_UNSUPPORTED, "bgl_edge_softmax: dtype %d (f32 and f64 only)", dtype);
    if (num_rows < 0 || num_items < 0 || d < 0)
        return fail(BGL_E_INVALID, "bgl_edge_softmax: negative size");
    if (num_rows == 0 || num_items == 0 || d == 0) return BGL_OK;
    if (!indptr || !logits || !out) return fail(BGL_E_INVALID, "bgl_edge_softmax: null buffer");
    cudaStream_t s = as_stream(stream);
    if (dtype == BGL_F32) {
        SoftArgs<float> a{indptr, eid, mask, num_rows, num_items, (const float *)logits,
                          (float *)out, d, 32};
        return run_softmax<float>(a, s);
    }
    SoftArgs<double> a{indptr, eid, mask, num_rows, num_items, (const double *)logits,
                       (double *)out, d, 32};
    return run_softmax<double>(a, s);
}

}  // extern "C"
