// Grouped GEMM: segment_mm and gather_mm (replace mdgl_segment_mm,
// src/ported.mojo:773-804, and mdgl_gather_mm, src/ported.mojo:1089-1130,
// plus gather_mm's sort -> segment_mm -> unsort route,
// python/mojodgl/ops/gather_mm.py:79-87).
//
// Rows are grouped into segments (segment_mm: consecutive rows by seglen;
// gather_mm: a stable device sort of the row ids by idx_b), each segment is cut
// into 128-row tiles, and a tile never crosses a segment, so every tile
// multiplies by a single b[r].  The tensor-core kernel (grouped_mm_tc.cu) runs
// fp32 inputs in TF32 and bf16 inputs in BF16 on tcgen05; this file holds the
// schedule, the sort, and the SIMT kernel that serves fp64 (where it
// reproduces the reference's k-ordered accumulation bit for bit) and any
// shape the tensor-core kernel does not take.
#include <cub/device/device_radix_sort.cuh>

#include "grouped_mm.cuh"

namespace bgl {

// Segment row offsets and tile offsets, clamped so no segment runs past n.
// A single thread walks the (short) relation list.
__global__ void k_gmm_schedule(const int64_t *__restrict__ seglen, int64_t r, int64_t n,
                               int64_t bm, int64_t *__restrict__ seg_off,
                               int64_t *__restrict__ tile_off) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    int64_t row = 0, tiles = 0;
    seg_off[0] = 0;
    tile_off[0] = 0;
    for (int64_t i = 0; i < r; ++i) {
        int64_t len = seglen[i];
        if (len < 0) len = 0;
        if (len > n - row) len = n - row;
        row += len;
        tiles += (len + bm - 1) / bm;
        seg_off[i + 1] = row;
        tile_off[i + 1] = tiles;
    }
}

// Rows past the last segment are zero (python/mojodgl/ops/segment.py:210).
template <typename T>
__global__ void k_zero_tail(T *__restrict__ out, const int64_t *__restrict__ seg_off, int64_t r,
                            int64_t n, int64_t d2) {
    const int64_t first = seg_off[r] * d2;
    for (int64_t i = first + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * d2;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = T(0);
}

// Sort keys, the identity permutation and the rows per relation.  With few
// relations (r <= kKeysSmem) each block counts in shared memory and adds its
// counts once, instead of every row hitting one of r global counters.
constexpr int kKeysSmem = 8192;

__global__ void k_gmm_keys(const int64_t *__restrict__ idx, int32_t *__restrict__ key,
                           int32_t *__restrict__ iota, int64_t *__restrict__ counts, int64_t n,
                           int64_t r) {
    extern __shared__ unsigned int hist[];
    const bool local = r <= kKeysSmem;
    if (local) {
        for (int64_t j = threadIdx.x; j < r; j += blockDim.x) hist[j] = 0;
        __syncthreads();
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int32_t k = (int32_t)idx[i];
        key[i] = k;
        iota[i] = (int32_t)i;
        if (local)
            atomicAdd(&hist[k], 1u);
        else
            atomicAdd(reinterpret_cast<unsigned long long *>(counts + k), 1ull);
    }
    if (local) {
        __syncthreads();
        for (int64_t j = threadIdx.x; j < r; j += blockDim.x)
            if (hist[j]) atomicAdd(reinterpret_cast<unsigned long long *>(counts + j), (unsigned long long)hist[j]);
    }
}

// SIMT tile: 64 x 64 outputs per 256 threads, 4 x 4 per thread; every output
// accumulates its k terms in order with separately rounded multiply and add.
template <typename T>
__global__ void __launch_bounds__(256) k_gmm_simt(const T *__restrict__ a, const T *__restrict__ b,
                                                  T *__restrict__ out,
                                                  const int64_t *__restrict__ seg_off,
                                                  const int64_t *__restrict__ tile_off,
                                                  int64_t r, int64_t d1, int64_t d2,
                                                  const int32_t *__restrict__ perm) {
    constexpr int BM = 64, BN = 64, BK = 16;
    __shared__ T As[BK][BM + 1];
    __shared__ T Bs[BK][BN + 1];
    const int64_t tile = blockIdx.x;
    if (tile >= tile_off[r]) return;
    int64_t lo = 0, hi = r;  // last relation whose first tile is <= tile
    while (lo < hi) {
        int64_t mid = (lo + hi + 1) >> 1;
        if (tile_off[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    const int64_t rel = lo;
    const int64_t row0 = seg_off[rel] + (tile - tile_off[rel]) * BM;
    const int64_t row_end = seg_off[rel + 1];
    const int64_t col0 = (int64_t)blockIdx.y * BN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const T *bb = b + rel * d1 * d2;
    T acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = T(0);
    for (int64_t k0 = 0; k0 < d1; k0 += BK) {
        for (int idx = threadIdx.x; idx < BM * BK; idx += 256) {
            int rr = idx / BK, kk = idx % BK;
            int64_t row = row0 + rr;
            T v = T(0);
            if (row < row_end && k0 + kk < d1) {
                int64_t src = perm ? (int64_t)perm[row] : row;
                v = a[src * d1 + k0 + kk];
            }
            As[kk][rr] = v;
        }
        for (int idx = threadIdx.x; idx < BK * BN; idx += 256) {
            int kk = idx / BN, cc = idx % BN;
            T v = T(0);
            if (k0 + kk < d1 && col0 + cc < d2) v = bb[(k0 + kk) * d2 + col0 + cc];
            Bs[kk][cc] = v;
        }
        __syncthreads();
        const int kn = (d1 - k0) < BK ? (int)(d1 - k0) : BK;
        for (int kk = 0; kk < kn; ++kk) {
            T av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    acc[i][j] = Arith<T>::add(acc[i][j], Arith<T>::mul(av[i], bv[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t row = row0 + ty * 4 + i;
        if (row >= row_end) continue;
        int64_t dst = perm ? (int64_t)perm[row] : row;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t col = col0 + tx * 4 + j;
            if (col < d2) out[dst * d2 + col] = acc[i][j];
        }
    }
}

namespace {

int elem_size(int dtype) { return dtype == BGL_F64 ? 8 : dtype == BGL_F32 ? 4 : 2; }

size_t sort_bytes(int64_t n, int64_t r) {
    size_t bytes = 0;
    int bits = 1;
    while (bits < 31 && (int64_t(1) << bits) < r) ++bits;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const int32_t *)nullptr, (int32_t *)nullptr,
                                    (const int32_t *)nullptr, (int32_t *)nullptr, (int)n, 0, bits);
    return bytes;
}

}  // namespace

GmmLayout gmm_layout(void *ws, int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype,
                     bool gather) {
    Carver c(ws);
    GmmLayout l;
    l.seg_off = c.take<int64_t>(r + 1);
    l.tile_off = c.take<int64_t>(r + 1);
    l.counts = gather ? c.take<int64_t>(r) : nullptr;
    l.keys = gather ? c.take<int32_t>(n) : nullptr;
    l.keys_sorted = gather ? c.take<int32_t>(n) : nullptr;
    l.iota = gather ? c.take<int32_t>(n) : nullptr;
    l.perm = gather ? c.take<int32_t>(n) : nullptr;
    const bool tc = gmm_tensor_core_supported(d1, d2, dtype);
    const size_t elem = dtype == BGL_BF16 ? 2 : 4;
    l.tc_b = tc ? c.take<char>(size_t(r) * d1 * d2 * elem) : nullptr;
    l.sort_temp_bytes = gather ? sort_bytes(n, r) : 0;
    l.sort_temp = gather ? c.take<char>(l.sort_temp_bytes) : nullptr;
    l.bytes = c.used + 256;
    return l;
}

// Runs the grouped product once the schedule (and for gather_mm the
// permutation) is on the device.  `tc` says the tensor-core kernel takes this
// shape (and the schedule was cut in its 128-row tiles).
static int run_gmm(const void *a, const void *b, void *out, const GmmLayout &l, int64_t n,
                   int64_t d1, int64_t r, int64_t d2, int dtype, bool tc, cudaStream_t s) {
    if (tc) return gmm_tensor_core(a, b, out, l, n, d1, r, d2, dtype, s);
    if (dtype == BGL_BF16)
        return fail(BGL_E_UNSUPPORTED, "grouped mm: bf16 needs d1 %% 16 == 0 and d2 %% 16 == 0");
    int64_t max_tiles = (n + 63) / 64 + r;
    dim3 grid((unsigned)(max_tiles > 0 ? max_tiles : 1), (unsigned)((d2 + 63) / 64));
    if (dtype == BGL_F64)
        k_gmm_simt<double><<<grid, 256, 0, s>>>((const double *)a, (const double *)b, (double *)out,
                                                 l.seg_off, l.tile_off, r, d1, d2, l.perm);
    else
        k_gmm_simt<float><<<grid, 256, 0, s>>>((const float *)a, (const float *)b, (float *)out,
                                                l.seg_off, l.tile_off, r, d1, d2, l.perm);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

static int check_gmm(const char *who, const void *a, const void *b, void *out, int64_t n,
                     int64_t d1, int64_t r, int64_t d2, int dtype) {
    if (dtype != BGL_F32 && dtype != BGL_F64 && dtype != BGL_BF16)
        return fail(BGL_E_UNSUPPORTED, "%s: dtype %d", who, dtype);
    if (n < 0 || d1 < 0 || r < 0 || d2 < 0) return fail(BGL_E_INVALID, "%s: negative size", who);
    if (n >= (int64_t(1) << 31)) return fail(BGL_E_UNSUPPORTED, "%s: n >= 2^31", who);
    if (n && d2 && (!out || (d1 && (!a || (r && !b)))))
        return fail(BGL_E_INVALID, "%s: null buffer", who);
    return BGL_OK;
}

}  // namespace bgl

using namespace bgl;

extern "C" {

size_t bgl_segment_mm_workspace_size(int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype) {
    if (n < 0 || r < 0 || d1 < 0 || d2 < 0) return 0;
    return gmm_layout(nullptr, n, d1, r, d2, dtype, false).bytes;
}

int bgl_segment_mm(const void *a, const void *b, void *out, const int64_t *seglen, int64_t n,
                   int64_t d1, int64_t r, int64_t d2, int dtype, void *workspace,
                   size_t workspace_bytes, void *stream) {
    int rc = check_gmm("bgl_segment_mm", a, b, out, n, d1, r, d2, dtype);
    if (rc) return rc;
    if (n == 0 || d2 == 0) return BGL_OK;
    if (r > 0 && !seglen) return fail(BGL_E_INVALID, "bgl_segment_mm: null seglen");
    GmmLayout l = gmm_layout(workspace, n, d1, r, d2, dtype, false);
    if (workspace_bytes < l.bytes) return fail(BGL_E_WORKSPACE, "bgl_segment_mm: workspace too small");
    cudaStream_t s = as_stream(stream);
    const bool tc = dtype != BGL_F64 && gmm_tensor_core_supported(d1, d2, dtype) &&
                    gmm_tensor_core_fits(n, r, d2);
    l.tile_rows = tc ? 128 : 64;
    k_gmm_schedule<<<1, 32, 0, s>>>(seglen, r, n, l.tile_rows, l.seg_off, l.tile_off);
    BGL_LAUNCH_CHECK();
    int ecount = (int)((n * d2 + 255) / 256);
    if (ecount > num_sms() * 8) ecount = num_sms() * 8;
    if (ecount < 1) ecount = 1;
    if (dtype == BGL_F64)
        k_zero_tail<double><<<ecount, 256, 0, s>>>((double *)out, l.seg_off, r, n, d2);
    else if (dtype == BGL_F32)
        k_zero_tail<float><<<ecount, 256, 0, s>>>((float *)out, l.seg_off, r, n, d2);
    else
        k_zero_tail<unsigned short><<<ecount, 256, 0, s>>>((unsigned short *)out, l.seg_off, r, n, d2);
    BGL_LAUNCH_CHECK();
    if (d1 == 0) {
        // an empty contraction is all zeros
        BGL_CUDA(cudaMemsetAsync(out, 0, size_t(n) * d2 * elem_size(dtype), s));
        return BGL_OK;
    }
    if (r == 0) return BGL_OK;  // no segment: every row was zeroed above
    return run_gmm(a, b, out, l, n, d1, r, d2, dtype, tc, s);
}

size_t bgl_gather_mm_workspace_size(int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype) {
    if (n < 0 || r < 0 || d1 < 0 || d2 < 0) return 0;
    return gmm_layout(nullptr, n, d1, r, d2, dtype, true).bytes;
}

int bgl_gather_mm(const void *a, const void *b, const int64_t *idx_b, void *out, int64_t n,
                  int64_t d1, int64_t r, int64_t d2, int dtype, void *workspace,
                  size_t workspace_bytes, void *stream) {
    int rc = check_gmm("bgl_gather_mm", a, b, out, n, d1, r, d2, dtype);
    if (rc) return rc;
    if (n == 0 || d2 == 0) return BGL_OK;
    if (r < 1 || !idx_b) return fail(BGL_E_INVALID, "bgl_gather_mm: needs r >= 1 and idx_b");
    if (r >= (int64_t(1) << 31)) return fail(BGL_E_UNSUPPORTED, "bgl_gather_mm: r >= 2^31");
    GmmLayout l = gmm_layout(workspace, n, d1, r, d2, dtype, true);
    if (workspace_bytes < l.bytes) return fail(BGL_E_WORKSPACE, "bgl_gather_mm: workspace too small");
    cudaStream_t s = as_stream(stream);
    if (d1 == 0) {
        BGL_CUDA(cudaMemsetAsync(out, 0, size_t(n) * d2 * elem_size(dtype), s));
        return BGL_OK;
    }
    BGL_CUDA(cudaMemsetAsync(l.counts, 0, size_t(r) * sizeof(int64_t), s));
    int g = (int)((n + 255) / 256);
    if (g > num_sms() * 16) g = num_sms() * 16;
    const size_t hist_bytes = r <= kKeysSmem ? size_t(r) * sizeof(unsigned int) : 0;
    k_gmm_keys<<<g, 256, hist_bytes, s>>>(idx_b, l.keys, l.iota, l.counts, n, r);
    BGL_LAUNCH_CHECK();
    int bits = 1;
    while (bits < 31 && (int64_t(1) << bits) < r) ++bits;
    size_t tb = l.sort_temp_bytes;
    BGL_CUDA(cub::DeviceRadixSort::SortPairs(l.sort_temp, tb, l.keys, l.keys_sorted, l.iota,
                                             l.perm, (int)n, 0, bits, s));
    const bool tc = dtype != BGL_F64 && gmm_tensor_core_supported(d1, d2, dtype) &&
                    gmm_tensor_core_fits(n, r, d2);
    l.tile_rows = tc ? 128 : 64;
    k_gmm_schedule<<<1, 32, 0, s>>>(l.counts, r, n, l.tile_rows, l.seg_off, l.tile_off);
    BGL_LAUNCH_CHECK();
    return run_gmm(a, b, out, l, n, d1, r, d2, dtype, tc, s);
}

}  // extern "C"
