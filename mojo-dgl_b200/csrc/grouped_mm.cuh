// Shared declarations of the grouped GEMM (segment_mm / gather_mm).
#pragma once

#include "common.cuh"

namespace bgl {

// Device-side schedule of one grouped product, carved from the caller's
// workspace.  seg_off[r + 1]: first row of each segment (in the permuted order
// for gather_mm); tile_off[r + 1]: first tile of each segment; perm (gather_mm
// only): the stable sort of the row ids by idx_b.
struct GmmLayout {
    int64_t *seg_off;
    int64_t *tile_off;
    int64_t *counts;
    int32_t *keys;
    int32_t *keys_sorted;
    int32_t *iota;
    int32_t *perm;
    void *tc_b;  // tensor-core path: K-major copy of B (r x d2 x d1)
    void *sort_temp;
    size_t sort_temp_bytes;
    int64_t tile_rows;
    size_t bytes;
};

GmmLayout gmm_layout(void *ws, int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype,
                     bool gather);

// tcgen05 path (grouped_mm_tc.cu).
bool gmm_tensor_core_supported(int64_t d1, int64_t d2, int dtype);
bool gmm_tensor_core_fits(int64_t n, int64_t r, int64_t d2);
int gmm_tensor_core(const void *a, const void *b, void *out, const GmmLayout &l, int64_t n,
                    int64_t d1, int64_t r, int64_t d2, int dtype, cudaStream_t s);

}  // namespace bgl
