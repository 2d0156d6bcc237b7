// gSpMM kernel instantiations for float (one translation unit per element type
// so the float and the other element type's kernels compile in parallel).
#include "spmm_impl.cuh"

namespace bgl {
namespace {

template <typename T, int OP, int RED, int V, int J, bool ACC, int LM, int RM>
int launch_kernels(const SpmmArgs<T> &a, cudaStream_t s) {
    int64_t threads = a.num_chunks * a.num_slices * a.ts;
    int grid = (int)((threads + kSpmmBlock - 1) / kSpmmBlock);
    if (grid < 1) grid = 1;
    // the gather ring lives in dynamic shared memory (64 KB per block for
    // 16-byte slots), above the 48 KB a launch gets without opting in
    constexpr int smem = Stages<T, OP, V>::smem;
    auto k = k_spmm<T, OP, RED, V, J, ACC, LM, RM>;
    BGL_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    BGL_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  cudaSharedmemCarveoutMaxShared));
    k<<<grid, kSpmmBlock, smem, s>>>(a);
    BGL_LAUNCH_CHECK();
    int fgrid = (int)((a.num_chunks * a.ts + 255) / 256);
    if (fgrid < 1) fgrid = 1;
    k_spmm_fixup<T, RED, V, J, ACC><<<fgrid, 256, 0, s>>>(a);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

template <typename T, int OP, int RED, int V, int J, int LM, int RM>
int launch_one(const SpmmArgs<T> &a, cudaStream_t s) {
    return a.accumulate ? launch_kernels<T, OP, RED, V, J, true, LM, RM>(a, s)
                        : launch_kernels<T, OP, RED, V, J, false, LM, RM>(a, s);
}

template <typename T, int OP, int V, int J, int LM = -1, int RM = -1>
int by_reduce(const SpmmArgs<T> &a, int red, cudaStream_t s) {
    switch (red) {
    case BGL_RED_SUM: return launch_one<T, OP, BGL_RED_SUM, V, J, LM, RM>(a, s);
    case BGL_RED_MEAN: return launch_one<T, OP, BGL_RED_MEAN, V, J, LM, RM>(a, s);
    // values only (no arg output, no accumulation): no winning positions
    case BGL_RED_MAX:
        if (!a.arg_u && !a.arg_e && !a.accumulate)
            return launch_kernels<T, OP, kRedMaxValue, V, J, false, LM, RM>(a, s);
        return launch_one<T, OP, BGL_RED_MAX, V, J, LM, RM>(a, s);
    case BGL_RED_MIN:
        if (!a.arg_u && !a.arg_e && !a.accumulate)
            return launch_kernels<T, OP, kRedMinValue, V, J, false, LM, RM>(a, s);
        return launch_one<T, OP, BGL_RED_MIN, V, J, LM, RM>(a, s);
    }
    return fail(BGL_E_INVALID, "gspmm: reduce code %d", red);
}

// A binary op on vectors whose operands are full rows on both sides, or full
// node rows against a per-head broadcast (attention weights): the kernels
// with those modes fixed.  Any other combination runs the general kernels.
template <typename T, int OP, int V, int J>
int by_modes(const SpmmArgs<T> &a, int red, cudaStream_t s) {
    if constexpr (V > 1) {
        if (a.lhs.full) {
            if (a.rhs.full) return by_reduce<T, OP, V, J, 0, 0>(a, red, s);
            if (a.rhs.uniform) return by_reduce<T, OP, V, J, 0, 1>(a, red, s);
        }
    }
    return by_reduce<T, OP, V, J>(a, red, s);
}

// A copy op on vectors reading full rows (the common case: node or edge
// features with no broadcast): the kernels with the read operand's mode
// fixed, so the per-edge copy and read-back carry no mode branches (they
// count at narrow rows, where the walk is issue-bound).
template <typename T, int OP, int V, int J>
int by_copy_mode(const SpmmArgs<T> &a, int red, cudaStream_t s) {
    if constexpr (V > 1) {
        if (OP == BGL_OP_COPY_LHS && a.lhs.full) return by_reduce<T, OP, V, J, 0, -1>(a, red, s);
        if (OP == BGL_OP_COPY_RHS && a.rhs.full) return by_reduce<T, OP, V, J, -1, 0>(a, red, s);
    }
    return by_reduce<T, OP, V, J>(a, red, s);
}

}  // namespace

template <typename T, int V, int J>
int launch_spmm_vj(const SpmmArgs<T> &a, int op, int red, cudaStream_t s) {
    switch (op) {
    case BGL_OP_ADD: return by_modes<T, BGL_OP_ADD, V, J>(a, red, s);
    case BGL_OP_SUB: return by_modes<T, BGL_OP_SUB, V, J>(a, red, s);
    case BGL_OP_MUL: return by_modes<T, BGL_OP_MUL, V, J>(a, red, s);
    case BGL_OP_DIV: return by_modes<T, BGL_OP_DIV, V, J>(a, red, s);
    case BGL_OP_COPY_LHS: return by_copy_mode<T, BGL_OP_COPY_LHS, V, J>(a, red, s);
    case BGL_OP_COPY_RHS: return by_copy_mode<T, BGL_OP_COPY_RHS, V, J>(a, red, s);
    }
    return fail(BGL_E_INVALID, "gspmm: op code %d", op);
}

template int launch_spmm_vj<float, 1, 1>(const SpmmArgs<float> &, int, int, cudaStream_t);
template int launch_spmm_vj<float, 4, 1>(const SpmmArgs<float> &, int, int, cudaStream_t);

}  // namespace bgl
