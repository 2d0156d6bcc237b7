// gSpMM launch chain (shared by the per-element-type translation units):
// op, reduce and operand-mode dispatch onto the k_spmm instantiations, then
// the split-row fixup.
#pragma once

#include "spmm_impl.cuh"

namespace bgl {
namespace {

template <typename T, int OP, int RED, int V, int J, bool ACC, int LM, int RM, bool NARROW = false>
int launch_kernels(const SpmmArgs<T> &a, cudaStream_t s) {
    int64_t threads = a.num_chunks * a.num_slices * a.ts;
    int grid = (int)((threads + kSpmmBlock - 1) / kSpmmBlock);
    if (grid < 1) grid = 1;
    // the gather ring lives in dynamic shared memory (64 KB per block for
    // 16-byte slots, 48 KB for the narrow ring), above the 48 KB a launch gets
    // without opting in
    constexpr int smem = Stages<T, OP, V, NARROW>::smem;
    auto k = k_spmm<T, OP, RED, V, J, ACC, LM, RM, NARROW>;
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

template <typename T, int OP, int RED, int V, int J, int LM, int RM, bool NARROW>
int launch_one(const SpmmArgs<T> &a, cudaStream_t s) {
    return a.accumulate ? launch_kernels<T, OP, RED, V, J, true, LM, RM, NARROW>(a, s)
                        : launch_kernels<T, OP, RED, V, J, false, LM, RM, NARROW>(a, s);
}

template <typename T, int OP, int V, int J, int LM = -1, int RM = -1, bool NARROW = false>
int by_reduce(const SpmmArgs<T> &a, int red, cudaStream_t s) {
    switch (red) {
    case BGL_RED_SUM: return launch_one<T, OP, BGL_RED_SUM, V, J, LM, RM, NARROW>(a, s);
    case BGL_RED_MEAN: return launch_one<T, OP, BGL_RED_MEAN, V, J, LM, RM, NARROW>(a, s);
    // values only (no arg output, no accumulation): no winning positions
    // (the kernels that keep winning positions carry more registers than the
    // narrow ring's 64 allow: they always take the default ring)
    case BGL_RED_MAX:
        if (!a.arg_u && !a.arg_e && !a.accumulate)
            return launch_kernels<T, OP, kRedMaxValue, V, J, false, LM, RM, NARROW>(a, s);
        return launch_one<T, OP, BGL_RED_MAX, V, J, LM, RM, false>(a, s);
    case BGL_RED_MIN:
        if (!a.arg_u && !a.arg_e && !a.accumulate)
            return launch_kernels<T, OP, kRedMinValue, V, J, false, LM, RM, NARROW>(a, s);
        return launch_one<T, OP, BGL_RED_MIN, V, J, LM, RM, false>(a, s);
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
// count at narrow rows, where the walk is issue-bound).  Float rows of 16 to
// 64 columns (teams of 4 to 16 lanes, several a warp) take the narrow ring:
// two groups in flight instead of three, four blocks an SM instead of three
// -- more warps to cover the latency of the ids and row ends that the teams
// of a warp wait on.  Measured on config 3's graph (copy_u_mean, whole
// graph, A/B on one box): D = 64 4.14 -> 3.79 ms, D = 32 2.24 -> 2.09 ms,
// D = 16 1.59 -> 1.50 ms; at D = 128 the narrow ring was 1 % slower and at
// D = 8 1-2 % slower.
template <typename T, int OP, int V, int J>
int by_copy_mode(const SpmmArgs<T> &a, int red, cudaStream_t s) {
    if constexpr (V > 1) {
        constexpr int L = OP == BGL_OP_COPY_LHS ? 0 : -1, R = OP == BGL_OP_COPY_RHS ? 0 : -1;
        if ((OP == BGL_OP_COPY_LHS && a.lhs.full) || (OP == BGL_OP_COPY_RHS && a.rhs.full)) {
            if constexpr (sizeof(T) == 4)
                if (a.ts >= 4 && a.ts < 32) return by_reduce<T, OP, V, J, L, R, true>(a, red, s);
            return by_reduce<T, OP, V, J, L, R>(a, red, s);
        }
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

}  // namespace bgl
