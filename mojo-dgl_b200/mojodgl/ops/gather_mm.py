"""gather_mm: out[i] = a[i] @ b[idx_b[i]].

Same public surface and validation as the reference's
python/mojodgl/ops/gather_mm.py:21-92.  The reference chooses between a fused
per-row kernel and a sort -> segment_mm -> unsort route on the size of the b
block (``gather_mm.py:79-91``); both compute the same product.  Here there is
one device route: a stable sort of the row ids by ``idx_b``, then the grouped
tensor-core GEMM reading A rows through the permutation and writing output
rows back through it.  ``_SEGMENT_BLOCK`` is kept so code that tunes the
reference's cut still runs; it does not change the result or the route.
"""

from __future__ import annotations

import os

import torch

from .. import _tensor as T
from .._lib import check, lib
from ..base import DGLError
from .segment import _mm_dtype

__all__ = ["gather_mm"]

_SEGMENT_BLOCK = int(os.environ.get("MOJODGL_GATHER_MM_SEGMENT_BLOCK", 16384))


def gather_mm(a, b, *, idx_b):
    r"""Gather a block of ``b`` per row and multiply: ``c[i] = a[i] @ b[idx_b[i]]``.

    ``a`` is (N, D1), ``b`` is (R, D1, D2), ``idx_b`` is (N,) integers in
    [0, R).  float32 runs in TF32 on the tensor cores, bfloat16 tensors in
    BF16 (fp32 accumulate), float64 exactly.  Returns (N, D2).
    """
    kind = T.kind_of(a, b, idx_b)
    dtype = _mm_dtype(a, b)
    if dtype != torch.bfloat16:
        a, b = T.feature(a), T.feature(b)
    if len(T.shape_of(a)) != 2 or len(T.shape_of(b)) != 3:
        raise DGLError("gather_mm wants a 2-D and a 3-D operand")
    n, d1 = T.shape_of(a)
    r, b_d1, d2 = T.shape_of(b)
    if b_d1 != d1:
        raise DGLError("inner dimensions do not match: a is {} wide, b blocks are {}".format(d1, b_d1))
    idx = T.ids(idx_b)
    if len(T.shape_of(idx)) != 1 or T.shape_of(idx)[0] != n:
        raise DGLError("idx_b must be 1-D with one index per row of a: got shape {} for N={}".format(
            T.shape_of(idx), n))
    it = T.to_dev(idx)
    if n and (int(it.min()) < 0 or int(it.max()) >= r):
        raise DGLError("idx_b must be in [0, {}), got [{}, {})".format(
            r, int(it.min()), int(it.max()) + 1))
    out = torch.empty((n, d2), dtype=dtype, device=T.device())
    if n and d2:
        at, bt = T.to_dev(a, dtype), T.to_dev(b, dtype)
        code = T.code_of(dtype)
        nbytes = lib().bgl_gather_mm_workspace_size(n, d1, r, d2, code)
        ws = T.workspace(nbytes)
        rc = lib().bgl_gather_mm(T.ptr(at), T.ptr(bt), T.ptr(it), T.ptr(out), n, d1, r, d2, code,
                                 T.ptr(ws), nbytes, T.stream())
        check(rc, "gather_mm")
    return T.result(out, kind)
