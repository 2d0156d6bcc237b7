"""Segment operators: segment_reduce, segment_softmax, segment_mm.

Same public surface and validation as the reference's
python/mojodgl/ops/segment.py:62-214.  A segment list is a CSR whose items are
the consecutive rows of ``value``, so segment_reduce runs on the gSpMM engine
(copy of the row, identity gather) with the mean divide and the max/min
inf->0 replacement fused into its epilogue, and segment_softmax runs on the
fused softmax kernel; segment_mm is the grouped GEMM (tcgen05 for fp32/bf16).
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _tensor as T
from .._lib import BGL_ZERO_INF, OP_COPY_RHS, REDUCERS, check, lib
from ..base import DGLError
from .sddmm import flat_feature, out_shape

__all__ = ["segment_reduce", "segment_softmax", "segment_mm"]


def _offsets(seglen):
    """[0, cumsum(seglen)] as a device int64 tensor, plus its last value and
    whether it is non-decreasing (python/mojodgl/ops/segment.py:12-38)."""
    seglen = T.ids(seglen)
    if T.is_torch(seglen):
        dev = T.to_dev(seglen)
        off = torch.zeros(dev.numel() + 1, dtype=torch.int64, device=dev.device)
        if dev.numel():
            torch.cumsum(dev, 0, out=off[1:])
        ok = bool((dev >= 0).all()) if dev.numel() else True
        return off, int(off[-1]), ok, seglen
    off = np.zeros(seglen.size + 1, dtype=np.int64)
    np.cumsum(seglen, out=off[1:])
    ok = bool(np.all(seglen >= 0)) if seglen.size else True
    return T.to_dev(off), int(off[-1]), ok, seglen


def _check_offsets(total: int, ok: bool, n: int) -> None:
    if total != n or not ok:
        raise DGLError(
            "segment lengths must be non-negative and sum to {}, got offsets ending at {} "
            "for {} rows".format(n, total, n))


def segment_reduce(seglen, value, reducer="sum"):
    """Reduce the rows of ``value`` by consecutive segments.

    ``seglen[i]`` rows form segment i (zero-length segments allowed; the
    lengths must sum to ``len(value)``).  ``reducer`` is ``sum``, ``max``,
    ``min`` or ``mean``; empty segments give 0 for every reducer.
    """
    if reducer not in ("sum", "max", "min", "mean"):
        raise DGLError("reducer {} not recognized.".format(reducer))
    kind = T.kind_of(seglen, value)
    offsets, total, ok, seglen = _offsets(seglen)
    value = T.feature(value)
    shape = T.shape_of(value)
    n = shape[0] if shape else 0
    _check_offsets(total, ok, n)
    feat, d = flat_feature(value)
    num_seg = int(offsets.numel()) - 1
    dtype = T.common_float(value)
    out = torch.empty((num_seg, d), dtype=dtype, device=T.device())
    if num_seg and d:
        vt = T.to_dev(value, dtype)
        red = REDUCERS[reducer]
        nbytes = lib().bgl_gspmm_workspace_size(num_seg, n, d, T.code_of(dtype), red)
        ws = T.workspace(nbytes)
        flags = BGL_ZERO_INF if reducer in ("max", "min") else 0
        rc = lib().bgl_gspmm(T.ptr(offsets), None, None, None, num_seg, n, None, 1, 1, T.ptr(vt),
                             d, 1, T.ptr(out), d, None, None, T.code_of(dtype), OP_COPY_RHS, red,
                             flags, T.ptr(ws), nbytes, T.stream())
        check(rc, "segment_reduce")
    return T.result(out.reshape(out_shape(num_seg, feat, len(feat))), kind)


def segment_softmax(seglen, value):
    """Softmax over the rows of each segment, independently per column.
    Returns an array shaped like ``value``."""
    kind = T.kind_of(seglen, value)
    offsets, total, ok, seglen = _offsets(seglen)
    value = T.feature(value)
    shape = T.shape_of(value)
    n = shape[0] if shape else 0
    _check_offsets(total, ok, n)
    feat, d = flat_feature(value)
    num_seg = int(offsets.numel()) - 1
    dtype = T.common_float(value)
    # every row of value belongs to one segment and is written
    out = torch.empty((n, d), dtype=dtype, device=T.device())
    if num_seg and n and d:
        vt = T.to_dev(value, dtype)
        nbytes = lib().bgl_softmax_workspace_size(num_seg, n, d, T.code_of(dtype))
        ws = T.workspace(nbytes)
        rc = lib().bgl_edge_softmax(T.ptr(offsets), None, None, num_seg, n, T.ptr(vt), T.ptr(out),
                                    d, T.code_of(dtype), T.ptr(ws), nbytes, T.stream())
        check(rc, "segment_softmax")
    return T.result(out.reshape(shape), kind)


def _mm_dtype(a, b):
    if T.is_torch(a) and T.is_torch(b) and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
        return torch.bfloat16
    return T.common_float(T.feature(a), T.feature(b))


def segment_mm(a, b, seglen_a):
    r"""Per-segment matrix products: with ``seglen_a == [10, 5, 0, 3]``,
    ``a[0:10] @ b[0]``, ``a[10:15] @ b[1]``, ``a[15:15] @ b[2]``,
    ``a[15:18] @ b[3]``.  ``a`` is (N, D1), ``b`` is (R, D1, D2); rows past
    ``sum(seglen_a)`` are zero.  float32 runs in TF32 on the tensor cores,
    bfloat16 tensors in BF16 (fp32 accumulate), float64 exactly.
    """
    kind = T.kind_of(a, b, seglen_a)
    dtype = _mm_dtype(a, b)
    if dtype != torch.bfloat16:
        a, b = T.feature(a), T.feature(b)
    if len(T.shape_of(a)) != 2 or len(T.shape_of(b)) != 3:
        raise DGLError("segment_mm wants a 2-D left operand and a 3-D right operand")
    n, d1 = T.shape_of(a)
    r, b_d1, d2 = T.shape_of(b)
    if b_d1 != d1:
        raise DGLError("inner dimensions do not match: {} vs {}".format(d1, b_d1))
    seg = T.ids(seglen_a)
    seg_np = seg.cpu().numpy() if T.is_torch(seg) else seg
    if seg_np.size != r:
        raise DGLError("seglen_a must have one entry per b block: {} != {}".format(seg_np.size, r))
    if seg_np.size:
        lo, total = int(seg_np.min()), int(seg_np.sum())
        if lo < 0 or total > n:
            raise DGLError("segment lengths must be non-negative and sum to {}, got a minimum of "
                           "{} and a sum of {}".format(n, lo, total))
    # the library writes every row (rows past sum(seglen_a) as zeros)
    out = torch.empty((n, d2), dtype=dtype, device=T.device())
    if n:
        at, bt, st = T.to_dev(a, dtype), T.to_dev(b, dtype), T.to_dev(seg)
        code = T.code_of(dtype)
        nbytes = lib().bgl_segment_mm_workspace_size(n, d1, r, d2, code)
        ws = T.workspace(nbytes)
        rc = lib().bgl_segment_mm(T.ptr(at), T.ptr(bt), T.ptr(out), T.ptr(st), n, d1, r, d2, code,
                                  T.ptr(ws), nbytes, T.stream())
        check(rc, "segment_mm")
    return T.result(out, kind)
