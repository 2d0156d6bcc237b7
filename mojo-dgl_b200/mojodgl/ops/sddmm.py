"""gSDDMM: edge features computed from node/edge operand pairs.

Same public surface as the reference's python/mojodgl/ops/sddmm.py (gsddmm,
copy_u/copy_v/copy_e and the 30 generated ``{u,v,e}_{op}_{u,v,e}``, registered
by ``sddmm.py:218-226``), computed by ``bgl_gsddmm`` on the device.

Broadcasting: the reference accepts 1-D/2-D features and widens a ``(n, 1)``
column (``sddmm.py:50-68``).  This build accepts the same shapes with the same
results and additionally DGL's head broadcast over trailing axes (for example
``(N, H, D)`` against ``(E, H, 1)``), which the kernels read in place through
a (width, div) operand descriptor instead of materialising the broadcast.
"""

from __future__ import annotations

import sys
from itertools import product

import numpy as np
import torch

from .. import _tensor as T
from .._lib import BINARY_OPS, OP_COPY_LHS, OP_COPY_RHS, OP_DOT, TARGETS, check, lib
from ..base import DGLError

__all__ = ["gsddmm", "copy_u", "copy_v", "copy_e"]


def reshape_lhs_rhs(lhs_data, rhs_data):
    """Pad the shorter operand's feature shape with unit axes right after the
    row axis, so both have the same rank ((N, 3, 1) & (E, 5, 3, 4) ->
    (N, 1, 3, 1) & (E, 5, 3, 4)); the reference's sddmm.py:24-47."""
    ls, rs = tuple(np.shape(lhs_data)), tuple(np.shape(rhs_data))
    if len(ls) == len(rs):
        return lhs_data, rhs_data
    rank = max(len(ls), len(rs))
    lhs_data = lhs_data.reshape((ls[0],) + (1,) * (rank - len(ls)) + ls[1:])
    rhs_data = rhs_data.reshape((rs[0],) + (1,) * (rank - len(rs)) + rs[1:])
    return lhs_data, rhs_data


def _prod(shape) -> int:
    p = 1
    for s in shape:
        p *= int(s)
    return p


def bcast_desc(xf, of):
    """(width, div) such that output column k reads operand column
    (k // div) % width, or None when the operand's kept axes are not one
    contiguous run (the caller then materialises the broadcast)."""
    xf, of = tuple(xf), tuple(of)
    if xf == of:
        return max(_prod(of), 1), 1
    axes = [i for i in range(len(of)) if of[i] != 1]
    kept = [i for i in axes if xf[i] == of[i]]
    if not kept:
        return 1, 1
    pos = [axes.index(i) for i in kept]
    if pos != list(range(pos[0], pos[0] + len(pos))):
        return None
    width = _prod(of[i] for i in kept)
    div = _prod(of[i] for i in axes[pos[-1] + 1:])
    return width, div


def flat_feature(a):
    """(n, ...) feature -> its element type, feature shape and row width."""
    shape = T.shape_of(a)
    feat = shape[1:] if len(shape) > 1 else ()
    return feat, max(_prod(feat), 1)


def check_rows(a, want: int, what: str) -> None:
    """Reject an operand whose row count its target does not imply (the
    reference's sddmm.py:71-80, upstream's check.h)."""
    n = T.shape_of(a)[0] if len(T.shape_of(a)) else 0
    if n != want:
        raise DGLError("{} data must have {} rows, got {}".format(what, want, n))


class Binary:
    """Device operands of a broadcast binary op, ready for the kernels."""

    def __init__(self, lhs, rhs, dtype):
        lhs, rhs = reshape_lhs_rhs(lhs, rhs)
        lf, _ = flat_feature(lhs)
        rf, _ = flat_feature(rhs)
        try:
            of = tuple(np.broadcast_shapes(lf, rf))
        except ValueError:
            raise DGLError("operands are not broadcastable: {} and {}".format(
                T.shape_of(lhs), T.shape_of(rhs)))
        self.out_feat = of
        self.dout = max(_prod(of), 1)
        self.lhs, self.lw, self.ldiv = self._operand(lhs, lf, of, dtype)
        self.rhs, self.rw, self.rdiv = self._operand(rhs, rf, of, dtype)
        self.rank = len(of)

    @staticmethod
    def _operand(x, xf, of, dtype):
        d = bcast_desc(xf, of)
        t = T.to_dev(x, dtype)
        if d is None:  # a broadcast the descriptor cannot express: materialise it
            t = t.reshape((t.shape[0],) + tuple(xf)).expand((t.shape[0],) + tuple(of)).contiguous()
            d = (max(_prod(of), 1), 1)
        return t, d[0], d[1]


def out_shape(n: int, feat, rank_hint: int):
    """The reference returns 2-D (n, d) results for its 1-D/2-D operands
    (spmm.py:102, sddmm.py:386); rank-3+ operands keep their feature shape."""
    if rank_hint <= 1:
        return (n, max(_prod(feat), 1))
    return (n,) + tuple(feat)


def gsddmm(g, op, lhs_data, rhs_data, lhs_target="u", rhs_target="v"):
    r"""Generalized sampled-dense-dense matrix multiplication.

    .. math:: x_e = \phi(x_{lhs}, x_{rhs}), \forall (u, e, v) \in \mathcal{G}

    ``op`` is ``add``, ``sub``, ``mul``, ``div``, ``dot``, ``copy_lhs`` or
    ``copy_rhs``; ``lhs_target``/``rhs_target`` pick ``u`` (source), ``v``
    (destination) or ``e`` (edge) for each operand.  Returns the per-edge
    result, ``(E, 1)`` for ``dot``.
    """
    if lhs_target not in TARGETS or rhs_target not in TARGETS:
        raise DGLError("lhs_target/rhs_target must be one of 'u', 'v', 'e'")
    if op not in list(BINARY_OPS) + ["copy_lhs", "copy_rhs"]:
        raise DGLError("op {} not recognized".format(op))
    num_edges = g.number_of_edges()
    num_nodes = g.number_of_nodes()
    kind = T.kind_of(lhs_data, rhs_data)
    lhs = None if lhs_data is None else T.feature(lhs_data)
    rhs = None if rhs_data is None else T.feature(rhs_data)
    dtype = T.common_float(lhs, rhs)

    def rows_for(target):
        return (num_edges, "edge") if target == "e" else (num_nodes, "node")

    if lhs is not None:
        check_rows(lhs, *rows_for(lhs_target))
    if rhs is not None:
        check_rows(rhs, *rows_for(rhs_target))

    dg = g._device()
    if op in ("copy_lhs", "copy_rhs"):
        src = lhs if op == "copy_lhs" else rhs
        if src is None:
            raise DGLError("{} needs its operand".format(op))
        feat, d = flat_feature(src)
        xt = T.to_dev(src, dtype)
        out = torch.empty((num_edges, d), dtype=dtype, device=T.device())
        code = OP_COPY_LHS if op == "copy_lhs" else OP_COPY_RHS
        tgt = TARGETS[lhs_target if op == "copy_lhs" else rhs_target]
        rc = lib().bgl_gsddmm(T.ptr(dg.u32), T.ptr(dg.v32), num_edges, T.ptr(xt), d, 1, tgt,
                              T.ptr(xt), d, 1, tgt, T.ptr(out), d, 0, T.code_of(dtype), code,
                              T.stream())
        check(rc, "gsddmm")
        return T.result(out.reshape(out_shape(num_edges, feat, len(feat))), kind)
    if lhs is None or rhs is None:
        raise DGLError("{} needs both operands".format(op))
    if op == "dot":
        lf, dl = flat_feature(lhs)
        rf, dr = flat_feature(rhs)
        if len(lf) > 1 or len(rf) > 1:
            raise DGLError("dot handles 1-D and 2-D features, got {} and {}".format(
                T.shape_of(lhs), T.shape_of(rhs)))
        if dl != dr:
            raise DGLError("dot needs matching feature widths, {} vs {}".format(dl, dr))
        lt, rt = T.to_dev(lhs, dtype), T.to_dev(rhs, dtype)
        out = torch.empty((num_edges, 1), dtype=dtype, device=T.device())
        rc = lib().bgl_gsddmm(T.ptr(dg.u32), T.ptr(dg.v32), num_edges, T.ptr(lt), dl, 1,
                              TARGETS[lhs_target], T.ptr(rt), dr, 1, TARGETS[rhs_target],
                              T.ptr(out), 1, dl, T.code_of(dtype), OP_DOT, T.stream())
        check(rc, "gsddmm")
        return T.result(out, kind)
    b = Binary(lhs, rhs, dtype)
    out = torch.empty((num_edges, b.dout), dtype=dtype, device=T.device())
    rc = lib().bgl_gsddmm(T.ptr(dg.u32), T.ptr(dg.v32), num_edges, T.ptr(b.lhs), b.lw, b.ldiv,
                          TARGETS[lhs_target], T.ptr(b.rhs), b.rw, b.rdiv, TARGETS[rhs_target],
                          T.ptr(out), b.dout, 0, T.code_of(dtype), BINARY_OPS[op], T.stream())
    check(rc, "gsddmm")
    return T.result(out.reshape(out_shape(num_edges, b.out_feat, b.rank)), kind)


def _make_sddmm(lhs_target, rhs_target, binary_op):
    names = {"u": "source node", "v": "destination node", "e": "edge"}

    def func(g, x, y):
        return gsddmm(g, binary_op, x, y, lhs_target=lhs_target, rhs_target=rhs_target)

    func.__name__ = "{}_{}_{}".format(lhs_target, binary_op, rhs_target)
    func.__doc__ = (
        "Generalized SDDMM: the edge feature {op}({l} feature x, {r} feature y).\n\n"
        "Operands broadcast over their trailing axes with NumPy semantics; "
        "`dot` contracts the feature axis to one column.".format(
            op=binary_op, l=names[lhs_target], r=names[rhs_target]))
    return func


for _l, _r in product("uve", "uve"):
    if _l != _r:
        for _op in ("add", "sub", "mul", "div", "dot"):
            _f = _make_sddmm(_l, _r, _op)
            setattr(sys.modules[__name__], _f.__name__, _f)
            __all__.append(_f.__name__)


def copy_u(g, x):
    """Copy source node features to their out-edges."""
    return gsddmm(g, "copy_lhs", x, None)


def copy_v(g, x):
    """Copy destination node features to their in-edges."""
    return gsddmm(g, "copy_rhs", None, x)


def copy_e(g, x):
    """Edge features are already per edge: returned as given."""
    return x
