"""Fused GAT aggregation (a next step beyond the reference's operator set).

The reference runs a GAT layer's attention as four operators: ``u_add_v`` of
the per-node scores (ops/sddmm.py), the caller's leaky_relu, ``edge_softmax``
over each destination's in-edges (ops/edge_softmax.py) and ``u_mul_e_sum`` of
the features by the attention (ops/spmm.py).  ``gat_aggregate`` computes the
same result in one device pass over the in-CSR with an online softmax per
destination row, without writing the (E, H) scores or attention weights.
"""

from __future__ import annotations

import torch

from .. import _tensor as T
from .._lib import check, lib
from ..base import DGLError

__all__ = ["gat_aggregate"]


def _heads(x, n, h, what):
    shape = tuple(T.shape_of(x))
    if len(shape) == 3 and shape[2] == 1:
        shape = shape[:2]
    if shape != (n, h):
        raise DGLError("{} must be ({}, {}) or ({}, {}, 1), got {}".format(
            what, n, h, n, h, tuple(T.shape_of(x))))


def gat_aggregate(graph, feat, el, er, negative_slope=0.2):
    r"""out[v] = sum over in-edges e = (u, v) of a_e * feat[u], per head, with
    a = edge_softmax(leaky_relu(el[u] + er[v])) over each node's in-edges.

    ``feat`` is (N, H, D); ``el`` and ``er`` are (N, H) or (N, H, 1).
    Returns (N, H, D); nodes without in-edges get 0.  Equal, within floating
    point rounding, to ``u_mul_e_sum(g, feat, edge_softmax(g,
    leaky_relu(u_add_v(g, el, er))))``.
    """
    kind = T.kind_of(feat, el, er)
    feat, el, er = T.feature(feat), T.feature(el), T.feature(er)
    fs = tuple(T.shape_of(feat))
    if len(fs) != 3:
        raise DGLError("feat must be (N, H, D), got {}".format(fs))
    n = graph.number_of_nodes()
    if fs[0] != n:
        raise DGLError("feat has {} rows but the graph has {} nodes".format(fs[0], n))
    h, d = int(fs[1]), int(fs[2])
    _heads(el, n, h, "el")
    _heads(er, n, h, "er")
    dtype = T.common_float(feat, el, er)
    out = torch.empty((n, h * d), dtype=dtype, device=T.device())
    if n and h and d:
        ft = T.to_dev(feat, dtype).reshape(n, h * d)
        elt = T.to_dev(el, dtype).reshape(n, h)
        ert = T.to_dev(er, dtype).reshape(n, h)
        indptr, indices, _, _ = graph._device().in_csr
        ne = graph.number_of_edges()
        code = T.code_of(dtype)
        nbytes = lib().bgl_gat_workspace_size(n, ne, h, d, code)
        ws = T.workspace(nbytes)
        check(lib().bgl_gat_aggregate(T.ptr(indptr), T.ptr(indices), n, ne, T.ptr(ft), T.ptr(elt),
                                      T.ptr(ert), h, d, float(negative_slope), T.ptr(out), code,
                                      T.ptr(ws), nbytes, T.stream()), "gat_aggregate")
    return T.result(out.reshape(n, h, d), kind)
