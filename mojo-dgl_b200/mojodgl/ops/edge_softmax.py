"""edge_softmax: softmax of edge logits over each node's in-edges (or out-edges).

Same public surface, shapes and validation as the reference's
python/mojodgl/ops/edge_softmax.py:11-173, on the fused device softmax.  With
``eids`` a subset, the reference reproduces upstream's positional rule
(``edge_softmax.py:119-158``): the selection's POSITIONS are grouped by the
endpoint of the selected edge (ascending node id, positions in the order they
appear in ``eids``) and position i takes the softmax of ``logits[i]`` over its
group; the result is as long as ``logits`` with the selected results in its
first ``len(eids)`` rows.  The reference builds that grouping in a Python loop;
here it is a stable device sort of the endpoint keys.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _tensor as T
from .._lib import check, lib
from ..base import ALL, DGLError, is_all

__all__ = ["edge_softmax"]


def edge_softmax(graph, logits, eids=ALL, norm_by="dst"):
    r"""Softmax of edge logits over the edges sharing a destination
    (``norm_by="dst"``, GAT's attention) or a source (``norm_by="src"``).

    .. math:: a_{ij} = \frac{\exp(z_{ij})}{\sum_{j \in \mathcal{N}(i)} \exp(z_{ij})}

    ``logits`` is ``(E,)``, ``(E, 1)`` or ``(E, *, 1)``; every trailing column
    is an independent softmax.  Returns an array shaped like ``logits``.
    """
    num_edges = graph.number_of_edges()
    kind = T.kind_of(logits, None if is_all(eids) else eids)
    logits = T.feature(logits)
    shape = T.shape_of(logits)
    if len(shape) == 1:
        d = 1
    elif len(shape) >= 2 and shape[-1] == 1:
        d = int(np.prod(shape[1:]))
    else:
        raise DGLError("logits must be (E,), (E, 1) or (E, *, 1); got shape {}".format(shape))
    if norm_by not in ("dst", "src"):
        raise DGLError("norm_by must be 'src' or 'dst'")
    out_len = shape[0]
    dtype = T.common_float(logits)
    dg = graph._device()
    if is_all(eids):
        if out_len != num_edges:
            raise DGLError("logits has {} rows but the graph has {} edges".format(out_len, num_edges))
        indptr, _, eid, _ = dg.in_csr if norm_by == "dst" else dg.out_csr
        num_rows, num_items, k = graph.number_of_nodes(), num_edges, None
        edge_row = dg.v32 if norm_by == "dst" else dg.u32  # every edge's row, by edge id
        lt = T.to_dev(logits, dtype).reshape(out_len, d)
    else:
        order = T.ids(eids)
        order_t = T.to_dev(order).reshape(-1)
        k = int(order_t.numel())
        if k and (int(order_t.min()) < 0 or int(order_t.max()) >= num_edges):
            raise DGLError("edge ids must be in [0, {}), got [{}, {})".format(
                num_edges, int(order_t.min()), int(order_t.max()) + 1))
        if k > out_len:
            raise DGLError("{} edge ids selected but logits has only {} rows".format(k, out_len))
        key_all = dg.v64 if norm_by == "dst" else dg.u64
        key = key_all[order_t]
        _, pos = torch.sort(key, stable=True)
        eid = pos.to(torch.int32)
        if k:
            _, counts = torch.unique_consecutive(key[pos], return_counts=True)
            indptr = torch.zeros(counts.numel() + 1, dtype=torch.int64, device=key.device)
            torch.cumsum(counts, 0, out=indptr[1:])
        else:
            indptr = torch.zeros(1, dtype=torch.int64, device=key.device)
        num_rows, num_items = int(indptr.numel()) - 1, k
        edge_row = None
        lt = T.to_dev(logits, dtype).reshape(out_len, d)[:k].contiguous()
    # every selected item is written; rows past the selection stay zero
    out = torch.empty((out_len, d), dtype=dtype, device=T.device())
    if k is not None and k < out_len:
        out[k:].zero_()
    if num_rows and num_items and d:
        nbytes = lib().bgl_softmax_workspace_size(num_rows, num_items, d, T.code_of(dtype))
        ws = T.workspace(nbytes)
        if edge_row is not None:
            rc = lib().bgl_edge_softmax_by_edge(T.ptr(indptr), T.ptr(eid), T.ptr(edge_row),
                                                num_rows, num_items, T.ptr(lt), T.ptr(out), d,
                                                T.code_of(dtype), T.ptr(ws), nbytes, T.stream())
        else:
            rc = lib().bgl_edge_softmax(T.ptr(indptr), T.ptr(eid), None, num_rows, num_items,
                                        T.ptr(lt), T.ptr(out), d, T.code_of(dtype), T.ptr(ws),
                                        nbytes, T.stream())
        check(rc, "edge_softmax")
    return T.result(out.reshape(shape), kind)
