"""Graph construction (DGL's dgl.convert.graph; the reference's
python/mojodgl/convert.py:13-68)."""

from __future__ import annotations

import numpy as np

from . import _tensor as T
from .base import DGLError
from .heterograph import DGLGraph

__all__ = ["graph"]


def graph(data, *, num_nodes=None, idtype=None, device=None, row_sorted=False, col_sorted=False):
    """Create a graph from a ``(u, v)`` pair of node-id arrays (numpy, lists or
    torch tensors) or from a scipy sparse matrix (its nonzeros are the edges).

    ``idtype``, ``device``, ``row_sorted`` and ``col_sorted`` are accepted for
    signature compatibility: ids are int64 on the host and int32 in the
    device CSR, which is built on the current CUDA device on first use, and
    edges always keep the order they were given.
    """
    if hasattr(data, "tocoo"):
        coo = data.tocoo()
        u, v = coo.row, coo.col
        if num_nodes is None:
            num_nodes = max(data.shape)
    elif isinstance(data, tuple) and len(data) == 2:
        u, v = data
        for ids in (u, v):
            if T.is_torch(ids):
                if ids.is_floating_point() or ids.is_complex():
                    raise DGLError("node ids must be integers")
            elif not np.issubdtype(np.asarray(ids).dtype, np.integer):
                raise DGLError("node ids must be integers")
        u = u if T.is_torch(u) else np.asarray(u)
        v = v if T.is_torch(v) else np.asarray(v)
    else:
        raise DGLError("expect data to be a tuple of two node-id arrays or a scipy sparse matrix")
    return DGLGraph(u, v, num_nodes=num_nodes, idtype=idtype or np.int64)
