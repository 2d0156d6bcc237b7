"""Feature stores and the batch objects handed to user-defined functions.

Public surface as DGL's ``dgl/udf.py`` defines it, which the reference's
python/mojodgl/udf.py also follows: ``g.ndata`` / ``g.edata`` map a field name
to an array with one row per node / edge; a message UDF receives an
``EdgeBatch`` (``edges.src[f]``, ``edges.dst[f]``, ``edges.data[f]``) and a
reduce or apply UDF a ``NodeBatch`` (``nodes.mailbox[f]``, ``nodes.data[f]``,
``nodes[f]``).

Arrays keep the caller's kind: numpy arrays stay on the host and torch CUDA
tensors stay resident on the device, and float32 stays float32 (the reference
widens every stored field to float64, its udf.py:18-26).
"""

from __future__ import annotations

from collections.abc import MutableMapping

import numpy as np
import torch

from . import _tensor as T

__all__ = ["FeatureDict", "NodeBatch", "EdgeBatch"]


def take_rows(arr, ids):
    """``arr[ids]`` for numpy arrays and torch tensors, ids of either kind."""
    if T.is_torch(arr):
        idx = ids if T.is_torch(ids) else torch.from_numpy(np.asarray(ids, dtype=np.int64))
        return arr[idx.to(arr.device)]
    if T.is_torch(ids):
        ids = ids.cpu().numpy()
    return arr[ids]


class FeatureDict(MutableMapping):
    """Field name -> array whose leading axis has one row per node (``ndata``)
    or per edge (``edata``).  Assigning an array of another length raises
    ``ValueError``; reading a missing field raises ``KeyError`` naming it."""

    def __init__(self, store: dict, num_rows: int, what: str):
        # `store` is shared with the graph, which reads fields from it directly
        self._store, self._num_rows, self._what = store, num_rows, what

    def _noun(self):
        # "ndata" -> "node", "edata" -> "edge" (the message DGL users know)
        return {"ndata": "node", "edata": "edge"}.get(self._what, self._what)

    def __setitem__(self, key, value):
        arr = T.feature(value)
        shape = tuple(T.shape_of(arr))
        if not shape or shape[0] != self._num_rows:
            raise ValueError("{} expects {} rows, got shape {}".format(
                self._what, self._num_rows, shape))
        self._store[key] = arr

    def __getitem__(self, key):
        if key not in self._store:
            raise KeyError("cannot find {} feature {}".format(self._noun(), key))
        return self._store[key]

    def __delitem__(self, key):
        del self._store[key]

    def __iter__(self):
        return iter(self._store)

    def __len__(self):
        return len(self._store)

    def __contains__(self, key):
        return key in self._store

    def __repr__(self):
        return repr(self._store)


class _Rows:
    """Read-only field view that gathers the rows ``ids`` of every field it is
    asked for: ``edges.src`` / ``edges.dst`` over the node store (ids = the
    batch's endpoints), ``edges.data`` over the edge store (ids = edge ids)."""

    __slots__ = ("_fields", "_ids")

    def __init__(self, fields, ids):
        self._fields, self._ids = fields, ids

    def __getitem__(self, key):
        return take_rows(self._fields[key], self._ids)

    def __contains__(self, key):
        return key in self._fields


class NodeBatch:
    """What a reduce or apply UDF receives.  ``nodes[f]`` looks in the mailbox
    first, then in the node data."""

    def __init__(self, data=None, mailbox=None, num_nodes: int = 0, batch_num_nodes=None):
        # the mapping objects are kept, not copied: a UDF sees the live stores
        self.__fields = ({} if mailbox is None else mailbox, {} if data is None else data)
        self.__count = int(num_nodes)

    mailbox = property(lambda self: self.__fields[0], doc="messages reduced per node")
    data = property(lambda self: self.__fields[1], doc="the nodes' own fields")

    def __getitem__(self, key):
        for fields in self.__fields:
            if key in fields:
                return fields[key]
        raise KeyError(key)

    def num_nodes(self, ntype=None):
        return self.__count

    def batch_num_nodes(self, ntype=None):
        return [self.__count]

    def __repr__(self):
        keys = [k for fields in self.__fields for k in fields]
        return "NodeBatch(num_nodes={}, keys={})".format(self.__count, keys)


class EdgeBatch:
    """What a message UDF receives: the batch's edges ``eids`` with their
    source rows (``src``), destination rows (``dst``) and edge rows
    (``data``)."""

    def __init__(self, graph, eids):
        self._graph, self._eids = graph, eids
        u, v = graph._edge_arrays()
        self.src = _Rows(graph.ndata, take_rows(u, eids))
        self.dst = _Rows(graph.ndata, take_rows(v, eids))
        self.data = _Rows(graph.edata, eids)

    @property
    def number_of_nodes(self):
        return self._graph.number_of_nodes()

    @property
    def number_of_edges(self):
        return len(self._eids)

    def batch_num_nodes(self, ntype=None):
        return [self._graph.number_of_nodes()]

    def batch_num_edges(self, etype=None):
        return [len(self._eids)]

    def __repr__(self):
        return "EdgeBatch(num_edges={})".format(len(self._eids))
