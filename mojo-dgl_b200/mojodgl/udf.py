"""Feature stores and the batches handed to user-defined functions.

Same names and behaviour as the reference's python/mojodgl/udf.py (itself
DGL's ``dgl/udf.py``): ``g.ndata``/``g.edata`` map a field name to a
row-per-node / row-per-edge array, and UDFs receive ``EdgeBatch`` /
``NodeBatch`` views.  Arrays keep the caller's kind: numpy stays on the host,
torch CUDA tensors stay resident on the device, and float32 stays float32
(the reference converts everything to float64 on assignment, udf.py:18-26).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _tensor as T

__all__ = ["FeatureDict", "NodeBatch", "EdgeBatch"]


def take_rows(arr, ids):
    """arr[ids] for numpy arrays and torch tensors alike."""
    if T.is_torch(arr):
        idx = ids if T.is_torch(ids) else torch.from_numpy(np.asarray(ids, dtype=np.int64))
        return arr[idx.to(arr.device)]
    if T.is_torch(ids):
        ids = ids.cpu().numpy()
    return arr[ids]


class FeatureDict:
    """``g.ndata`` / ``g.edata``: field name -> array with one row per node/edge."""

    def __init__(self, store: dict, num_rows: int, what: str):
        self._store = store
        self._num_rows = num_rows
        self._what = what

    def __setitem__(self, key, value):
        arr = T.feature(value)
        shape = T.shape_of(arr)
        if len(shape) == 0 or shape[0] != self._num_rows:
            raise ValueError("{} expects {} rows, got shape {}".format(
                self._what, self._num_rows, shape))
        self._store[key] = arr

    def __getitem__(self, key):
        try:
            return self._store[key]
        except KeyError:
            raise KeyError("cannot find {} feature {}".format(self._what[:-1], key))

    def __contains__(self, key):
        return key in self._store

    def __delitem__(self, key):
        del self._store[key]

    def __len__(self):
        return len(self._store)

    def __iter__(self):
        return iter(self._store)

    def keys(self):
        return self._store.keys()

    def items(self):
        return self._store.items()

    def pop(self, key, *default):
        return self._store.pop(key, *default)

    def __repr__(self):
        return repr(self._store)


class _EndpointView:
    """``edges.src`` / ``edges.dst``: node fields gathered at the batch's endpoints."""

    def __init__(self, graph, ids):
        self._graph = graph
        self._ids = ids

    def __getitem__(self, key):
        return take_rows(self._graph.ndata[key], self._ids)

    def __contains__(self, key):
        return key in self._graph.ndata


class _EdgeDataView:
    def __init__(self, graph, eids):
        self._graph = graph
        self._eids = eids

    def __getitem__(self, key):
        return take_rows(self._graph.edata[key], self._eids)

    def __contains__(self, key):
        return key in self._graph.edata


class NodeBatch:
    """The ``nodes`` argument of a reduce or apply UDF: ``data`` and ``mailbox``."""

    def __init__(self, data=None, mailbox=None, num_nodes: int = 0, batch_num_nodes=None):
        self._data = data if data is not None else {}
        self._mailbox = mailbox if mailbox is not None else {}
        self._num_nodes = num_nodes

    def __getitem__(self, key):
        if key in self._mailbox:
            return self._mailbox[key]
        return self._data[key]

    @property
    def mailbox(self):
        return self._mailbox

    @property
    def data(self):
        return self._data

    def batch_num_nodes(self, ntype=None):
        return [self._num_nodes]

    def num_nodes(self, ntype=None):
        return self._num_nodes

    def __repr__(self):
        return "NodeBatch(num_nodes={}, keys={})".format(
            self._num_nodes, list(self._mailbox) + list(self._data))


class EdgeBatch:
    """The ``edges`` argument of a message UDF: ``src``, ``dst`` and ``data``."""

    def __init__(self, graph, eids):
        self._graph = graph
        self._eids = eids
        u, v = graph._edge_arrays()
        self._src = _EndpointView(graph, take_rows(u, eids))
        self._dst = _EndpointView(graph, take_rows(v, eids))

    @property
    def src(self):
        return self._src

    @property
    def dst(self):
        return self._dst

    @property
    def data(self):
        return _EdgeDataView(self._graph, self._eids)

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
