"""DGLGraph: a homogeneous graph with device-resident CSR views, and the
message-passing driver (update_all / pull).

Same public surface and semantics as the reference's
python/mojodgl/heterograph.py (itself DGL's homogeneous DGLGraph):

* edges keep the order they were given (heterograph.py:25-66);
* the in-CSR (destination-major, for aggregation and norm_by="dst") and the
  out-CSR (source-major, for norm_by="src") are built by a *stable* sort of the
  edge ids by endpoint (heterograph.py:69-86) -- here once per device by
  ``bgl_csr_build`` and cached, instead of by numpy on every construction;
* ``update_all`` fuses copy_u / copy_e / u_{add,sub,mul,div}_e with a builtin
  reducer into one gSpMM and runs everything else as gSDDMM followed by a
  copy_rhs gSpMM (heterograph.py:206-290); max/min then map +-inf to 0 --
  fused into the gSpMM epilogue here;
* ``pull`` reduces over the in-edges of the requested nodes only and writes
  only their rows (heterograph.py:318-347).
"""

from __future__ import annotations

from collections import namedtuple

import numpy as np
import torch

from . import _tensor as T
from ._lib import check, lib
from .base import DGLError, is_all
from .function.base import TargetCode
from .function.message import BinaryMessageFunction, CopyMessageFunction, MessageFunction
from .function.reducer import ReduceFunction
from .ops import spmm as _spmm
from .ops.sddmm import gsddmm
from .udf import EdgeBatch, FeatureDict, NodeBatch, take_rows

__all__ = ["DGLGraph"]

_EdgeTuple = namedtuple("EdgeTuple", "u v eid")
_Code2Str = TargetCode.CODE2STR


class _DeviceGraph:
    """The graph's arrays on one CUDA device.

    ``in_csr``/``out_csr`` = (indptr int64 [n+1], neighbour int32 [E],
    edge id int32 [E], degree int64 [n]); u64/v64 the endpoint arrays, u32/v32
    their int32 copies for gSDDMM."""

    def __init__(self, u, v, num_nodes):
        n, ne = num_nodes, int(u.numel())
        if n >= 2 ** 31 or ne >= 2 ** 31:
            raise DGLError("the device kernels index with int32: at most 2^31-1 nodes and edges")
        dev = u.device
        self.u64, self.v64 = u, v
        self.u32 = torch.empty(ne, dtype=torch.int32, device=dev)
        self.v32 = torch.empty(ne, dtype=torch.int32, device=dev)
        s = T.stream()
        check(lib().bgl_narrow_i64(T.ptr(u), T.ptr(self.u32), ne, s), "bgl_narrow_i64")
        check(lib().bgl_narrow_i64(T.ptr(v), T.ptr(self.v32), ne, s), "bgl_narrow_i64")
        self.in_csr = self._csr(v, u, ne, n, dev)
        self.out_csr = self._csr(u, v, ne, n, dev)

    def in_row_slices(self, parts):
        """The in-CSR cut into about `parts` destination-row slices holding
        equal numbers of edges, for aggregations that copy each slice's rows
        to the host while the next slice is computed: [(r0, r1, e0, e1,
        indptr)] with indptr rebased to the slice's first edge.  Built once
        per part count."""
        cache = self.__dict__.setdefault("_row_slices", {})
        if parts not in cache:
            indptr = self.in_csr[0]
            n = indptr.numel() - 1
            ne = int(indptr[-1])
            targets = torch.arange(1, parts, device=indptr.device, dtype=torch.int64) * ne // parts
            cuts = torch.searchsorted(indptr, targets).clamp_(0, n).cpu().tolist()
            bounds = sorted(set([0, n] + cuts))
            ends = indptr[torch.tensor(bounds, device=indptr.device)].cpu().tolist()
            slices = []
            for k in range(len(bounds) - 1):
                r0, r1 = bounds[k], bounds[k + 1]
                if r1 > r0:
                    slices.append((r0, r1, ends[k], ends[k + 1], (indptr[r0:r1 + 1] - ends[k]).contiguous()))
            cache[parts] = slices
        return cache[parts]

    @staticmethod
    def _csr(key, other, ne, n, dev):
        indptr = torch.empty(n + 1, dtype=torch.int64, device=dev)
        deg = torch.empty(n, dtype=torch.int64, device=dev)
        order = torch.empty(ne, dtype=torch.int32, device=dev)
        nbr = torch.empty(ne, dtype=torch.int32, device=dev)
        nbytes = lib().bgl_csr_build_workspace_size(ne, n)
        ws = T.workspace(nbytes)
        check(lib().bgl_csr_build(T.ptr(key), T.ptr(other), ne, n, T.ptr(indptr), T.ptr(deg),
                                  T.ptr(order), T.ptr(nbr), T.ptr(ws), nbytes, T.stream()),
              "bgl_csr_build")
        return indptr, nbr, order, deg


class DGLGraph:
    """A homogeneous graph; edges are stored in the order they were supplied."""

    def __init__(self, u, v, num_nodes=None, idtype=np.int64):
        u = T.ids(u)
        v = T.ids(v)
        if T.is_torch(u) != T.is_torch(v):
            u = u if T.is_torch(u) else torch.from_numpy(u).to(v.device)
            v = v if T.is_torch(v) else torch.from_numpy(v).to(u.device)
        if tuple(u.shape) != tuple(v.shape):
            raise DGLError("u and v must have the same length")
        u, v = u.reshape(-1), v.reshape(-1)
        ne = int(u.shape[0])
        if num_nodes is None:
            num_nodes = 0 if ne == 0 else int(max(u.max(), v.max())) + 1
        num_nodes = int(num_nodes)
        if num_nodes < 0:
            raise DGLError("num_nodes must be non-negative, got {}".format(num_nodes))
        if ne:
            lo, hi = int(min(u.min(), v.min())), int(max(u.max(), v.max()))
            if lo < 0 or hi >= num_nodes:
                raise DGLError("node ids must be in [0, {}), got [{}, {}]".format(num_nodes, lo, hi))
        self._u, self._v = u, v
        self._num_nodes = num_nodes
        self.idtype = idtype
        self._nstore = {}
        self._estore = {}
        self.ndata = FeatureDict(self._nstore, num_nodes, "ndata")
        self.edata = FeatureDict(self._estore, ne, "edata")
        self._dev_cache = {}
        self._host_cache = {}

    # --------------------------------------------------------- device views
    def _device(self) -> _DeviceGraph:
        dev = T.device()
        dg = self._dev_cache.get(dev.index)
        if dg is None:
            dg = _DeviceGraph(T.to_dev(self._u), T.to_dev(self._v), self._num_nodes)
            self._dev_cache[dev.index] = dg
        return dg

    def _host(self, name):
        """Host (numpy int64) copies of the device CSR, for the query API."""
        if name not in self._host_cache:
            dg = self._device()
            ip, nbr, order, deg = dg.in_csr if name == "in" else dg.out_csr
            self._host_cache[name] = tuple(
                t.to(torch.int64).cpu().numpy() for t in (ip, nbr, order, deg))
        return self._host_cache[name]

    def _as_kind(self, arr):
        """Return a host int64 array in the kind the graph was built from."""
        if T.is_torch(self._u):
            return torch.from_numpy(arr).to(self._u.device)
        return arr

    def _edge_arrays(self):
        return self._u, self._v

    def _in_csr(self):
        ip, nbr, order, _ = self._host("in")
        return ip, nbr, order

    def _out_csr(self):
        ip, nbr, order, _ = self._host("out")
        return ip, nbr, order

    # -------------------------------------------------------------- queries
    def number_of_nodes(self, ntype=None):
        return self._num_nodes

    def number_of_src_nodes(self, ntype=None):
        return self._num_nodes

    def number_of_dst_nodes(self, ntype=None):
        return self._num_nodes

    def number_of_edges(self, etype=None):
        return int(self._u.shape[0])

    def num_nodes(self, ntype=None):
        return self._num_nodes

    def num_edges(self, etype=None):
        return int(self._u.shape[0])

    def num_src_nodes(self, ntype=None):
        return self._num_nodes

    def num_dst_nodes(self, ntype=None):
        return self._num_nodes

    @property
    def canonical_etypes(self):
        return (("_N", "_E", "_N"),)

    def __len__(self):
        return self._num_nodes

    def __repr__(self):
        return "Graph(num_nodes={}, num_edges={},)".format(self._num_nodes, self.num_edges())

    __str__ = __repr__

    def edges(self, form="uv", order="eid", etype=None):
        """All edges as (u, v, eid) in edge-id order."""
        if form not in ("uv", "all"):
            raise DGLError("form must be 'uv' or 'all'")
        if order != "eid":
            raise DGLError("only order='eid' is supported")
        if T.is_torch(self._u):
            eid = torch.arange(self.num_edges(), dtype=torch.int64, device=self._u.device)
        else:
            eid = np.arange(self.num_edges(), dtype=np.int64)
        return _EdgeTuple(self._u, self._v, eid)

    def _select(self, ids, order, on_src):
        u = self._u.cpu().numpy() if T.is_torch(self._u) else self._u
        v = self._v.cpu().numpy() if T.is_torch(self._v) else self._v
        if is_all(ids):
            sel = np.arange(u.size)
        else:
            want = T.ids(ids)
            want = want.cpu().numpy() if T.is_torch(want) else want
            sel = np.nonzero(np.isin(u if on_src else v, want))[0]
        if order == "srcid":
            sel = sel[np.argsort(u[sel], kind="stable")]
        elif order == "dstid":
            sel = sel[np.argsort(v[sel], kind="stable")]
        sel = sel.astype(np.int64)
        return _EdgeTuple(self._as_kind(u[sel]), self._as_kind(v[sel]), self._as_kind(sel))

    def in_edges(self, v, form="uv", order="eid", etype=None):
        """In-edges of ``v`` (every node when ``v`` is ALL), in edge-id order."""
        return self._select(v, order, False)

    def out_edges(self, u, form="uv", order="eid", etype=None):
        """Out-edges of ``u`` (every node when ``u`` is ALL), in edge-id order."""
        return self._select(u, order, True)

    def in_degrees(self, v=None):
        deg = self._as_kind(self._host("in")[3])
        return deg if v is None else take_rows(deg, T.ids(v))

    def out_degrees(self, u=None):
        deg = self._as_kind(self._host("out")[3])
        return deg if u is None else take_rows(deg, T.ids(u))

    # ------------------------------------------------------ message passing
    def _builtin_message(self, mfunc):
        """Per-edge messages of a builtin message function."""
        if isinstance(mfunc, CopyMessageFunction):
            target = _Code2Str[mfunc.target]
            if target == "e":
                return T.feature(self.edata[mfunc.in_field])
            return gsddmm(self, "copy_lhs" if target == "u" else "copy_rhs",
                          self.ndata[mfunc.in_field], None, lhs_target=target)
        if not isinstance(mfunc, BinaryMessageFunction):
            raise DGLError("unrecognised message function {}".format(mfunc))
        lhs, rhs = _Code2Str[mfunc.lhs], _Code2Str[mfunc.rhs]
        ld = self.edata[mfunc.lhs_field] if lhs == "e" else self.ndata[mfunc.lhs_field]
        rd = self.edata[mfunc.rhs_field] if rhs == "e" else self.ndata[mfunc.rhs_field]
        return gsddmm(self, mfunc.binary_op, ld, rd, lhs_target=lhs, rhs_target=rhs)

    @staticmethod
    def _fusable(mfunc):
        """(op, lhs_field, rhs_field) when one gSpMM computes message + reduce."""
        if isinstance(mfunc, CopyMessageFunction):
            target = _Code2Str[mfunc.target]
            if target == "u":
                return "copy_lhs", mfunc.in_field, None
            if target == "e":
                return "copy_rhs", None, mfunc.in_field
            return None
        if not isinstance(mfunc, BinaryMessageFunction) or mfunc.binary_op == "dot":
            return None
        if _Code2Str[mfunc.lhs] != "u" or _Code2Str[mfunc.rhs] != "e":
            return None
        return mfunc.binary_op, mfunc.lhs_field, mfunc.rhs_field

    def _reduce(self, op, reducer, lhs, rhs):
        # max/min: nodes without in-edges come out as the identity and are
        # mapped to 0, with every other +-inf, exactly as the reference's
        # _reduce_result does with replace_inf_with_zero -- fused here.
        return _spmm._run(self, op, reducer, lhs, rhs, zero_inf=reducer in ("max", "min"))

    def _pass(self, message_func, reduce_func, apply_node_func, write=True):
        """One message-passing round; returns the new node features."""
        fused = self._fusable(message_func) if isinstance(message_func, MessageFunction) else None
        if fused is not None and isinstance(reduce_func, ReduceFunction):
            op, lf, rf = fused
            lhs = self.ndata[lf] if lf is not None else None
            rhs = self.edata[rf] if rf is not None else None
            result = {reduce_func.out_field: self._reduce(op, reduce_func.name, lhs, rhs)}
        else:
            if isinstance(message_func, MessageFunction):
                messages = {message_func.out_field: self._builtin_message(message_func)}
            else:
                eids = np.arange(self.num_edges(), dtype=np.int64)
                messages = dict(message_func(EdgeBatch(self, self._as_kind(eids))))
            if isinstance(reduce_func, ReduceFunction):
                msg = messages[next(iter(messages))]
                result = {reduce_func.out_field: self._reduce("copy_rhs", reduce_func.name, None, msg)}
            else:
                # documented divergence kept from the reference: the mailbox
                # holds the (N, D) sum over in-edges, not a ragged mailbox
                mailbox = {k: self._reduce("copy_rhs", "sum", None, m) for k, m in messages.items()}
                result = dict(reduce_func(NodeBatch(data=self._nstore, mailbox=mailbox,
                                                    num_nodes=self._num_nodes)))
        if apply_node_func is not None:
            result = dict(apply_node_func(NodeBatch(data=result, mailbox=None,
                                                    num_nodes=self._num_nodes)))
        result = {k: T.feature(v) for k, v in result.items()}
        if write:
            for key, value in result.items():
                self.ndata[key] = value
        return result

    def update_all(self, message_func, reduce_func, apply_node_func=None, etype=None):
        """Send messages along every edge and reduce them on every node.

        Nodes without in-edges receive 0 from every builtin reducer;
        ``apply_node_func`` still runs on them."""
        if etype is not None and etype not in self.canonical_etypes:
            raise DGLError("etype {} not in {}".format(etype, self.canonical_etypes))
        self._pass(message_func, reduce_func, apply_node_func)

    def pull(self, v, message_func, reduce_func, apply_node_func=None, etype=None):
        """Reduce the in-edge messages of the nodes ``v`` only; only their
        rows of the output fields are written (every other row is 0)."""
        if etype is not None and etype not in self.canonical_etypes:
            raise DGLError("etype {} not in {}".format(etype, self.canonical_etypes))
        want = T.ids(v)
        want = want.cpu().numpy() if T.is_torch(want) else want
        want = np.unique(want)
        if want.size == 0:
            return
        vv = self._v.cpu().numpy() if T.is_torch(self._v) else self._v
        mask = np.isin(vv, want)
        sel = np.nonzero(mask)[0]
        sub = DGLGraph(take_rows(self._u, sel), take_rows(self._v, sel), num_nodes=self._num_nodes)
        for key, value in self._nstore.items():
            sub.ndata[key] = value
        for key, value in self._estore.items():
            sub.edata[key] = take_rows(value, sel)
        result = sub._pass(message_func, reduce_func, apply_node_func, write=False)
        for key, value in result.items():
            if T.is_torch(value):
                rows = torch.zeros_like(value)
                idx = torch.from_numpy(want).to(value.device)
                rows[idx] = value[idx]
            else:
                rows = np.zeros_like(value)
                rows[want] = value[want]
            self.ndata[key] = rows
