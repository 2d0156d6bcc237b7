"""TEST INFRASTRUCTURE -- the CPU oracle's Python half.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this module, as the checker and as the timed CPU baseline; the product
(``mojo-dgl_b200/``) never does.

It restates, in numpy, the host-side logic of the reference's Python package
(lee101/mojo-dgl ``python/mojodgl``), and runs the arithmetic through
``oracle/_build/libported_ref.so``, the C restatement of ``src/ported.mojo``
exported under the reference's own ``mdgl_*`` ABI.  Every function cites the
reference file:line it follows.  All arithmetic is float64, as the reference's
``f64()`` gate makes it (``python/mojodgl/_lib.py:127-163``): float32 inputs are
widened to float64 first, so the oracle of an fp32 GPU run is the fp64 result
on the *same* fp32 values.

Pinning: ``tests/test_oracle_pins.py`` checks this module against every
known-answer vector the reference's own tests and README hold, and against the
reference's Python package itself (run on the same C kernels) through the
fixtures in ``tests/golden/``.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ORACLE_LIB") or os.path.join(HERE, "_build", "libported_ref.so")

# python/mojodgl/_lib.py:66-73
SRC_CODE, DST_CODE, EDGE_CODE = 0, 1, 2
OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_DOT = 0, 1, 2, 3, 4
OP_COPY_LHS, OP_COPY_RHS = 5, 6
REDUCE_SUM, REDUCE_MAX, REDUCE_MIN, REDUCE_MEAN = 0, 1, 2, 3
BINARY_OPS = {"add": OP_ADD, "sub": OP_SUB, "mul": OP_MUL, "div": OP_DIV, "dot": OP_DOT}
REDUCERS = {"sum": REDUCE_SUM, "max": REDUCE_MAX, "min": REDUCE_MIN, "mean": REDUCE_MEAN}
TARGETS = {"u": SRC_CODE, "v": DST_CODE, "e": EDGE_CODE}

_I = ctypes.c_int64
_SIGS = {
    "mdgl_cumsum": 3, "mdgl_replace_inf_with_zero": 3, "mdgl_clamp_i64": 5,
    "mdgl_gsddmm": 12, "mdgl_gspmm": 13, "mdgl_segment_reduce": 7,
    "mdgl_segment_softmax": 7, "mdgl_segment_mm": 8, "mdgl_edge_softmax_": 10,
    "mdgl_gather_mm": 7, "oref_gspmm_arg": 15, "oref_csr_build": 8,
}
_lib = None


def build() -> str:
    """Compile the C restatement if its .so is missing or stale."""
    src = os.path.join(HERE, "ported_ref.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        import subprocess

        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        for name, n in _SIGS.items():
            fn = getattr(_lib, name)
            fn.argtypes = [_I] * n
            fn.restype = None
        _lib.mdgl_workers.argtypes = []
        _lib.mdgl_workers.restype = _I
        _lib.oref_threads.argtypes = []
        _lib.oref_threads.restype = _I
    return _lib


def _a(x):
    return x.ctypes.data


def f64(a):
    """python/mojodgl/_lib.py:127-163 (the lossless-conversion checks are the
    product's business; the oracle only widens)."""
    a = np.asarray(a)
    return np.ascontiguousarray(a, dtype=np.float64)


def i64(a):
    return np.ascontiguousarray(np.asarray(a), dtype=np.int64)


# --------------------------------------------------------------------- graph
class Graph:
    """The reference's DGLGraph CSR views (python/mojodgl/heterograph.py:69-95):
    in-degree by bincount, indptr by cumsum, the edge order by a *stable*
    argsort of the destination (source for the out-CSR), and the CSR's
    neighbour column gathered through that order."""

    def __init__(self, u, v, num_nodes=None):
        self.u = i64(u)
        self.v = i64(v)
        if num_nodes is None:
            num_nodes = 0 if self.u.size == 0 else int(max(self.u.max(), self.v.max())) + 1
        self.num_nodes = int(num_nodes)
        n = self.num_nodes
        self.indeg = np.bincount(self.v, minlength=n).astype(np.int64)
        self.outdeg = np.bincount(self.u, minlength=n).astype(np.int64)
        self.indptr = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(self.indeg, out=self.indptr[1:])
        self.outptr = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(self.outdeg, out=self.outptr[1:])
        self.in_order = np.argsort(self.v, kind="stable").astype(np.int64)
        self.out_order = np.argsort(self.u, kind="stable").astype(np.int64)
        self.in_indices = i64(self.u[self.in_order])
        self.out_indices = i64(self.v[self.out_order])

    @property
    def num_edges(self):
        return int(self.u.size)

    def in_csr(self):
        return self.indptr, self.in_indices, self.in_order

    def out_csr(self):
        return self.outptr, self.out_indices, self.out_order


def csr_arrays(key, other, num_nodes):
    """(indptr, deg, order, indices) of the CSR keyed by ``key``
    (heterograph.py:69-86) through the C counting sort: identical to the
    stable-argsort construction of Graph, in O(E) for full-size graphs."""
    key, other = i64(key), i64(other)
    n, e = int(num_nodes), int(key.size)
    indptr = np.empty(n + 1, dtype=np.int64)
    deg = np.empty(n, dtype=np.int64)
    order = np.empty(e, dtype=np.int64)
    indices = np.empty(e, dtype=np.int64)
    lib().oref_csr_build(_a(key), _a(other), e, n, _a(indptr), _a(deg), _a(order), _a(indices))
    return indptr, deg, order, indices


# ------------------------------------------------------ shape handling (sddmm)
def reshape_lhs_rhs(lhs, rhs):
    """python/mojodgl/ops/sddmm.py:24-47."""
    ls, rs = np.shape(lhs), np.shape(rhs)
    if len(ls) != len(rs):
        m = max(len(ls), len(rs))
        lhs = np.reshape(lhs, (ls[0],) + (1,) * (m - len(ls)) + ls[1:])
        rhs = np.reshape(rhs, (rs[0],) + (1,) * (m - len(rs)) + rs[1:])
    return lhs, rhs


def flat_bcast(lhs, rhs):
    """DGL's broadcast of the trailing feature axes, materialised.

    The reference's ``_flat``/``_broadcast`` (sddmm.py:50-68) only widen a
    ``(n, 1)`` column; for those shapes this is the same thing.  For the
    head-broadcast shapes the B200 build adds (``(N, H, D)`` against
    ``(E, H, 1)``) the oracle broadcasts with numpy and then flattens, which is
    what the reference computes once its inputs are given the broadcast shape.
    """
    lhs, rhs = reshape_lhs_rhs(f64(lhs), f64(rhs))
    out_feat = np.broadcast_shapes(lhs.shape[1:], rhs.shape[1:])
    lf = np.ascontiguousarray(np.broadcast_to(lhs, lhs.shape[:1] + out_feat))
    rf = np.ascontiguousarray(np.broadcast_to(rhs, rhs.shape[:1] + out_feat))
    d = int(np.prod(out_feat)) if out_feat else 1
    return lf.reshape(len(lf), d), rf.reshape(len(rf), d), out_feat


def _shape_out(out, n, feat):
    """The reference returns 2-D (n, d) results for its 1-D/2-D operands
    (spmm.py:102, sddmm.py:386); the head-broadcast superset keeps the
    broadcast feature shape."""
    if len(feat) <= 1:
        return out
    return out.reshape((n,) + tuple(feat))


def _flat2(a):
    a = f64(a)
    if a.ndim == 1:
        return a.reshape(-1, 1), 1
    return a.reshape(len(a), -1), int(np.prod(a.shape[1:]))


# --------------------------------------------------------------------- gspmm
def gspmm(g: Graph, op, reduce_op, lhs, rhs, with_arg=False):
    """python/mojodgl/ops/spmm.py:21-110 -> mdgl_gspmm (capi.mojo:95-115).

    Returns the (num_nodes, *feat) result; with ``with_arg`` also the
    (arg_u, arg_e) int64 arrays of the arg-index extension."""
    if op == "copy_lhs":
        l, dl = _flat2(lhs)
        r, dr = l, dl
        feat = f64(lhs).shape[1:]
    elif op == "copy_rhs":
        r, dr = _flat2(rhs)
        l, dl = r, dr
        feat = f64(rhs).shape[1:]
    else:
        l, r, feat = flat_bcast(lhs, rhs)
        dl = dr = l.shape[1]
    dout = max(dl, dr)
    n = g.num_nodes
    indptr, indices, eid = g.in_csr()
    out = np.empty((n, dout), dtype=np.float64)
    code = {"copy_lhs": OP_COPY_LHS, "copy_rhs": OP_COPY_RHS}.get(op, BINARY_OPS.get(op))
    la = _a(l) if l.size else _a(r)
    ra = _a(r) if r.size else _a(l)
    deg = i64(g.indeg)
    if with_arg:
        au = np.empty((n, dout), dtype=np.int64)
        ae = np.empty((n, dout), dtype=np.int64)
        lib().oref_gspmm_arg(_a(indptr), _a(indices), _a(eid), la, ra, _a(out), n, code, dl, dr,
                             dout, REDUCERS[reduce_op], _a(deg), _a(au), _a(ae))
        return _shape_out(out, n, feat), _shape_out(au, n, feat), _shape_out(ae, n, feat)
    lib().mdgl_gspmm(_a(indptr), _a(indices), _a(eid), la, ra, _a(out), n, code, dl, dr, dout,
                     REDUCERS[reduce_op], _a(deg))
    return _shape_out(out, n, feat)


def gspmm_abs_bound(g: Graph, op, lhs, rhs):
    """S = sum over each row's in-edges of |message| (an upper bound for
    add/sub), the scale the fp32 tolerance is taken relative to."""
    if op in ("copy_lhs", "copy_rhs"):
        return gspmm(g, op, "sum", None if lhs is None else np.abs(f64(lhs)),
                     None if rhs is None else np.abs(f64(rhs)))
    bop = {"add": "add", "sub": "add", "mul": "mul", "div": "div"}[op]
    return gspmm(g, bop, "sum", np.abs(f64(lhs)), np.abs(f64(rhs)))


def replace_inf_with_zero(x):
    """python/mojodgl/ops/segment.py:55-59 -> ported.mojo:157-177."""
    x = f64(x)
    out = np.zeros(x.shape, dtype=np.float64)
    lib().mdgl_replace_inf_with_zero(_a(x), _a(out), x.size)
    return out


# --------------------------------------------------------------------- sddmm
def gsddmm(g: Graph, op, lhs, rhs, lhs_target="u", rhs_target="v"):
    """python/mojodgl/ops/sddmm.py:83-170 -> mdgl_gsddmm (capi.mojo:70-91)."""
    uids, vids = g.u, g.v
    ne = g.num_edges
    if op == "copy_lhs":
        l, dl = _flat2(lhs)
        r, dr, dout = l, dl, dl
        feat = f64(lhs).shape[1:]
    elif op == "copy_rhs":
        r, dr = _flat2(rhs)
        l, dl, dout = r, dr, dr
        feat = f64(rhs).shape[1:]
    elif op == "dot":
        l, dl = _flat2(lhs)
        r, dr = _flat2(rhs)
        dout = 1
        feat = (1,) if f64(lhs).ndim > 1 else ()
    else:
        l, r, feat = flat_bcast(lhs, rhs)
        dl = dr = dout = l.shape[1]
    out = np.empty((ne, dout), dtype=np.float64)
    code = {"copy_lhs": OP_COPY_LHS, "copy_rhs": OP_COPY_RHS}.get(op, BINARY_OPS.get(op))
    la = _a(l) if l.size else _a(r)
    ra = _a(r) if r.size else _a(l)
    lib().mdgl_gsddmm(_a(uids), _a(vids), la, ra, _a(out), ne, TARGETS[lhs_target],
                      TARGETS[rhs_target], code, dl, dr, dout)
    return _shape_out(out, ne, feat) if op != "dot" else out


# -------------------------------------------------------------- segment ops
def offsets_of(seglen):
    """python/mojodgl/ops/segment.py:12-21."""
    seglen = i64(seglen)
    src = np.concatenate([np.zeros(1, dtype=np.int64), seglen])
    dst = np.zeros(src.shape, dtype=np.int64)
    lib().mdgl_cumsum(_a(src), _a(dst), src.size)
    return dst


def segment_reduce(seglen, value, reducer="sum"):
    """python/mojodgl/ops/segment.py:41-112."""
    seglen = i64(seglen)
    offsets = offsets_of(seglen)
    value = f64(value)
    shape = value.shape
    v2, d = _flat2(value)

    def core(red):
        ns = offsets.size - 1
        dst = np.empty((ns, d), dtype=np.float64)
        if ns == 0 or v2.size == 0:
            return dst
        lib().mdgl_segment_reduce(_a(offsets), _a(v2), _a(dst), ns, d, REDUCERS[red], len(v2))
        return dst

    if reducer == "mean":
        rst = core("sum")
        z = np.clip(seglen, 1, len(value)).astype(np.float64)
        rst = rst / z.reshape(-1, 1)
    else:
        rst = core(reducer)
        if reducer in ("min", "max"):
            rst = replace_inf_with_zero(rst)
    return _shape_out(rst, len(seglen), shape[1:])


def segment_softmax(seglen, value):
    """python/mojodgl/ops/segment.py:115-154."""
    seglen = i64(seglen)
    value = f64(value)
    shape = value.shape
    v2, d = _flat2(value)
    n = len(v2)
    offsets = offsets_of(seglen)
    dst = np.zeros(v2.shape, dtype=np.float64)
    if seglen.size == 0 or n == 0:
        return dst.reshape(shape)
    scratch = np.empty(lib().mdgl_workers() * 2 * d, dtype=np.float64)
    lib().mdgl_segment_softmax(_a(offsets), _a(v2), _a(dst), _a(scratch), seglen.size, d, n)
    return dst.reshape(shape)


def segment_mm(a, b, seglen_a):
    """python/mojodgl/ops/segment.py:157-214 (rows past sum(seglen) stay 0)."""
    a, b, seglen_a = f64(a), f64(b), i64(seglen_a)
    n, d1 = a.shape
    r, _, d2 = b.shape
    dst = np.zeros((n, d2), dtype=np.float64)
    if n == 0:
        return dst
    lib().mdgl_segment_mm(_a(a), _a(b), _a(dst), _a(seglen_a), n, d1, r, d2)
    return dst


def gather_mm(a, b, idx_b, segment_block=16384):
    """python/mojodgl/ops/gather_mm.py:21-92, both routes (:79-91)."""
    a, b, idx_b = f64(a), f64(b), i64(idx_b)
    n, d1 = a.shape
    r, _, d2 = b.shape
    if d1 * d2 > segment_block:
        perm = np.argsort(idx_b, kind="stable")
        rev = np.argsort(perm, kind="stable")
        pos_l = np.searchsorted(np.sort(idx_b), np.arange(r))
        pos_r = np.append(pos_l[1:], len(idx_b))
        return segment_mm(a[perm], b, pos_r - pos_l)[rev]
    dst = np.empty((n, d2), dtype=np.float64)
    if n == 0:
        return dst
    lib().mdgl_gather_mm(_a(a), _a(b), _a(idx_b), _a(dst), n, d1, d2)
    return dst


# -------------------------------------------------------------- edge_softmax
def selection_csr(g: Graph, eids, norm_by):
    """The positional-``eids`` CSR of python/mojodgl/ops/edge_softmax.py:119-158:
    the selection's POSITIONS grouped by endpoint (ascending node id), kept in
    the order they appear in ``eids``; row i reads ``logits[i]``.  A stable
    argsort of the endpoint key gives exactly that grouping."""
    order = i64(eids)
    key = (g.v if norm_by == "dst" else g.u)[order]
    pos = np.argsort(key, kind="stable").astype(np.int64)
    nodes, counts = np.unique(key[pos], return_counts=True)
    row_ptr = np.zeros(len(nodes) + 1, dtype=np.int64)
    np.cumsum(counts, out=row_ptr[1:])
    return row_ptr, pos


def edge_softmax(g: Graph, logits, eids=None, norm_by="dst"):
    """python/mojodgl/ops/edge_softmax.py:11-173 -> mdgl_edge_softmax_."""
    logits = f64(logits)
    shape = logits.shape
    d = 1 if len(shape) == 1 else int(np.prod(shape[1:]))
    lg = logits.reshape(shape[0], d)
    if eids is None:
        indptr, indices, eid = g.in_csr() if norm_by == "dst" else g.out_csr()
        num_rows = g.num_nodes
        row_ptr, row_ids = indptr, eid
    else:
        row_ptr, row_ids = selection_csr(g, eids, norm_by)
        num_rows = len(row_ptr) - 1
        lg = np.ascontiguousarray(lg[: len(i64(eids))])
    dst = np.zeros((g.num_edges, d), dtype=np.float64)
    mask = np.ones(1, dtype=np.int8)
    scratch = np.empty(lib().mdgl_workers() * 2 * d, dtype=np.float64)
    lib().mdgl_edge_softmax_(_a(row_ptr), _a(row_ids), _a(row_ids), _a(mask), _a(lg), _a(dst),
                             _a(scratch), num_rows, 1, d)
    if eids is not None:
        picked = np.zeros((shape[0], d), dtype=np.float64)
        k = len(i64(eids))
        picked[:k] = dst[:k]
        dst = picked
    return dst.reshape(shape)


# ----------------------------------------------------------- message passing
def update_all(g: Graph, ndata: dict, edata: dict, msg, red):
    """python/mojodgl/heterograph.py:206-290 for builtin message and reduce
    functions.  ``msg`` is ("copy_u", field) / ("copy_e", field) /
    (lhs_target, op, rhs_target, lhs_field, rhs_field); ``red`` is the reducer
    name.  Returns the reduced (and inf->0 for max/min) node feature."""
    if msg[0] == "copy_u":
        out = gspmm(g, "copy_lhs", red, ndata[msg[1]], None)
    elif msg[0] == "copy_e":
        out = gspmm(g, "copy_rhs", red, None, edata[msg[1]])
    else:
        lt, op, rt, lf, rf = msg
        ld = edata[lf] if lt == "e" else ndata[lf]
        rd = edata[rf] if rt == "e" else ndata[rf]
        if op != "dot" and lt == "u" and rt == "e":
            out = gspmm(g, op, red, ld, rd)
        else:
            m = gsddmm(g, op, ld, rd, lhs_target=lt, rhs_target=rt)
            out = gspmm(g, "copy_rhs", red, None, m)
    if red in ("max", "min"):
        out = replace_inf_with_zero(out)
    return out


def gat_aggregate(g: Graph, feat, el, er, negative_slope=0.2):
    """The chain a GAT layer runs on the reference's operators: u_add_v
    (ops/sddmm.py:83-170), leaky_relu (the caller's), edge_softmax norm_by dst
    (ops/edge_softmax.py:11-173), u_mul_e_sum (ops/spmm.py:21-110)."""
    n, h = feat.shape[0], feat.shape[1]
    el3 = f64(el).reshape(n, h, 1)
    er3 = f64(er).reshape(n, h, 1)
    s = gsddmm(g, "add", el3, er3, "u", "v")
    s = np.where(s > 0, s, negative_slope * s)
    a = edge_softmax(g, s)
    return gspmm(g, "mul", "sum", f64(feat), a)
