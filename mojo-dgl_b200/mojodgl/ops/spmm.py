"""gSpMM: message computation fused with the reduction onto destinations.

Same public surface as the reference's python/mojodgl/ops/spmm.py (``gspmm``
and the 24 generated ``u_{add,sub,mul,div}_e_{sum,max,min,mean}``,
``copy_{u,e}_{sum,max,min,mean}``, registered by ``spmm.py:214-231``), computed
by ``bgl_gspmm`` on the device over the graph's cached in-CSR.

Rows with no in-edges keep the reduce identity (0, -inf, +inf), as the
reference's kernel returns them (src/ported.mojo:347-350); ``update_all``
replaces the infinities with zero.  ``_gspmm`` additionally returns DGL's
``(arg_u, arg_e)`` for max/min: the source node and edge id of the first
message in CSR (ascending edge id) order that attains the extreme.
"""

from __future__ import annotations

import sys

import torch

from .. import _tensor as T
from .._lib import (BGL_ZERO_INF, BINARY_OPS, OP_COPY_LHS, OP_COPY_RHS, REDUCERS, check, lib)
from ..base import DGLError
from .sddmm import Binary, check_rows, flat_feature, out_shape

__all__ = ["gspmm"]


def _run(g, op, reduce_op, lhs_data, rhs_data, with_arg=False, zero_inf=False, csr=None):
    if reduce_op not in REDUCERS:
        raise DGLError("reduce_op {} not recognized".format(reduce_op))
    if op not in list(BINARY_OPS) + ["copy_lhs", "copy_rhs"]:
        raise DGLError("op {} not recognized".format(op))
    if op == "dot":
        raise DGLError("dot is not a gspmm operator; use gsddmm")
    kind = T.kind_of(lhs_data, rhs_data)
    num_dst = g.number_of_nodes()
    num_edges = g.number_of_edges()
    lhs = None if lhs_data is None else T.feature(lhs_data)
    rhs = None if rhs_data is None else T.feature(rhs_data)
    dtype = T.common_float(lhs, rhs)
    if op == "copy_lhs":
        if lhs is None:
            raise DGLError("copy_lhs needs the node operand")
        check_rows(lhs, num_dst, "node")
        feat, dout = flat_feature(lhs)
        lt, lw, ldiv, rt, rw, rdiv, rank = T.to_dev(lhs, dtype), dout, 1, None, 1, 1, len(feat)
        code = OP_COPY_LHS
    elif op == "copy_rhs":
        if rhs is None:
            raise DGLError("copy_rhs needs the edge operand")
        check_rows(rhs, num_edges, "edge")
        feat, dout = flat_feature(rhs)
        lt, lw, ldiv, rt, rw, rdiv, rank = None, 1, 1, T.to_dev(rhs, dtype), dout, 1, len(feat)
        code = OP_COPY_RHS
    else:
        if lhs is None or rhs is None:
            raise DGLError("{} needs both operands".format(op))
        check_rows(lhs, num_dst, "node")
        check_rows(rhs, num_edges, "edge")
        b = Binary(lhs, rhs, dtype)
        feat, dout, rank = b.out_feat, b.dout, b.rank
        lt, lw, ldiv, rt, rw, rdiv = b.lhs, b.lw, b.ldiv, b.rhs, b.rw, b.rdiv
        code = BINARY_OPS[op]

    # the in-CSR holds every in-edge, so the mean divides by the row length,
    # which the kernel has in hand: no degree array is passed
    indptr, indices, eid, _ = csr if csr is not None else g._device().in_csr
    red = REDUCERS[reduce_op]
    flags = BGL_ZERO_INF if zero_inf else 0
    elem = torch.empty((), dtype=dtype).element_size()
    if (kind != T.TORCH_CUDA and not with_arg and csr is None
            and num_dst * dout * elem >= _OVERLAP_MIN_BYTES):
        out = _run_host_overlapped(g, lt, lw, ldiv, rt, rw, rdiv, dout, dtype, code, red, flags)
        shape = out_shape(num_dst, feat, rank)
        res = out.reshape(shape)
        return res.numpy() if kind == T.NUMPY else res
    dev = T.device()
    out = torch.empty((num_dst, dout), dtype=dtype, device=dev)
    arg_u = arg_e = None
    if with_arg and reduce_op in ("max", "min"):
        arg_u = torch.empty((num_dst, dout), dtype=torch.int64, device=dev) if code != OP_COPY_RHS else None
        arg_e = torch.empty((num_dst, dout), dtype=torch.int64, device=dev) if code != OP_COPY_LHS else None
    nbytes = lib().bgl_gspmm_workspace_size(num_dst, num_edges, dout, T.code_of(dtype), red)
    ws = T.workspace(nbytes)
    rc = lib().bgl_gspmm(T.ptr(indptr), T.ptr(indices), T.ptr(eid), None, num_dst, num_edges,
                         T.ptr(lt), lw, ldiv, T.ptr(rt), rw, rdiv, T.ptr(out), dout, T.ptr(arg_u),
                         T.ptr(arg_e), T.code_of(dtype), code, red, flags, T.ptr(ws), nbytes,
                         T.stream())
    check(rc, "gspmm")
    shape = out_shape(num_dst, feat, rank)
    res = T.result(out.reshape(shape), kind)
    if not with_arg:
        return res
    conv = lambda a: None if a is None else T.result(a.reshape(shape), kind)  # noqa: E731
    return res, (conv(arg_u), conv(arg_e))


# A host-bound result of at least this size is computed in destination-row
# slices, each slice's rows copied back while the next slice runs.
_OVERLAP_MIN_BYTES = 64 << 20
_OVERLAP_SLICES = 8
_copy_streams = {}


def _run_host_overlapped(g, lt, lw, ldiv, rt, rw, rdiv, dout, dtype, code, red, flags):
    """gSpMM over the graph's in-CSR in edge-balanced destination-row slices
    (every slice holds all in-edges of its rows, so its rows are final when
    its launch ends); the copy of slice k's rows into pinned host memory
    runs on a second stream while slice k + 1 is computed.  Returns the
    pinned host result."""
    dg = g._device()
    dev = T.device()
    num_dst = g.number_of_nodes()
    _, indices, eid, _ = dg.in_csr
    out = torch.empty((num_dst, dout), dtype=dtype, device=dev)
    host = torch.empty((num_dst, dout), dtype=dtype, pin_memory=True)
    slices = dg.in_row_slices(_OVERLAP_SLICES)
    dcode = T.code_of(dtype)
    nbytes = max(lib().bgl_gspmm_workspace_size(r1 - r0, e1 - e0, dout, dcode, red)
                 for r0, r1, e0, e1, _ in slices)
    ws = T.workspace(nbytes)
    compute = torch.cuda.current_stream()
    copier = _copy_streams.get(dev.index)
    if copier is None:
        copier = _copy_streams[dev.index] = torch.cuda.Stream(device=dev)
    row_bytes = dout * out.element_size()
    for r0, r1, e0, e1, ip in slices:
        rc = lib().bgl_gspmm(T.ptr(ip), T.ptr(indices) + 4 * e0, T.ptr(eid) + 4 * e0, None, r1 - r0,
                             e1 - e0, T.ptr(lt), lw, ldiv, T.ptr(rt), rw, rdiv,
                             T.ptr(out) + r0 * row_bytes, dout, None, None, dcode, code, red, flags,
                             T.ptr(ws), nbytes, compute.cuda_stream)
        check(rc, "gspmm")
        done = torch.cuda.Event()
        done.record(compute)
        copier.wait_event(done)
        with torch.cuda.stream(copier):
            host[r0:r1].copy_(out[r0:r1], non_blocking=True)
    copier.synchronize()  # every slice's kernel and copy are done
    return host


def gspmm(g, op, reduce_op, lhs_data, rhs_data):
    r"""Generalized sparse-dense matrix multiplication, message and reduce fused.

    .. math:: x_v = \psi_{(u, v, e) \in \mathcal{G}}(\rho(x_u, x_e))

    ``op`` is ``add``, ``sub``, ``mul``, ``div``, ``copy_lhs`` or ``copy_rhs``;
    ``reduce_op`` is ``sum``, ``max``, ``min`` or ``mean``.  ``lhs_data`` is
    the source-node operand, ``rhs_data`` the edge operand (either may be
    None when the op does not read it).
    """
    return _run(g, op, reduce_op, lhs_data, rhs_data)


def _gspmm(g, op, reduce_op, lhs_data, rhs_data):
    """gspmm plus DGL's ``(arg_u, arg_e)`` for max/min (None otherwise): the
    int64 source node / edge id of the first winning message per output
    element in CSR order, -1 for rows without in-edges."""
    return _run(g, op, reduce_op, lhs_data, rhs_data, with_arg=True)


def _make_spmm(binary_op, reduce_op):
    def func(g, x, y):
        return gspmm(g, binary_op, reduce_op, x, y)

    func.__name__ = "u_{}_e_{}".format(binary_op, reduce_op)
    func.__doc__ = (
        "Generalized SpMM: the message {op}(source feature x, edge feature y) "
        "reduced by {red} onto every destination node.\n\nOperands broadcast "
        "with NumPy semantics.  Nodes without in-edges get {ident}.".format(
            op=binary_op, red=reduce_op,
            ident={"max": "-inf", "min": "+inf"}.get(reduce_op, "0")))
    return func


def _make_copy(src, reduce_op):
    def func(g, x):
        if src == "copy_u":
            return gspmm(g, "copy_lhs", reduce_op, x, None)
        return gspmm(g, "copy_rhs", reduce_op, None, x)

    func.__name__ = "{}_{}".format(src, reduce_op)
    func.__doc__ = (
        "Generalized SpMM: the {what} feature x taken as the message and "
        "reduced by {red} onto every destination node.".format(
            what="source node" if src == "copy_u" else "edge", red=reduce_op))
    return func


for _op in ("add", "sub", "mul", "div", "copy_u", "copy_e"):
    for _red in ("sum", "max", "min", "mean"):
        _f = _make_copy(_op, _red) if _op.startswith("copy") else _make_spmm(_op, _red)
        setattr(sys.modules[__name__], _f.__name__, _f)
        __all__.append(_f.__name__)
