"""The C-ABI library loads and exports exactly what include/bgl.h declares.

CPU-only: symbols, signatures and argument validation that returns before any
CUDA call.  No kernel runs here.
"""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bgl.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:bgl|mdgl)_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from mojodgl import _lib

    return _lib.lib()


def test_header_declares_both_layers():
    names = header_functions()
    compat = [n for n in names if n.startswith("mdgl_")]
    # the reference's src/capi.mojo exports exactly these eleven
    assert compat == sorted([
        "mdgl_workers", "mdgl_cumsum", "mdgl_replace_inf_with_zero", "mdgl_clamp_i64",
        "mdgl_gsddmm", "mdgl_gspmm", "mdgl_segment_reduce", "mdgl_segment_softmax",
        "mdgl_segment_mm", "mdgl_edge_softmax_", "mdgl_gather_mm"])
    assert "bgl_gspmm" in names and "bgl_csr_build" in names


def test_library_exports_every_declared_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name


def test_python_signature_table_covers_the_header():
    from mojodgl import _lib

    assert sorted(_lib.exported_symbols()) == header_functions()


def test_compat_signatures_are_all_int64():
    from mojodgl import _lib

    arity = {"mdgl_cumsum": 3, "mdgl_replace_inf_with_zero": 3, "mdgl_clamp_i64": 5,
             "mdgl_gsddmm": 12, "mdgl_gspmm": 13, "mdgl_segment_reduce": 7,
             "mdgl_segment_softmax": 7, "mdgl_segment_mm": 8, "mdgl_edge_softmax_": 10,
             "mdgl_gather_mm": 7, "mdgl_workers": 0}  # python/mojodgl/_lib.py:51-63
    for name, (args, _) in _lib.COMPAT_SIGNATURES.items():
        assert len(args) == arity[name]
        assert all(a is ctypes.c_int64 for a in args)


def test_workers_and_version(lib):
    assert lib.mdgl_workers() == 32
    assert lib.bgl_abi_version() == 1


def test_set_param_validates(lib):
    assert lib.bgl_set_param(b"no_such_knob", 1) == 1
    assert b"unknown parameter" in lib.bgl_last_error()
    assert lib.bgl_set_param(b"spmm_min_items", 0) == 1
    assert lib.bgl_set_param(b"spmm_max_chunks", 0) == 0


def test_gspmm_rejects_bad_codes_before_any_device_call(lib):
    null = None
    args = dict(indptr=null, indices=null, eid=null, deg=null, n=4, e=4, lhs=null, lw=1, ld=1,
                rhs=null, rw=1, rd=1, out=null, dout=1, au=null, ae=null)

    def call(dtype, op, red):
        return lib.bgl_gspmm(*args.values(), dtype, op, red, 0, null, 0, null)

    assert call(0, 4, 0) == 1  # dot is not a gspmm op
    assert b"not a gspmm operator" in lib.bgl_last_error()
    assert call(0, 9, 0) == 1
    assert call(0, 0, 7) == 1
    assert call(5, 0, 0) == 3  # unsupported dtype
    assert call(0, 0, 0) == 1  # null buffers with rows and edges


def test_gsddmm_and_softmax_validation(lib):
    assert lib.bgl_gsddmm(None, None, 3, None, 1, 1, 7, None, 1, 1, 0, None, 1, 0, 0, 0, None) == 1
    assert lib.bgl_gsddmm(None, None, 3, None, 4, 1, 0, None, 4, 1, 1, None, 2, 4, 0, 4, None) == 1
    assert lib.bgl_edge_softmax(None, None, None, 2, 2, None, None, 1, 0, None, 0, None) == 1
    assert b"null buffer" in lib.bgl_last_error()
    assert lib.bgl_edge_softmax(None, None, None, 0, 0, None, None, 1, 0, None, 0, None) == 0
    assert lib.bgl_edge_softmax(None, None, None, 1, 1, None, None, 1, 9, None, 0, None) == 3


def test_grouped_mm_validation(lib):
    assert lib.bgl_segment_mm(None, None, None, None, -1, 1, 1, 1, 0, None, 0, None) == 1
    assert lib.bgl_gather_mm(None, None, None, None, 4, 2, 0, 2, 0, None, 0, None) == 1
    assert lib.bgl_segment_mm(None, None, None, None, 1, 1, 1, 1, 7, None, 0, None) == 3


def test_peer_buffer_validation(lib):
    inv = 1  # BGL_E_INVALID
    off = ctypes.c_int64(0)
    ptr = ctypes.c_void_p(0)
    handle = ctypes.create_string_buffer(64)
    assert lib.bgl_peer_copy(None, None, 16, None) == inv
    assert lib.bgl_ipc_export(None, 16, handle, ctypes.byref(off)) == inv
    assert lib.bgl_ipc_open(None, 0, 16, ctypes.byref(ptr)) == inv
    assert lib.bgl_ipc_open(handle, -1, 16, ctypes.byref(ptr)) == inv
    assert lib.bgl_ipc_close(None) == inv


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback_without_a_device():
    """Without a CUDA device every operator raises instead of computing on
    the host: the product path is the B200 library or nothing."""
    import numpy as np

    import mojodgl as dgl
    import mojodgl.ops as ops
    from mojodgl.base import DGLError

    g = dgl.graph((np.array([0, 1, 2]), np.array([1, 2, 0])))
    x = np.ones((3, 4))
    calls = [lambda: ops.copy_u_sum(g, x), lambda: ops.u_add_v(g, x, x),
             lambda: ops.edge_softmax(g, np.ones((3, 1))),
             lambda: ops.segment_reduce(np.array([1, 2]), x),
             lambda: ops.segment_mm(x, np.ones((2, 4, 2)), np.array([1, 2])),
             lambda: ops.gat_aggregate(g, np.ones((3, 2, 4)), np.ones((3, 2)), np.ones((3, 2)))]
    for call in calls:
        with pytest.raises(DGLError, match="CUDA device"):
            call()
