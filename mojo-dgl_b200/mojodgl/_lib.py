"""Loads libbgl.so (the sm_100a kernels) and declares its C ABI.

Replaces the reference's python/mojodgl/_lib.py (which loads the Mojo build,
``_lib.py:51-63,116-124``).  The op/reduce/target codes are the reference's
(``_lib.py:66-73``).  There is no CPU fallback: if the library or a CUDA
device is missing, every kernel call raises.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

from .base import DGLError

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.environ.get("BGL_LIB") or os.path.join(PKG_ROOT, "lib", "libbgl.so")

# src/ported.mojo:44-65 / python/mojodgl/_lib.py:66-73
SRC_CODE, DST_CODE, EDGE_CODE = 0, 1, 2
OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_DOT = 0, 1, 2, 3, 4
OP_COPY_LHS, OP_COPY_RHS = 5, 6
REDUCE_SUM, REDUCE_MAX, REDUCE_MIN, REDUCE_MEAN = 0, 1, 2, 3
BINARY_OPS = {"add": OP_ADD, "sub": OP_SUB, "mul": OP_MUL, "div": OP_DIV, "dot": OP_DOT}
REDUCERS = {"sum": REDUCE_SUM, "max": REDUCE_MAX, "min": REDUCE_MIN, "mean": REDUCE_MEAN}
TARGETS = {"u": SRC_CODE, "v": DST_CODE, "e": EDGE_CODE}

# include/bgl.h
BGL_F32, BGL_F64, BGL_BF16 = 0, 1, 2
BGL_ZERO_INF = 1
BGL_ACCUMULATE = 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_SZ = ctypes.c_size_t

# Native layer: name -> (argtypes, restype).
SIGNATURES = {
    "bgl_last_error": ([], ctypes.c_char_p),
    "bgl_abi_version": ([], _INT),
    "bgl_set_param": ([ctypes.c_char_p, _I64], _INT),
    "bgl_csr_build_workspace_size": ([_I64, _I64], _SZ),
    "bgl_csr_build": ([_P, _P, _I64, _I64, _P, _P, _P, _P, _P, _SZ, _P], _INT),
    "bgl_narrow_i64": ([_P, _P, _I64, _P], _INT),
    "bgl_check_csr": ([_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "bgl_ipc_export": ([_P, _I64, _P, _P], _INT),
    "bgl_ipc_open": ([_P, _I64, _I64, _P], _INT),
    "bgl_ipc_close": ([_P], _INT),
    "bgl_peer_copy": ([_P, _P, _I64, _P], _INT),
    "bgl_gspmm_workspace_size": ([_I64, _I64, _I64, _INT, _INT], _SZ),
    "bgl_gspmm": ([_P, _P, _P, _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _P, _P,
                   _INT, _INT, _INT, _INT, _P, _SZ, _P], _INT),
    "bgl_static_scratch_bytes": ([], _SZ),
    "bgl_gspmm_static_scratch": ([_P, _P, _P, _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _P,
                                  _I64, _P, _P, _INT, _INT, _INT, _INT, _P], _INT),
    "bgl_gsddmm": ([_P, _P, _I64, _P, _I64, _I64, _INT, _P, _I64, _I64, _INT, _P, _I64, _I64,
                    _INT, _INT, _P], _INT),
    "bgl_softmax_workspace_size": ([_I64, _I64, _I64, _INT], _SZ),
    "bgl_edge_softmax": ([_P, _P, _P, _I64, _I64, _P, _P, _I64, _INT, _P, _SZ, _P], _INT),
    "bgl_edge_softmax_by_edge": ([_P, _P, _P, _I64, _I64, _P, _P, _I64, _INT, _P, _SZ, _P], _INT),
    "bgl_gat_workspace_size": ([_I64, _I64, _I64, _I64, _INT], _SZ),
    "bgl_gat_aggregate": ([_P, _P, _I64, _I64, _P, _P, _P, _I64, _I64, ctypes.c_double, _P, _INT,
                           _P, _SZ, _P], _INT),
    "bgl_segment_mm_workspace_size": ([_I64, _I64, _I64, _I64, _INT], _SZ),
    "bgl_segment_mm": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _INT, _P, _SZ, _P], _INT),
    "bgl_gather_mm_workspace_size": ([_I64, _I64, _I64, _I64, _INT], _SZ),
    "bgl_gather_mm": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _INT, _P, _SZ, _P], _INT),
    "bgl_tc_error": ([], _INT),
    "bgl_cumsum_workspace_size": ([_I64], _SZ),
    "bgl_cumsum_i64": ([_P, _P, _I64, _P, _SZ, _P], _INT),
    "bgl_clamp_i64": ([_P, _P, _I64, _I64, _I64, _P], _INT),
    "bgl_replace_inf_with_zero": ([_P, _P, _I64, _INT, _P], _INT),
}

# Reference-compatible layer (src/capi.mojo:48-173): every argument int64.
COMPAT_SIGNATURES = {
    "mdgl_cumsum": ([_I64] * 3, None),
    "mdgl_replace_inf_with_zero": ([_I64] * 3, None),
    "mdgl_clamp_i64": ([_I64] * 5, None),
    "mdgl_gsddmm": ([_I64] * 12, None),
    "mdgl_gspmm": ([_I64] * 13, None),
    "mdgl_segment_reduce": ([_I64] * 7, None),
    "mdgl_segment_softmax": ([_I64] * 7, None),
    "mdgl_segment_mm": ([_I64] * 8, None),
    "mdgl_edge_softmax_": ([_I64] * 10, None),
    "mdgl_gather_mm": ([_I64] * 7, None),
    "mdgl_workers": ([], _I64),
}


class BuildError(RuntimeError):
    pass


def build(force: bool = False) -> str:
    """Compile libbgl.so in-tree with the package Makefile (nvcc, sm_100a)."""
    if force or not os.path.exists(LIB):
        proc = subprocess.run(["make", "-C", PKG_ROOT, "-j8"] + (["-B"] if force else []),
                              capture_output=True, text=True)
        if proc.returncode != 0 or not os.path.exists(LIB):
            raise BuildError((proc.stderr or proc.stdout).strip()[-4000:])
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise DGLError(
                "libbgl.so not found at {}; build it with `make -C {}`".format(LIB, PKG_ROOT))
        handle = ctypes.CDLL(LIB)
        for table in (SIGNATURES, COMPAT_SIGNATURES):
            for name, (argtypes, restype) in table.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = restype
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    """Raise DGLError carrying the library's message for a failed call."""
    if rc != 0:
        msg = lib().bgl_last_error()
        raise DGLError("{} failed (status {}): {}".format(
            what, rc, msg.decode() if msg else "unknown error"))


def set_param(name: str, value: int) -> None:
    check(lib().bgl_set_param(name.encode(), int(value)), "bgl_set_param")


def exported_symbols():
    """Every symbol include/bgl.h declares."""
    return list(SIGNATURES) + list(COMPAT_SIGNATURES)
