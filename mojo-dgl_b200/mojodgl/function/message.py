"""Builtin message functions (DGL's dgl/function/message.py).

Each builtin is a description, not a computation: ``u_mul_e('h', 'e', 'm')``
records the op, the two operand targets and fields and the output field, and
``DGLGraph.update_all`` hands it to gspmm/gsddmm.  The 30 binary builtins
``{u,v,e}_{add,sub,mul,div,dot}_{u,v,e}`` are generated, as upstream does.
"""

from __future__ import annotations

import sys
from itertools import product

from .base import BuiltinFunction, TargetCode

__all__ = ["copy_u", "copy_e", "BinaryMessageFunction", "CopyMessageFunction"]


class MessageFunction(BuiltinFunction):
    """Base of the builtin message functions."""


class BinaryMessageFunction(MessageFunction):
    """``lhs_op_rhs``: op applied to a (lhs target, field) and a (rhs target, field)."""

    def __init__(self, binary_op, lhs, rhs, lhs_field, rhs_field, out_field):
        self.binary_op = binary_op
        self.lhs, self.rhs = lhs, rhs
        self.lhs_field, self.rhs_field = lhs_field, rhs_field
        self.out_field = out_field

    @property
    def name(self):
        return "{}_{}_{}".format(TargetCode.CODE2STR[self.lhs], self.binary_op,
                                 TargetCode.CODE2STR[self.rhs])


class CopyMessageFunction(MessageFunction):
    """``copy_u`` / ``copy_e``: one field taken as the message."""

    def __init__(self, target, in_field, out_field):
        self.target = target
        self.in_field = in_field
        self.out_field = out_field

    @property
    def name(self):
        return "copy_{}".format(TargetCode.CODE2STR[self.target])


def copy_u(u, out):
    """Message = the source node's field ``u``, written to ``out``."""
    return CopyMessageFunction(TargetCode.SRC, u, out)


def copy_e(e, out):
    """Message = the edge's field ``e``, written to ``out``."""
    return CopyMessageFunction(TargetCode.EDGE, e, out)


_CODE = {"u": TargetCode.SRC, "v": TargetCode.DST, "e": TargetCode.EDGE}
_WHAT = {"u": "source node", "v": "destination node", "e": "edge"}


def _make(lhs, rhs, op):
    def func(lhs_field, rhs_field, out):
        return BinaryMessageFunction(op, _CODE[lhs], _CODE[rhs], lhs_field, rhs_field, out)

    func.__name__ = "{}_{}_{}".format(lhs, op, rhs)
    func.__doc__ = (
        "Builtin message: {op} of the {l} field and the {r} field (NumPy "
        "broadcasting over feature axes), written to ``out``.".format(
            op=op, l=_WHAT[lhs], r=_WHAT[rhs]))
    return func


for _l, _r in product("uve", "uve"):
    if _l != _r:
        for _op in ("add", "sub", "mul", "div", "dot"):
            _f = _make(_l, _r, _op)
            setattr(sys.modules[__name__], _f.__name__, _f)
            __all__.append(_f.__name__)
