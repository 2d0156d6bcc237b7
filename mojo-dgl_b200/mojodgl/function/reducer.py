"""Builtin reduce functions sum/max/min/mean (DGL's dgl/function/reducer.py)."""

from __future__ import annotations

import sys

from .base import BuiltinFunction

__all__ = []


class ReduceFunction(BuiltinFunction):
    """Base of the builtin reducers."""


class SimpleReduceFunction(ReduceFunction):
    """Reduce the message field ``msg_field`` into the node field ``out_field``."""

    def __init__(self, name, msg_field, out_field):
        self._name = name
        self.msg_field = msg_field
        self.out_field = out_field

    @property
    def name(self):
        return self._name


def _make(reducer):
    def func(msg, out):
        return SimpleReduceFunction(reducer, msg, out)

    func.__name__ = func.__qualname__ = reducer
    func.__doc__ = ("Builtin reducer: {0} of the incoming messages ``msg`` into node "
                    "field ``out`` (0 for nodes without in-edges).".format(reducer))
    return func


for _red in ("max", "min", "sum", "mean"):
    setattr(sys.modules[__name__], _red, _make(_red))
    __all__.append(_red)
