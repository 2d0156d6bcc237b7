"""Builtin function base and target codes (DGL's dgl/function/base.py).

The codes are the kernels' target codes (src/ported.mojo:45-47)."""

from __future__ import annotations

__all__ = ["BuiltinFunction", "TargetCode"]


class TargetCode:
    """Which endpoint an operand lives on: source node, destination node, edge."""

    SRC = 0
    DST = 1
    EDGE = 2
    CODE2STR = {0: "u", 1: "v", 2: "e"}


class BuiltinFunction:
    """A builtin message or reduce function: a plain description of the
    computation that update_all/pull dispatch to the fused kernels."""

    @property
    def name(self):
        raise NotImplementedError
