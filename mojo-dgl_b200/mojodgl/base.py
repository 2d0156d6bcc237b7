"""Shared API objects: the error type and the ALL sentinel.

Same public names and meaning as the reference's python/mojodgl/base.py:8-38
(which mirrors dgl/base.py), so callers catch and pass them unchanged.
"""

from __future__ import annotations

__all__ = ["ALL", "EID", "ETYPE", "NID", "NTYPE", "DGLError", "is_all"]


class DGLError(RuntimeError):
    """Raised for every rejected argument and every failed kernel call."""


class _All:
    """Singleton meaning "every node" / "every edge"; falsy like upstream's."""

    _one = None

    def __new__(cls):
        if cls._one is None:
            cls._one = super().__new__(cls)
        return cls._one

    def __repr__(self) -> str:
        return "ALL"

    def __bool__(self) -> bool:
        return False


ALL = _All()
EID = ETYPE = NID = NTYPE = ALL


def is_all(x) -> bool:
    return isinstance(x, _All)
