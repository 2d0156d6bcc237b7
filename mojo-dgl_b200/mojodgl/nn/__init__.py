"""Neural-network helpers (DGL's dgl.nn namespace)."""

from . import functional  # noqa: F401
