"""Builtin message and reduce functions (DGL's dgl.function)."""

from .base import *  # noqa: F401,F403
from .message import *  # noqa: F401,F403
from .reducer import *  # noqa: F401,F403
