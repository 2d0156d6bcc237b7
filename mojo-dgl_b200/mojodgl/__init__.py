"""mojodgl on B200: DGL's message-passing API over hand-written sm_100a kernels.

The names are DGL's, as in the reference package (lee101/mojo-dgl):
``mojodgl.graph``, ``mojodgl.ops``, ``mojodgl.function``, ``g.update_all``.
The kernels live in ``libbgl.so`` (see ``include/bgl.h``); arrays go to the
current CUDA device, numpy in -> numpy out, torch in -> torch out.
"""

from . import function, nn, ops  # noqa: F401
from ._lib import build  # noqa: F401
from .base import ALL, EID, ETYPE, NID, NTYPE, DGLError  # noqa: F401
from .convert import graph  # noqa: F401
from .function import *  # noqa: F401,F403
from .heterograph import DGLGraph  # noqa: F401
from .ops import *  # noqa: F401,F403
from .udf import EdgeBatch, NodeBatch  # noqa: F401

__version__ = "0.1.0"

__all__ = [
    "DGLGraph", "graph", "DGLError", "ALL", "EID", "ETYPE", "NID", "NTYPE",
    "EdgeBatch", "NodeBatch", "build", "function", "ops", "nn",
] + ops.__all__
