"""The operator API (the reference's python/mojodgl/ops, DGL's dgl.ops).

The star imports shadow the ``edge_softmax`` and ``gather_mm`` submodule names
with the same-named functions, as the reference and upstream do.
"""

from . import edge_softmax as _es_mod
from . import gat as _gat_mod
from . import gather_mm as _gm_mod
from . import sddmm as _sddmm_mod
from . import segment as _seg_mod
from . import spmm as _spmm_mod
from .edge_softmax import *  # noqa: F401,F403
from .gat import *  # noqa: F401,F403
from .gather_mm import *  # noqa: F401,F403
from .sddmm import *  # noqa: F401,F403
from .segment import *  # noqa: F401,F403
from .spmm import *  # noqa: F401,F403

__all__ = (_es_mod.__all__ + _gm_mod.__all__ + _sddmm_mod.__all__ + _seg_mod.__all__
           + _spmm_mod.__all__ + _gat_mod.__all__)
