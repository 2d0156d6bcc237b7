"""dgl.nn.functional: edge_softmax is the ops function itself."""

from ...ops import edge_softmax  # noqa: F401
