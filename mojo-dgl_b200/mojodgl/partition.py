"""Destination-row partitioning of one graph across the GPUs of a node.

Every output row of gSpMM is independent (the reference splits its 32 CPU
workers the same way, src/ported.mojo:34-39, 442-443), so the graph is cut
into P contiguous destination-row ranges with about E/P in-edges each (a
row-count split would not balance a power-law in-degree).  Node features are
owned in P contiguous, equal row blocks; before an aggregation every rank
gathers the full feature matrix with one NCCL all-gather (the halo: with
uniform sources a shard references nearly every source row, so a selective
exchange would not pay), then runs gSpMM on its own rows.  Outputs stay
sharded by destination row.

The host logic here (ranges, shard extraction, block layout) is plain numpy
and is tested with gloo ranks on CPU; the kernels run through mojodgl.
"""

from __future__ import annotations

import numpy as np


def edge_balanced_ranges(indeg: np.ndarray, parts: int):
    """P+1 row boundaries so each range holds ~E/P in-edges (ties -> rows)."""
    n = int(indeg.size)
    csum = np.concatenate([[0], np.cumsum(indeg, dtype=np.int64)])
    total = int(csum[-1])
    bounds = [0]
    for p in range(1, parts):
        target = total * p // parts
        r = int(np.searchsorted(csum, target, side="left"))
        bounds.append(min(max(r, bounds[-1]), n))
    bounds.append(n)
    return np.asarray(bounds, dtype=np.int64)


def owner_blocks(n: int, parts: int):
    """Equal contiguous feature-row blocks (the last ones may be shorter);
    block p covers rows [p * b, min((p + 1) * b, n)), b = ceil(n / P)."""
    b = (n + parts - 1) // parts
    return b, [(min(p * b, n), min((p + 1) * b, n)) for p in range(parts)]


class DstShard:
    """One rank's destination-row range and the in-edges that land in it.

    ``u`` keeps global source ids (they index the all-gathered features);
    ``v_local`` is the destination minus the range start; edges keep their
    global order, so the shard's in-CSR (stable by destination) lists every
    row's in-edges in the same order as the full graph's CSR and the
    per-row accumulation order -- hence the result -- is unchanged."""

    def __init__(self, u: np.ndarray, v: np.ndarray, lo: int, hi: int):
        sel = np.nonzero((v >= lo) & (v < hi))[0]
        self.lo, self.hi = int(lo), int(hi)
        self.eids = sel.astype(np.int64)
        self.u = np.ascontiguousarray(u[sel], dtype=np.int64)
        self.v_local = np.ascontiguousarray(v[sel] - lo, dtype=np.int64)

    @property
    def num_rows(self):
        return self.hi - self.lo

    @property
    def num_edges(self):
        return int(self.u.size)


def assemble_gathered(blocks, n: int):
    """Concatenate the P gathered (padded) owner blocks into the (n, ...) matrix."""
    return np.concatenate(blocks, axis=0)[:n]


class DeviceShard:
    """A DstShard's in-CSR on the current CUDA device, ready for gSpMM over
    all-gathered source features (sources are global ids, destinations are
    the shard's local rows)."""

    def __init__(self, shard: DstShard):
        import torch

        from . import _tensor as T
        from ._lib import check, lib

        self.shard = shard
        n, ne = shard.num_rows, shard.num_edges
        dev = T.device()
        key = torch.from_numpy(shard.v_local).to(dev)
        other = torch.from_numpy(shard.u).to(dev)
        self.indptr = torch.empty(n + 1, dtype=torch.int64, device=dev)
        self.deg = torch.empty(n, dtype=torch.int64, device=dev)
        self.eid = torch.empty(ne, dtype=torch.int32, device=dev)
        self.indices = torch.empty(ne, dtype=torch.int32, device=dev)
        nbytes = lib().bgl_csr_build_workspace_size(ne, n)
        ws = T.workspace(nbytes)
        check(lib().bgl_csr_build(T.ptr(key), T.ptr(other), ne, n, T.ptr(self.indptr),
                                  T.ptr(self.deg), T.ptr(self.eid), T.ptr(self.indices),
                                  T.ptr(ws), nbytes, T.stream()), "bgl_csr_build")
        del key, other, ws

    def copy_u(self, feat, reduce_op: str, out=None, arg_u=None, workspace=None):
        """gSpMM copy_u over this shard: feat is the full (N, D) device matrix."""
        import torch

        from . import _tensor as T
        from ._lib import BGL_ZERO_INF, OP_COPY_LHS, REDUCERS, check, lib

        n, ne = self.shard.num_rows, self.shard.num_edges
        d = int(feat.shape[1])
        code = T.code_of(feat.dtype)
        red = REDUCERS[reduce_op]
        if out is None:
            out = torch.empty((n, d), dtype=feat.dtype, device=feat.device)
        nbytes = lib().bgl_gspmm_workspace_size(n, ne, d, code, red)
        if workspace is None or workspace.numel() < nbytes:
            workspace = T.workspace(nbytes)
        check(lib().bgl_gspmm(T.ptr(self.indptr), T.ptr(self.indices), None, T.ptr(self.deg), n, ne,
                              T.ptr(feat), d, 1, None, 1, 1, T.ptr(out), d, T.ptr(arg_u), None, code,
                              OP_COPY_LHS, red, BGL_ZERO_INF if reduce_op in ("max", "min") else 0,
                              T.ptr(workspace), nbytes, T.stream()), "gspmm")
        return out
