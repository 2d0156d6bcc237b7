"""TEST INFRASTRUCTURE -- the oracle on a sample of a full-size graph.

Only ``tests/`` and the CPU leg of ``bench.py`` use this module, as the
checker; the product never does.

At the BASELINE configurations' full sizes (125M edges, 64 GB of edge
features) the float64 oracle cannot recompute every output row in seconds, so
the checks sample: a set of destination rows (or edges, or segments) is
chosen, and the oracle runs the reference's algorithm on a *local* graph made
of exactly the in-edges of the sampled rows.  Because every sampled row keeps
all of its in-edges, in ascending global edge id (the order of the
reference's in-CSR: a stable argsort by destination,
python/mojodgl/heterograph.py:69-86), each sampled row's result -- value,
rounding and arg indices -- is the one the full-graph oracle would give.
Node and edge features are fetched for the local graph only, so memory stays
bounded by the sample, processed in batches of at most ``max_edges`` edges.
"""

from __future__ import annotations

import numpy as np

from . import oracle as orc


def sample_rows(indeg, count, top, seed):
    """``count`` distinct random destination rows plus the ``top`` rows of
    highest in-degree (the hubs a merge-path split cuts into pieces), sorted."""
    n = int(indeg.size)
    rng = np.random.default_rng(seed)
    rand = rng.choice(n, size=min(count, n), replace=False)
    hubs = np.argsort(-np.asarray(indeg), kind="stable")[: min(top, n)]
    return np.unique(np.concatenate([rand, hubs]).astype(np.int64))


class RowSample:
    """The in-edges of the sampled destination ``rows`` of the graph (u, v)."""

    def __init__(self, u, v, rows, num_nodes):
        self.u, self.v = u, v
        self.rows = np.unique(np.asarray(rows, dtype=np.int64))
        pos = np.full(int(num_nodes), -1, dtype=np.int64)
        pos[self.rows] = np.arange(self.rows.size)
        r = pos[v]
        self.sel = np.flatnonzero(r >= 0)      # ascending global edge ids
        self.pos = r[self.sel]                 # each edge's sampled-row position
        self.deg = np.bincount(self.pos, minlength=self.rows.size)

    @property
    def num_edges(self):
        return int(self.sel.size)

    def batches(self, max_edges):
        """Consecutive runs of sampled rows holding at most ``max_edges``
        in-edges (a longer row forms a batch of its own): yields
        (row positions slice, LocalGraph)."""
        cum = np.concatenate([[0], np.cumsum(self.deg)])
        start, k = 0, self.rows.size
        while start < k:
            end = int(np.searchsorted(cum, cum[start] + max_edges, side="right")) - 1
            end = min(max(end, start + 1), k)
            m = (self.pos >= start) & (self.pos < end)
            yield slice(start, end), LocalGraph(self.u, self.v, self.sel[m], self.rows[start:end])
            start = end


class LocalGraph:
    """The edges ``sel`` (ascending global ids) relabelled onto the local node
    set ``nodes`` (sources and the sampled rows, ascending global ids), as an
    oracle Graph.  ``rows`` are the local ids of the sampled rows."""

    def __init__(self, u, v, sel, rows):
        us, vs = np.asarray(u[sel], dtype=np.int64), np.asarray(v[sel], dtype=np.int64)
        self.sel = np.asarray(sel, dtype=np.int64)
        self.nodes = np.unique(np.concatenate([us, vs, np.asarray(rows, dtype=np.int64)]))
        self.graph = orc.Graph(np.searchsorted(self.nodes, us), np.searchsorted(self.nodes, vs),
                               num_nodes=self.nodes.size)
        self.rows = np.searchsorted(self.nodes, rows)

    def global_args(self, arg_u, arg_e):
        """Map the oracle's local arg indices back to global node / edge ids
        (-1, an empty row, stays -1)."""
        gu = np.where(arg_u >= 0, self.nodes[np.maximum(arg_u, 0)], -1)
        ge = np.where(arg_e >= 0, self.sel[np.maximum(arg_e, 0)], -1)
        return gu, ge


def edge_sample(num_edges, count, seed):
    """``count`` distinct random edge ids, sorted."""
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(int(num_edges), size=min(count, int(num_edges)), replace=False))


def segment_rows(seglen, segs):
    """The value rows of the segments ``segs`` (ascending), concatenated, and
    those segments' lengths (python/mojodgl/ops/segment.py:12-21 offsets)."""
    seglen = np.asarray(seglen, dtype=np.int64)
    off = np.concatenate([[0], np.cumsum(seglen)])
    lens = seglen[segs]
    starts = off[segs]
    total = int(lens.sum())
    base = np.repeat(starts - np.concatenate([[0], np.cumsum(lens)[:-1]]), lens)
    return base + np.arange(total, dtype=np.int64), lens


def excess(got, ref, s, tol):
    """Largest amount by which |got - ref| exceeds tol |ref| + tol S (<= 0 when
    the bound holds everywhere) and the largest |got - ref|."""
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    if err.size == 0:
        return -np.inf, 0.0
    return float((err - (tol * np.abs(ref) + tol * s)).max()), float(err.max())
