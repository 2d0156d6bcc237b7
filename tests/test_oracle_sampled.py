"""The sampled oracle (oracle/sampled.py) against the full-graph oracle, on
CPU: every sampled row's result -- values, arg indices, softmax, the fused
GAT chain, segment ops -- is bit-identical to the full computation's row, for
any batch size.  This is what lets the full-size GPU checks trust a sample."""

import numpy as np
import pytest

from oracle import sampled as smp


def hub_graph(n=3000, e=60_000, seed=5):
    rng = np.random.default_rng(seed)
    u = rng.integers(0, n, e)
    v = rng.integers(0, n, e)
    v[rng.choice(e, 9000, replace=False)] = 17   # a hub of ~9000 in-edges
    return u, v


@pytest.mark.parametrize("max_edges", [200, 5000, 1 << 30])
def test_sampled_gspmm_matches_full(orc, max_edges):
    n = 3000
    u, v = hub_graph(n)
    rng = np.random.default_rng(6)
    h = rng.normal(size=(n, 6))
    ef = rng.normal(size=(u.size, 6))
    og = orc.Graph(u, v, num_nodes=n)
    rows = smp.sample_rows(og.indeg, 300, 5, seed=7)
    assert 17 in rows
    full_sum = orc.gspmm(og, "mul", "sum", h, ef)
    full_mean = orc.gspmm(og, "copy_lhs", "mean", h, None)
    full_max, fu, fe = orc.gspmm(og, "mul", "max", h, ef, with_arg=True)
    s = smp.RowSample(u, v, rows, n)
    for sl, lg in s.batches(max_edges):
        hl, el = h[lg.nodes], ef[lg.sel]
        r = rows[sl]
        np.testing.assert_array_equal(orc.gspmm(lg.graph, "mul", "sum", hl, el)[lg.rows],
                                      full_sum[r])
        np.testing.assert_array_equal(orc.gspmm(lg.graph, "copy_lhs", "mean", hl, None)[lg.rows],
                                      full_mean[r])
        mx, au, ae = orc.gspmm(lg.graph, "mul", "max", hl, el, with_arg=True)
        gu, ge = lg.global_args(au[lg.rows], ae[lg.rows])
        np.testing.assert_array_equal(mx[lg.rows], full_max[r])
        np.testing.assert_array_equal(gu, fu[r])
        np.testing.assert_array_equal(ge, fe[r])


def test_sampled_softmax_and_gat_match_full(orc):
    n = 3000
    u, v = hub_graph(n, seed=8)
    rng = np.random.default_rng(9)
    logits = rng.normal(size=(u.size, 4, 1))
    feat = rng.normal(size=(n, 4, 3))
    el, er = rng.normal(size=(n, 4, 1)), rng.normal(size=(n, 4, 1))
    og = orc.Graph(u, v, num_nodes=n)
    full_sm = orc.edge_softmax(og, logits)
    full_gat = orc.gat_aggregate(og, feat, el, er, 0.2)
    rows = smp.sample_rows(og.indeg, 200, 3, seed=10)
    s = smp.RowSample(u, v, rows, n)
    for sl, lg in s.batches(4000):
        np.testing.assert_array_equal(orc.edge_softmax(lg.graph, logits[lg.sel]), full_sm[lg.sel])
        got = orc.gat_aggregate(lg.graph, feat[lg.nodes], el[lg.nodes], er[lg.nodes], 0.2)
        np.testing.assert_array_equal(got[lg.rows], full_gat[rows[sl]])


def test_sampled_edges_and_segments_match_full(orc):
    n = 2000
    u, v = hub_graph(n, e=30_000, seed=11)
    rng = np.random.default_rng(12)
    a, b = rng.normal(size=(n, 5)), rng.normal(size=(n, 5))
    og = orc.Graph(u, v, num_nodes=n)
    full = orc.gsddmm(og, "dot", a, b, "u", "v")
    sel = smp.edge_sample(u.size, 700, seed=13)
    lg = smp.LocalGraph(u, v, sel, np.unique(v[sel]))
    np.testing.assert_array_equal(orc.gsddmm(lg.graph, "dot", a[lg.nodes], b[lg.nodes], "u", "v"),
                                  full[sel])
    seglen = rng.geometric(1 / 8, size=500)
    seglen[[3, 40]] = 0
    val = rng.normal(size=(int(seglen.sum()), 3))
    segs = np.sort(rng.choice(seglen.size, 120, replace=False))
    segs = np.union1d(segs, [3, 40])
    idx, lens = smp.segment_rows(seglen, segs)
    off = np.concatenate([[0], np.cumsum(seglen)])
    assert np.array_equal(idx, np.concatenate([np.arange(off[k], off[k + 1]) for k in segs]))
    for red in ("sum", "max", "mean"):
        np.testing.assert_array_equal(orc.segment_reduce(lens, val[idx], red),
                                      orc.segment_reduce(seglen, val, red)[segs])
    np.testing.assert_array_equal(orc.segment_softmax(lens, val[idx]),
                                  orc.segment_softmax(seglen, val)[idx])


def test_counting_sort_csr_matches_stable_argsort(orc):
    """oracle.csr_arrays (the O(E) CSR the full-size CPU arm uses) equals the
    stable-argsort CSR of oracle.Graph, in- and out-side, zero-degree nodes
    and a hub included."""
    u, v = hub_graph(3100, seed=14)
    og = orc.Graph(u, v, num_nodes=3100)
    indptr, deg, order, indices = orc.csr_arrays(v, u, 3100)
    np.testing.assert_array_equal(indptr, og.indptr)
    np.testing.assert_array_equal(deg, og.indeg)
    np.testing.assert_array_equal(order, og.in_order)
    np.testing.assert_array_equal(indices, og.in_indices)
    outptr, _, out_order, out_idx = orc.csr_arrays(u, v, 3100)
    np.testing.assert_array_equal(outptr, og.outptr)
    np.testing.assert_array_equal(out_order, og.out_order)
    np.testing.assert_array_equal(out_idx, og.out_indices)
