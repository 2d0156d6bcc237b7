"""Fused GAT aggregation against the reference's four-operator chain
(u_add_v -> leaky_relu -> edge_softmax(dst) -> u_mul_e_sum) computed by the
oracle in float64.

Tolerances: float64 rtol 1e-10 (the fused pass rescales running sums and
divides once; the chain forms per-edge weights first); float32 |got - want| <=
1e-5 |want| + 1e-5 S with S the same chain over |feat|.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import mojodgl as dgl  # noqa: E402
import mojodgl.ops as ops  # noqa: E402
from mojodgl import _lib  # noqa: E402


def power_law(n, seed, mean_deg=12, cap=3000):
    rng = np.random.default_rng(seed)
    w = np.minimum(rng.zipf(2.1, n), cap).astype(np.float64)
    deg = np.floor(w / w.sum() * n * mean_deg).astype(np.int64)
    v = np.repeat(np.arange(n), deg)
    u = rng.integers(0, n, v.size)
    p = rng.permutation(v.size)
    return u[p], v[p]


@pytest.fixture(params=[False, True], ids=["chunks", "split-rows"])
def chunking(request):
    if request.param:
        _lib.set_param("spmm_min_items", 16)
        _lib.set_param("spmm_max_chunks", 1 << 40)
        _lib.set_param("spmm_split_min", 0)
    yield request.param
    _lib.set_param("spmm_min_items", 32)
    _lib.set_param("spmm_max_chunks", 0)
    _lib.set_param("spmm_split_min", 512)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("heads,dim", [(8, 16), (2, 3)])
def test_gat_aggregate_matches_the_operator_chain(orc, chunking, dtype, heads, dim):
    u, v = power_law(3000, 61)
    n = 3050  # 50 nodes without in-edges
    rng = np.random.default_rng(62)
    feat = rng.normal(size=(n, heads, dim)).astype(dtype)
    el = (rng.normal(size=(n, heads, 1)) * 2).astype(dtype)
    er = (rng.normal(size=(n, heads, 1)) * 2).astype(dtype)
    g, og = dgl.graph((u, v), num_nodes=n), orc.Graph(u, v, num_nodes=n)
    got = ops.gat_aggregate(g, feat, el, er, negative_slope=0.2)
    assert got.shape == (n, heads, dim) and got.dtype == dtype
    want = orc.gat_aggregate(og, feat, el, er, 0.2)
    if dtype == np.float64:
        np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-13)
    else:
        s = orc.gat_aggregate(og, np.abs(feat), el, er, 0.2)
        err = np.abs(got.astype(np.float64) - want)
        assert np.all(err <= 1e-5 * np.abs(want) + 1e-5 * s + 1e-30), err.max()
    lonely = np.setdiff1d(np.arange(n), v)
    assert lonely.size and np.all(got[lonely] == 0)
