"""bench.py's host-side pieces, on CPU: the config-3 generator, the default
rank grids, the gathered-bytes model, and the sampled parity check that
every bench line carries -- it must pass a correct result and flag a result
with one wrong value."""

import numpy as np

import bench


def small_cfg3(seed=3):
    return bench.make_cfg3(num_nodes=4000, num_edges=150_000, dim=8, seed=seed)


def test_cfg3_generator_is_exact_and_deterministic():
    u, v, h = small_cfg3()
    assert u.size == v.size == 150_000  # degrees rounded to sum to E exactly
    assert np.all(np.diff(u) >= 0)  # source-major edge order
    assert 0 <= u.min() and u.max() < 4000 and 0 <= v.min() and v.max() < 4000
    assert h.shape == (4000, 8) and h.dtype == np.float32
    assert h.min() >= -1.0 and h.max() < 1.0
    u2, v2, h2 = small_cfg3()
    np.testing.assert_array_equal(u, u2)
    np.testing.assert_array_equal(v, v2)
    np.testing.assert_array_equal(h, h2)
    # the out-degree tail is capped, as the generator states
    assert np.bincount(u, minlength=4000).max() <= 20_000


def test_default_grids_tile_ranks_and_columns():
    from mojodgl.partition import column_range, rank_grid

    d = bench.CFG3["dim"]
    for n, cols in bench.GRID_COLS.items():
        assert n % cols == 0 and d % cols == 0
        widths = {column_range(d, cols, cg)[1] - column_range(d, cols, cg)[0]
                  for cg in range(cols)}
        assert widths == {d // cols}
        cells = {rank_grid(r, n, cols)[1:] for r in range(n)}
        assert cells == {(rg, cg) for rg in range(n // cols) for cg in range(cols)}


def test_gathered_bytes_model():
    rows, edges, d = 10, 100, 4
    want = edges * d * 4 + edges * 4 + rows * d * 4 + (rows + 1) * 8
    assert bench.algorithmic_bytes(rows, edges, d) == want
    assert bench.algorithmic_bytes(rows, edges, d, arg=True) == want + rows * d * 8
    assert bench.algorithmic_bytes(rows, edges, d, elem=8) == (
        edges * d * 8 + edges * 4 + rows * d * 8 + (rows + 1) * 8)


def test_parity_check_passes_a_correct_result_and_flags_one_wrong_value(orc):
    u, v, h = small_cfg3(seed=4)
    n = h.shape[0]
    indeg = np.bincount(v, minlength=n)
    full = orc.gspmm(orc.Graph(u, v, num_nodes=n), "copy_lhs", "mean", h.astype(np.float64),
                     None).astype(np.float32)
    lo, hi = 700, 3300
    r = bench.check_parity(u, v, h, indeg, full[lo:hi], lo, hi, n, seed=1, rows=400, top=25)
    assert r["ok"] and r["max_excess"] <= 0.0
    # 400 random rows of the range plus its 25 highest in-degree rows, with overlaps merged
    assert 400 <= r["rows"] <= 425 and r["edges"] > 0
    # the range's highest in-degree row is always among the sampled rows
    bad = full[lo:hi].copy()
    k = int(np.argmax(indeg[lo:hi]))
    bad[k, 3] += 1e-3 * (1.0 + abs(bad[k, 3]))
    r2 = bench.check_parity(u, v, h, indeg, bad, lo, hi, n, seed=1, rows=400, top=25)
    assert not r2["ok"] and r2["max_excess"] > 0.0
