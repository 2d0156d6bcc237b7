"""Pins the CPU oracle (oracle/) before anything is checked against it.

1. Every known-answer vector the reference's own suite and README hold that
   needs no upstream dgl to evaluate (the values are restated from the
   reference's files, cited per test).
2. The reference's serial CSR-order restatement of gspmm
   (tests/test_parallel.py:74-111), which the oracle must match bit for bit.
3. The golden fixtures: the reference's own Python package run on the oracle's
   C kernels (tests/golden/make_golden.py).  oracle.py restates that Python
   layer in numpy; both must agree exactly.
"""

import itertools

import numpy as np
import pytest


# ------------------------------------------------------ known-answer vectors
def test_readme_example(orc):
    """README.md:9-28."""
    g = orc.Graph([0, 1, 2, 0, 1], [1, 2, 0, 2, 2])
    h = np.array([[1.0, 0.0], [0.0, 1.0], [2.0, 2.0]])
    e = np.array([[0.5, 0.5], [1.0, 0.0], [0.0, 1.0], [2.0, 1.0], [1.0, 1.0]])
    z = orc.update_all(g, {"h": h}, {"e": e}, ("u", "mul", "e", "h", "e"), "mean")
    np.testing.assert_allclose(z, [[0.0, 2.0], [0.5, 0.0], [2 / 3, 1 / 3]], rtol=1e-12)


def test_update_all_docstring_example(orc):
    """tests/test_function.py:172-177."""
    g = orc.Graph([0, 1, 2, 3], [1, 2, 3, 4])
    h = orc.update_all(g, {"x": np.ones((5, 2))}, {}, ("copy_u", "x"), "sum")
    np.testing.assert_array_equal(h, [[0, 0], [1, 1], [1, 1], [1, 1], [1, 1]])


def test_edge_softmax_docstring_example(orc):
    """tests/test_function.py:180-194, including the stale-docstring quirk
    (a four-row result for a four-edge selection)."""
    g = orc.Graph([0, 0, 0, 1, 1, 2], [0, 1, 2, 1, 2, 2])
    ones = np.ones((6, 1))
    np.testing.assert_allclose(orc.edge_softmax(g, ones).ravel(),
                               [1, 0.5, 1 / 3, 0.5, 1 / 3, 1 / 3], rtol=1e-15)
    np.testing.assert_allclose(orc.edge_softmax(g, ones, norm_by="src").ravel(),
                               [1 / 3, 1 / 3, 1 / 3, 0.5, 0.5, 1.0], rtol=1e-15)
    np.testing.assert_allclose(orc.edge_softmax(g, ones[:4], eids=np.array([0, 1, 2, 3])).ravel(),
                               [1.0, 0.5, 1.0, 0.5], rtol=1e-15)


def test_segment_docstring_example(orc):
    """tests/test_function.py:197-207."""
    val = np.ones((10, 3))
    seg = np.array([1, 0, 5, 4])
    np.testing.assert_array_equal(orc.segment_reduce(seg, val),
                                  [[1.0] * 3, [0.0] * 3, [5.0] * 3, [4.0] * 3])
    soft = orc.segment_softmax(seg, val)
    np.testing.assert_allclose(soft[0], [1, 1, 1])
    np.testing.assert_allclose(soft[1], [0.2, 0.2, 0.2])
    np.testing.assert_allclose(soft[6], [0.25, 0.25, 0.25])


def test_zero_degree_mean(orc):
    """tests/test_ops.py:452-457."""
    g = orc.Graph([0, 0], [1, 1], num_nodes=4)
    out = orc.gspmm(g, "add", "mean", np.ones((4, 4)), np.ones((2, 4)))
    np.testing.assert_array_equal(out[0], 0.0)
    np.testing.assert_array_equal(out[1], 2.0)
    np.testing.assert_array_equal(out[2:], 0.0)


def test_segment_mm_exact_n_boundary(orc):
    """tests/test_ops.py:496-499: a total of exactly n is accepted, = 3.0."""
    out = orc.segment_mm(np.ones((6, 3)), np.ones((4, 3, 2)), np.array([6, 0, 0, 0]))
    np.testing.assert_array_equal(out, np.full((6, 2), 3.0))


def test_gather_mm_two_to_the_53(orc):
    """tests/test_ops.py:543-551: 2^53 lands on float64 exactly."""
    half = float(2 ** 53)
    got = orc.gather_mm(np.full((2, 2), half), np.full((2, 2, 3), half), np.zeros(2, np.int64))
    np.testing.assert_array_equal(got, np.full((2, 3), 2.0 * half * half))


def test_gspmm_max_min_empty_rows_keep_identity(orc):
    """ported.mojo:347-350: no in-edges -> -inf / +inf before update_all's
    inf->0 (heterograph.py:232-239)."""
    g = orc.Graph([0, 1], [1, 2], num_nodes=5)
    x = np.arange(10.0).reshape(5, 2)
    assert np.all(orc.gspmm(g, "copy_lhs", "max", x, None)[[0, 3, 4]] == -np.inf)
    assert np.all(orc.gspmm(g, "copy_lhs", "min", x, None)[[0, 3, 4]] == np.inf)
    h = orc.update_all(g, {"x": x}, {}, ("copy_u", "x"), "max")
    np.testing.assert_array_equal(h[[0, 3, 4]], 0.0)


@pytest.mark.parametrize("norm_by", ["dst", "src"])
def test_positional_eids_rule(orc, norm_by):
    """tests/test_edge_softmax_eids.py:266-290: the rule stated as a formula --
    position i takes the softmax of logits[i] over the positions whose
    selected edge shares its endpoint."""
    rng = np.random.default_rng(21)
    u = rng.integers(0, 9, size=26)
    v = rng.integers(0, 9, size=26)
    g = orc.Graph(u, v)
    logits = rng.normal(size=(26, 1))
    eids = np.array([23, 4, 15, 11, 20, 3, 6])
    key = (v if norm_by == "dst" else u).tolist()
    want = np.zeros((len(eids), 1))
    for i in range(len(eids)):
        group = [j for j in range(len(eids)) if key[eids[j]] == key[eids[i]]]
        w = logits[np.array(group)]
        ex = np.exp(w - w.max())
        want[i] = (ex / ex.sum())[group.index(i)]
    got = orc.edge_softmax(g, logits, eids=eids, norm_by=norm_by)
    np.testing.assert_allclose(got[: len(eids)], want, rtol=1e-11, atol=1e-13)
    np.testing.assert_array_equal(got[len(eids):], 0.0)


def test_gspmm_matches_serial_csr_order_loop_bitwise(orc):
    """tests/test_parallel.py:74-111: a destination's messages accumulated in
    CSR order, per column, with separate multiply and add -- bit for bit."""
    rng = np.random.default_rng(8)
    nodes, edges = 6000, 24000  # above PARALLEL_MIN: the 32-way split runs
    u = rng.integers(0, nodes, size=edges)
    v = rng.integers(0, nodes, size=edges)
    x = rng.normal(size=(nodes, 5))
    e = rng.normal(size=(edges, 5))
    got = orc.gspmm(orc.Graph(u, v), "mul", "sum", x, e)
    order = np.argsort(v, kind="stable")
    bounds = np.searchsorted(v[order], np.arange(nodes + 1))
    ref = np.zeros((nodes, 5))
    for node in range(nodes):
        acc = ref[node]
        for pos in range(bounds[node], bounds[node + 1]):
            edge = order[pos]
            acc += x[u[edge]] * e[edge]
    np.testing.assert_array_equal(got, ref)


# ----------------------------------------------------- against the fixtures
def G0(golden, orc):
    return orc.Graph(golden["graph0/u"], golden["graph0/v"])


def test_graph_csr_matches_reference(golden, orc):
    g = G0(golden, orc)
    for a, b in [(g.indptr, "indptr"), (g.in_indices, "in_indices"), (g.in_order, "in_order"),
                 (g.outptr, "outptr"), (g.out_indices, "out_indices"),
                 (g.out_order, "out_order"), (g.indeg, "indeg"), (g.outdeg, "outdeg")]:
        np.testing.assert_array_equal(a, golden["graph0/" + b])


def test_spmm_families_match_reference(golden, orc):
    g = G0(golden, orc)
    x, e = golden["graph0/x"], golden["graph0/e"]
    for bop, red in itertools.product(["add", "sub", "mul", "div"], ["sum", "max", "min", "mean"]):
        np.testing.assert_array_equal(orc.gspmm(g, bop, red, x, e),
                                      golden["spmm/u_{}_e_{}/out".format(bop, red)])
    for src, red in itertools.product(["copy_u", "copy_e"], ["sum", "max", "min", "mean"]):
        op = "copy_lhs" if src == "copy_u" else "copy_rhs"
        got = orc.gspmm(g, op, red, x if src == "copy_u" else None, e if src == "copy_e" else None)
        np.testing.assert_array_equal(got, golden["spmm/{}_{}/out".format(src, red)])
    np.testing.assert_array_equal(orc.gspmm(g, "add", "sum", golden["graph0/y1"], e),
                                  golden["spmm/u_add_e_sum_bcast/out"])


def test_sddmm_families_match_reference(golden, orc):
    g = G0(golden, orc)
    data = {"u": golden["graph0/x"], "v": golden["graph0/x"], "e": golden["graph0/e"]}
    for (lt, rt), op in itertools.product(itertools.permutations("uve", 2),
                                          ["add", "sub", "mul", "div", "dot"]):
        np.testing.assert_array_equal(orc.gsddmm(g, op, data[lt], data[rt], lt, rt),
                                      golden["sddmm/{}_{}_{}/out".format(lt, op, rt)])


def test_segment_and_mm_match_reference(golden, orc):
    seglen = golden["segred/arange/seglen"]
    for red in ["sum", "max", "min", "mean"]:
        np.testing.assert_array_equal(orc.segment_reduce(seglen, golden["segred/arange/value"], red),
                                      golden["segred/arange/{}/out".format(red)])
    for i in range(4):
        for d in [1, 3, 4, 32]:
            k = "segsoft/{}/{}/".format(i, d)
            np.testing.assert_array_equal(orc.segment_softmax(golden[k + "seglen"], golden[k + "value"]),
                                          golden[k + "out"])
    for d2 in [1, 3, 4, 5, 8, 9]:
        k = "gathermm/d2_{}/".format(d2)
        np.testing.assert_array_equal(orc.gather_mm(golden[k + "a"], golden[k + "b"], golden[k + "idx"]),
                                      golden[k + "out"])
    k = "gathermm/segment_route/"
    np.testing.assert_array_equal(
        orc.gather_mm(golden[k + "a"], golden[k + "b"], golden[k + "idx"], segment_block=0),
        golden[k + "out"])


def test_edge_softmax_matches_reference(golden, orc):
    g = G0(golden, orc)
    lg = golden["esoft/logits1/logits"]
    for nb in ["dst", "src"]:
        np.testing.assert_array_equal(orc.edge_softmax(g, lg, norm_by=nb), golden["esoft/{}/out".format(nb)])
    np.testing.assert_array_equal(orc.edge_softmax(g, lg, eids=golden["esoft/subset/eids"]),
                                  golden["esoft/subset/out"])
    for case in range(40):
        k = "esoft/rand{}/".format(case)
        gg = orc.Graph(golden[k + "u"], golden[k + "v"])
        got = orc.edge_softmax(gg, golden[k + "logits"], eids=golden[k + "eids"],
                               norm_by=str(golden[k + "norm_by"]))
        np.testing.assert_array_equal(got, golden[k + "out"])


def test_update_all_matches_reference(golden, orc):
    g = orc.Graph(golden["fn/u"], golden["fn/v"])
    nd, ed = {"x": golden["fn/x"]}, {"e": golden["fn/e"]}
    for name, red in itertools.product(["copy_u", "copy_e"], ["sum", "max", "min", "mean"]):
        msg = (name, "x" if name == "copy_u" else "e")
        np.testing.assert_array_equal(orc.update_all(g, nd, ed, msg, red),
                                      golden["fn/{}_{}/h".format(name, red)])
    for (lt, rt), op in itertools.product(itertools.permutations("uve", 2),
                                          ["add", "sub", "mul", "div", "dot"]):
        for red in ["sum", "max"]:
            msg = (lt, op, rt, "e" if lt == "e" else "x", "e" if rt == "e" else "x")
            np.testing.assert_array_equal(orc.update_all(g, nd, ed, msg, red),
                                          golden["fn/{}_{}_{}/{}/h".format(lt, op, rt, red)])
