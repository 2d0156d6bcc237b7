"""GPU parity against the golden fixtures (the reference's Python package run
on the oracle kernels, tests/golden/make_golden.py), through mojodgl's public
API on the sm_100a kernels, at float64.

Bars: integer outputs (CSR arrays, degrees) bit-exact; gspmm, segment_reduce,
segment_mm and gather_mm bit-exact (same per-column CSR-order accumulation,
separately rounded multiply and add); gsddmm element-wise ops bit-exact;
`dot` and the softmaxes within the reference's own rtol 1e-12
(tests/upstream.py:40-46) because their summation order or exp differ.
"""

import itertools

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import mojodgl as dgl  # noqa: E402
import mojodgl.function as fn  # noqa: E402
import mojodgl.ops as ops  # noqa: E402

RTOL = 1e-12


def close(got, want, atol=1e-13):
    got = np.asarray(got)
    assert got.shape == want.shape, (got.shape, want.shape)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=atol)


@pytest.fixture(scope="module")
def g0(golden):
    return dgl.graph((golden["graph0/u"], golden["graph0/v"]))


def test_csr_and_degrees_bit_exact(golden, g0):
    ip, nbr, order = g0._in_csr()
    np.testing.assert_array_equal(ip, golden["graph0/indptr"])
    np.testing.assert_array_equal(nbr, golden["graph0/in_indices"])
    np.testing.assert_array_equal(order, golden["graph0/in_order"])
    ip, nbr, order = g0._out_csr()
    np.testing.assert_array_equal(ip, golden["graph0/outptr"])
    np.testing.assert_array_equal(nbr, golden["graph0/out_indices"])
    np.testing.assert_array_equal(order, golden["graph0/out_order"])
    np.testing.assert_array_equal(g0.in_degrees(), golden["graph0/indeg"])
    np.testing.assert_array_equal(g0.out_degrees(), golden["graph0/outdeg"])


@pytest.mark.parametrize("bop,red", list(itertools.product(
    ["add", "sub", "mul", "div"], ["sum", "max", "min", "mean"])))
def test_gspmm_families(golden, g0, bop, red):
    name = "u_{}_e_{}".format(bop, red)
    got = getattr(ops, name)(g0, golden["graph0/x"], golden["graph0/e"])
    np.testing.assert_array_equal(got, golden["spmm/{}/out".format(name)])


@pytest.mark.parametrize("src,red", list(itertools.product(["copy_u", "copy_e"],
                                                           ["sum", "max", "min", "mean"])))
def test_gspmm_copy_families(golden, g0, src, red):
    name = "{}_{}".format(src, red)
    data = golden["graph0/x"] if src == "copy_u" else golden["graph0/e"]
    np.testing.assert_array_equal(getattr(ops, name)(g0, data), golden["spmm/{}/out".format(name)])


def test_gspmm_scalar_column_broadcast(golden, g0):
    np.testing.assert_array_equal(ops.u_add_e_sum(g0, golden["graph0/y1"], golden["graph0/e"]),
                                  golden["spmm/u_add_e_sum_bcast/out"])


@pytest.mark.parametrize("lt,rt", list(itertools.permutations("uve", 2)))
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "dot"])
def test_gsddmm_families(golden, g0, lt, rt, op):
    data = {"u": golden["graph0/x"], "v": golden["graph0/x"], "e": golden["graph0/e"]}
    name = "{}_{}_{}".format(lt, op, rt)
    got = getattr(ops, name)(g0, data[lt], data[rt])
    want = golden["sddmm/{}/out".format(name)]
    if op == "dot":
        close(got, want)
    else:
        np.testing.assert_array_equal(got, want)


def test_gsddmm_copies(golden, g0):
    x = golden["graph0/x"]
    np.testing.assert_array_equal(ops.gsddmm(g0, "copy_lhs", x, None), golden["sddmm/copy_lhs/out"])
    np.testing.assert_array_equal(ops.gsddmm(g0, "copy_rhs", None, golden["graph0/y1"]),
                                  golden["sddmm/copy_rhs_y1/out"])
    np.testing.assert_array_equal(ops.copy_u(g0, x), golden["sddmm/copy_u/out"])
    np.testing.assert_array_equal(ops.copy_v(g0, x), golden["sddmm/copy_v/out"])
    e = golden["graph0/e"]
    assert ops.copy_e(g0, e) is e


@pytest.mark.parametrize("d", [1, 2, 3, 5, 7, 8, 16, 33])
def test_every_feature_width(golden, g0, d):
    k = "width{}/".format(d)
    x, e = golden[k + "x"], golden[k + "e"]
    for name, args in (("u_add_e_sum", (x, e)), ("u_div_e_min", (x, e)),
                       ("u_mul_e_mean", (x, e)), ("copy_u_max", (x,)), ("copy_e_sum", (e,)),
                       ("u_mul_v", (x, x)), ("u_add_e", (x, e))):
        np.testing.assert_array_equal(getattr(ops, name)(g0, *args), golden[k + name], err_msg=name)
    close(ops.u_dot_e(g0, x, e), golden[k + "u_dot_e"])


def test_offset_views(golden, g0):
    """Views whose base is one element into the allocation (tests/test_ops.py:416-449)."""
    x = golden["width5/x"]
    buf = np.empty(x.size + 1)
    buf[1:] = x.ravel()
    xv = buf[1:].reshape(x.shape)
    np.testing.assert_array_equal(ops.copy_u_max(g0, xv), golden["width5/copy_u_max"])


@pytest.mark.parametrize("red", ["sum", "max", "min", "mean"])
def test_segment_reduce(golden, red):
    seglen = golden["segred/arange/seglen"]
    np.testing.assert_array_equal(ops.segment_reduce(seglen, golden["segred/arange/value"], red),
                                  golden["segred/arange/{}/out".format(red)])
    for d in [1, 3, 5, 8, 33]:
        k = "segred/w{}/".format(d)
        np.testing.assert_array_equal(ops.segment_reduce(seglen, golden[k + "value"], red),
                                      golden[k + red])


def test_segment_softmax(golden):
    for i in range(4):
        for d in [1, 3, 4, 32]:
            k = "segsoft/{}/{}/".format(i, d)
            close(ops.segment_softmax(golden[k + "seglen"], golden[k + "value"]), golden[k + "out"])
    close(ops.segment_softmax(golden["segsoft/arange/seglen"], golden["segsoft/arange/value"]),
          golden["segsoft/arange/out"])


def test_segment_mm_and_gather_mm(golden):
    k = "segmm/arange/"
    np.testing.assert_array_equal(ops.segment_mm(golden[k + "a"], golden[k + "b"], golden[k + "seglen"]),
                                  golden[k + "out"])
    for d2 in [1, 3, 4, 5, 8, 9]:
        k = "segmm/d2_{}/".format(d2)
        np.testing.assert_array_equal(
            ops.segment_mm(golden[k + "a"], golden[k + "b"], np.array([10, 5, 0, 3])), golden[k + "out"])
        k = "gathermm/d2_{}/".format(d2)
        np.testing.assert_array_equal(ops.gather_mm(golden[k + "a"], golden[k + "b"], idx_b=golden[k + "idx"]),
                                      golden[k + "out"])
    for k in ["gathermm/arange/", "gathermm/segment_route/"]:
        np.testing.assert_array_equal(ops.gather_mm(golden[k + "a"], golden[k + "b"], idx_b=golden[k + "idx"]),
                                      golden[k + "out"])


def test_edge_softmax(golden, g0):
    lg = golden["esoft/logits1/logits"]
    for nb in ["dst", "src"]:
        close(ops.edge_softmax(g0, lg, norm_by=nb), golden["esoft/{}/out".format(nb)])
        for h in [1, 3, 8]:
            k = "esoft/{}/h{}/".format(nb, h)
            close(ops.edge_softmax(g0, golden[k + "logits"], norm_by=nb), golden[k + "out"])
    close(ops.edge_softmax(g0, lg, eids=golden["esoft/subset/eids"]), golden["esoft/subset/out"])
    close(ops.edge_softmax(g0, golden["esoft/subset_h4/logits"], eids=golden["esoft/subset/eids"]),
          golden["esoft/subset_h4/out"])
    close(ops.edge_softmax(g0, lg, eids=golden["esoft/repeat/eids"]), golden["esoft/repeat/out"])
    for case in range(40):
        k = "esoft/rand{}/".format(case)
        g = dgl.graph((golden[k + "u"], golden[k + "v"]))
        close(ops.edge_softmax(g, golden[k + "logits"], eids=golden[k + "eids"],
                               norm_by=str(golden[k + "norm_by"])), golden[k + "out"])


def _pair(golden):
    g = dgl.graph((golden["fn/u"], golden["fn/v"]))
    g.ndata["x"] = golden["fn/x"]
    g.edata["e"] = golden["fn/e"]
    return g


def test_update_all_builtins(golden):
    for name, red in itertools.product(["copy_u", "copy_e"], ["sum", "max", "min", "mean"]):
        g = _pair(golden)
        g.update_all(getattr(fn, name)("x" if name == "copy_u" else "e", "m"), getattr(fn, red)("m", "h"))
        np.testing.assert_array_equal(g.ndata["h"], golden["fn/{}_{}/h".format(name, red)])
    for (lt, rt), op in itertools.product(itertools.permutations("uve", 2),
                                          ["add", "sub", "mul", "div", "dot"]):
        for red in ["sum", "max"]:
            g = _pair(golden)
            g.update_all(getattr(fn, "{}_{}_{}".format(lt, op, rt))(
                "e" if lt == "e" else "x", "e" if rt == "e" else "x", "m"), getattr(fn, red)("m", "h"))
            want = golden["fn/{}_{}_{}/{}/h".format(lt, op, rt, red)]
            if op == "dot":
                close(g.ndata["h"], want, atol=1e-12)
            else:
                np.testing.assert_array_equal(g.ndata["h"], want)


def test_update_all_udfs_and_pull(golden):
    g = _pair(golden)
    g.update_all(lambda edges: {"m": edges.src["x"] * edges.data["e"] + 1.0}, fn.mean("m", "h"))
    np.testing.assert_array_equal(g.ndata["h"], golden["fn/udf_msg_mean/h"])
    g = _pair(golden)
    g.update_all(fn.copy_u("x", "m"), fn.sum("m", "h"), lambda nodes: {"h": nodes.data["h"] * 0.5 + 2.0})
    np.testing.assert_array_equal(g.ndata["h"], golden["fn/apply/h"])
    g = _pair(golden)
    g.update_all(fn.u_mul_e("x", "e", "m"), lambda nodes: {"h": nodes.mailbox["m"] * 2.0})
    np.testing.assert_array_equal(g.ndata["h"], golden["fn/udf_reduce/h"])
    g = _pair(golden)
    g.pull(golden["fn/pull/targets"], fn.u_mul_e("x", "e", "m"), fn.sum("m", "h"),
           apply_node_func=lambda nodes: {"h": nodes.data["h"] + 1.0})
    np.testing.assert_array_equal(g.ndata["h"], golden["fn/pull/h"])
    g = _pair(golden)
    g.pull(golden["fn/pull/targets"], lambda edges: {"m": edges.src["x"] * edges.data["e"] + 1.0},
           fn.mean("m", "h"))
    np.testing.assert_array_equal(g.ndata["h"], golden["fn/pull_udf/h"])


def test_udfs_on_device_tensors(golden):
    """The UDF paths with the graph and its features as CUDA tensors: the
    message and reduce functions see device tensors, nothing leaves the
    device, and the results equal the reference's (float64, bit for bit)."""
    import torch

    dev = torch.device("cuda", 0)

    def pair():
        g = dgl.graph((torch.from_numpy(golden["fn/u"]).to(dev), torch.from_numpy(golden["fn/v"]).to(dev)))
        g.ndata["x"] = torch.from_numpy(golden["fn/x"]).to(dev)
        g.edata["e"] = torch.from_numpy(golden["fn/e"]).to(dev)
        return g

    seen = []

    def msg(edges):
        seen.append(edges.src["x"].device)
        return {"m": edges.src["x"] * edges.data["e"] + 1.0}

    g = pair()
    g.update_all(msg, fn.mean("m", "h"))
    h = g.ndata["h"]
    assert isinstance(h, torch.Tensor) and h.is_cuda and seen[-1].type == "cuda"
    np.testing.assert_array_equal(h.cpu().numpy(), golden["fn/udf_msg_mean/h"])
    g = pair()
    g.update_all(fn.u_mul_e("x", "e", "m"), lambda nodes: {"h": nodes.mailbox["m"] * 2.0})
    assert g.ndata["h"].is_cuda
    np.testing.assert_array_equal(g.ndata["h"].cpu().numpy(), golden["fn/udf_reduce/h"])
    g = pair()
    g.pull(torch.from_numpy(golden["fn/pull/targets"]).to(dev), msg, fn.mean("m", "h"))
    np.testing.assert_array_equal(g.ndata["h"].cpu().numpy(), golden["fn/pull_udf/h"])


def test_zero_degree_rows(golden):
    g = dgl.graph((golden["zero/u"], golden["zero/v"]), num_nodes=5)
    x, e = golden["zero/x"], golden["zero/e"]
    np.testing.assert_array_equal(ops.u_add_e_sum(g, x, e), golden["zero/u_add_e_sum"])
    np.testing.assert_array_equal(ops.u_mul_e_mean(g, x, e), golden["zero/u_mul_e_mean"])
    np.testing.assert_array_equal(ops.copy_u_max(g, x), golden["zero/copy_u_max"])
    np.testing.assert_array_equal(ops.copy_e_min(g, e), golden["zero/copy_e_min"])


def test_large_graph_with_a_hub(golden):
    """A destination with 2500 in-edges: its row is split across merge-path
    chunks and its pieces folded in CSR order -- max/min stay exact, sums
    agree to rtol 1e-12."""
    g = dgl.graph((golden["large/u"], golden["large/v"]))
    x, e = golden["large/x"], golden["large/e"]
    close(ops.u_mul_e_sum(g, x, e), golden["large/u_mul_e_sum"], atol=1e-12)
    np.testing.assert_array_equal(ops.u_mul_e_max(g, x, e), golden["large/u_mul_e_max"])
    np.testing.assert_array_equal(ops.copy_u_min(g, x), golden["large/copy_u_min"])
    close(ops.u_sub_e_mean(g, x, e), golden["large/u_sub_e_mean"], atol=1e-12)
    close(ops.edge_softmax(g, golden["large/logits"]), golden["large/esoft_dst"])
    close(ops.edge_softmax(g, golden["large/logits"], norm_by="src"), golden["large/esoft_src"])
    close(ops.u_dot_e(g, x, e), golden["large/u_dot_e"], atol=1e-12)


def test_empty_graph():
    empty = np.array([], dtype=np.int64)
    g = dgl.graph((empty, empty))
    assert g.num_nodes() == 0
    assert ops.u_mul_e_sum(g, np.zeros((0, 4)), np.zeros((0, 4))).shape == (0, 4)
    assert ops.edge_softmax(g, np.zeros((0, 1))).shape == (0, 1)
