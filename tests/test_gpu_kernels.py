"""GPU parity for the paths the fixtures do not reach: float32 (the B200
path), arg-index outputs, split rows, head broadcast, the device CSR build at
scale, torch inputs, determinism, and the reference-compatible mdgl_* ABI.

Tolerances (fixed by the build's specification):
  * float32 gSpMM/segment sums: |ours - ref| <= 1e-5 |ref| + 1e-5 S, where
    S = sum of |message| over the row (the oracle computes it), because a pure
    relative bound fails on cancellation near zero;
  * float32 element-wise/softmax: rtol 1e-5 (+ tiny atol);
  * TF32/BF16 tensor-core grouped GEMM: the same form with 1e-2;
  * max/min values and every integer output (arg indices, CSR): exact.
The oracle computes in float64 from the same float32 values.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import mojodgl as dgl  # noqa: E402
import mojodgl.ops as ops  # noqa: E402
from mojodgl import _lib  # noqa: E402


def within_s(got, ref, s, tol=1e-5):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    bound = tol * np.abs(ref) + tol * s + 1e-30
    bad = err > bound
    assert not bad.any(), "max excess {} at {}".format((err - bound).max(), np.argwhere(bad)[:5])


def rand_graph(n, e, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, n, e), rng.integers(0, n, e)


@pytest.fixture
def small_chunks():
    """Force merge-path chunks of ~16 items so rows longer than that split."""
    _lib.set_param("spmm_min_items", 16)
    _lib.set_param("spmm_max_chunks", 1 << 40)
    _lib.set_param("spmm_split_min", 0)
    yield
    _lib.set_param("spmm_min_items", 32)
    _lib.set_param("spmm_max_chunks", 0)
    _lib.set_param("spmm_split_min", 512)


def test_config1_update_all_u_mul_e_sum(orc):
    """BASELINE config 1 (N=10k, E=200k, D=64, seed 0), float32, through
    g.update_all(fn.u_mul_e, fn.sum) -- the minimum end-to-end slice."""
    import mojodgl.function as fn

    rng = np.random.default_rng(0)
    n, e = 10_000, 200_000
    u = rng.integers(0, n, e)
    v = rng.integers(0, n, e)
    h = rng.normal(size=(n, 64)).astype(np.float32)
    ef = rng.normal(size=(e, 64)).astype(np.float32)
    g = dgl.graph((u, v))
    g.ndata["h"] = h
    g.edata["e"] = ef
    g.update_all(fn.u_mul_e("h", "e", "m"), fn.sum("m", "z"))
    z = g.ndata["z"]
    assert z.dtype == np.float32
    og = orc.Graph(u, v)
    ref = orc.gspmm(og, "mul", "sum", h, ef)
    within_s(z, ref, orc.gspmm_abs_bound(og, "mul", h, ef))
    # the float64 run of the same inputs is bit-identical to the oracle
    z64 = ops.u_mul_e_sum(g, h.astype(np.float64), ef.astype(np.float64))
    np.testing.assert_array_equal(z64, ref)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "copy_lhs", "copy_rhs"])
@pytest.mark.parametrize("red", ["sum", "max", "min", "mean"])
def test_gspmm_float32(orc, op, red):
    u, v = rand_graph(3000, 40_000, 11)
    rng = np.random.default_rng(12)
    x = rng.normal(size=(3000, 12)).astype(np.float32)
    e = (rng.normal(size=(40_000, 12)) + 3.0).astype(np.float32)
    g, og = dgl.graph((u, v)), orc.Graph(u, v)
    lhs = None if op == "copy_rhs" else x
    rhs = None if op == "copy_lhs" else e
    got = ops.gspmm(g, op, red, lhs, rhs)
    assert got.dtype == np.float32
    if red in ("max", "min"):
        if op in ("copy_lhs", "copy_rhs"):
            np.testing.assert_array_equal(got, orc.gspmm(og, op, red, lhs, rhs))
        else:  # the fp32 message equals the fp64 one rounded to fp32
            ref = orc.gspmm(og, op, red, lhs, rhs)
            np.testing.assert_allclose(got, ref, rtol=1e-6)
        return
    ref = orc.gspmm(og, op, red, lhs, rhs)
    s = orc.gspmm_abs_bound(og, op, lhs, rhs)
    if red == "mean":
        s = s / np.maximum(og.indeg, 1)[:, None]
    within_s(got, ref, s)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("red", ["max", "min"])
def test_arg_indices_exact(orc, dtype, red):
    u, v = rand_graph(2000, 30_000, 21)
    rng = np.random.default_rng(22)
    # few distinct values: plenty of ties, which the first-in-CSR-order rule settles
    x = rng.integers(-3, 4, size=(2000, 8)).astype(dtype)
    e = rng.integers(-3, 4, size=(30_000, 8)).astype(dtype)
    g, og = dgl.graph((u, v)), orc.Graph(u, v)
    for op, lhs, rhs in (("copy_lhs", x, None), ("copy_rhs", None, e), ("mul", x, e), ("sub", x, e)):
        out, (au, ae) = ops.spmm._gspmm(g, op, red, lhs, rhs)
        ref, ru, re_ = orc.gspmm(og, op, red, lhs, rhs, with_arg=True)
        np.testing.assert_array_equal(out, ref)
        if au is not None:
            np.testing.assert_array_equal(au, ru)
        if ae is not None:
            np.testing.assert_array_equal(ae, re_)


def power_law(n, seed, mean_deg=12, cap=3000):
    rng = np.random.default_rng(seed)
    w = np.minimum(rng.zipf(2.1, n), cap).astype(np.float64)
    deg = np.floor(w / w.sum() * n * mean_deg).astype(np.int64)
    v = np.repeat(np.arange(n), deg)
    u = rng.integers(0, n, v.size)
    p = rng.permutation(v.size)
    return u[p], v[p]


def test_split_rows_float64_and_args(orc, small_chunks):
    u, v = power_law(4000, 31)
    rng = np.random.default_rng(32)
    x = rng.normal(size=(4000, 6))
    e = rng.normal(size=(u.size, 6))
    g, og = dgl.graph((u, v)), orc.Graph(u, v)
    assert og.indeg.max() > 200  # hubs span many 16-item chunks
    np.testing.assert_allclose(ops.u_mul_e_sum(g, x, e), orc.gspmm(og, "mul", "sum", x, e),
                               rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(ops.copy_u_mean(g, x), orc.gspmm(og, "copy_lhs", "mean", x, None),
                               rtol=1e-12, atol=1e-12)
    for red in ("max", "min"):
        out, (au, ae) = ops.spmm._gspmm(g, "add", red, x, e)
        ref, ru, re_ = orc.gspmm(og, "add", red, x, e, with_arg=True)
        np.testing.assert_array_equal(out, ref)
        np.testing.assert_array_equal(au, ru)
        np.testing.assert_array_equal(ae, re_)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("heads", [1, 8, 64, 130])
def test_edge_softmax_split_rows_both_paths(orc, small_chunks, dtype, heads):
    """Rows split over many merge-path chunks (chunks of ~16 items), for the
    lane walk (narrow rows: 1 and 8 columns) and the team walk (64 and 130
    columns, the latter in column blocks), norm_by dst and src."""
    u, v = power_law(3000, 37)
    rng = np.random.default_rng(38)
    z = (rng.normal(size=(u.size, heads, 1)) * 3).astype(dtype)
    g, og = dgl.graph((u, v)), orc.Graph(u, v)
    rtol = 2e-5 if dtype == np.float32 else 1e-12
    for norm_by in ("dst", "src"):
        got = ops.edge_softmax(g, z, norm_by=norm_by)
        want = orc.edge_softmax(og, z.astype(np.float64), norm_by=norm_by)
        np.testing.assert_allclose(got, want, rtol=rtol, atol=1e-7 if dtype == np.float32 else 0)


@pytest.fixture(params=[1, 0], ids=["segment-per-warp", "merge-path"])
def seg_mode(request):
    """segment_softmax's two schedules: one warp per segment (the default for
    rows of whole 16-byte vectors) and the merge-path passes."""
    _lib.set_param("softmax_segment_warp", request.param)
    yield request.param
    _lib.set_param("softmax_segment_warp", 1)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("d", [4, 8, 64, 128, 12])
def test_segment_softmax_schedules(orc, seg_mode, dtype, d):
    """Geometric segment lengths with empty segments, then the same with one
    segment longer than the per-warp bound (4,096 rows: it sends the call
    through the merge-path passes); widths whose rows are whole 16-byte
    vectors (4 .. 128 float32 columns) and one that is not (12)."""
    rng = np.random.default_rng(d)
    seglen = rng.geometric(1 / 24, size=3000)
    seglen[[5, 17, 400]] = 0
    rtol = 2e-5 if dtype == np.float32 else 1e-12
    atol = 1e-7 if dtype == np.float32 else 0
    for lens in (seglen, np.concatenate([seglen[:100], [5000], seglen[100:]])):
        v = (rng.normal(size=(int(lens.sum()), d)) * 3).astype(dtype)
        got = ops.segment_softmax(lens, v)
        want = orc.segment_softmax(lens, v)
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


@pytest.fixture(params=[16, 100, 1000], ids=["chunk16", "chunk100", "chunk1000"])
def chunk_items(request):
    """Merge-path chunks of a fixed size: 16 gives the lane walk's runs (32 /
    L per warp, L lanes a run) about one item each, 100 a few, 1000 dozens."""
    _lib.set_param("spmm_min_items", request.param)
    _lib.set_param("spmm_max_chunks", 1 << 40)
    _lib.set_param("spmm_split_min", 0)
    yield request.param
    _lib.set_param("spmm_min_items", 32)
    _lib.set_param("spmm_max_chunks", 0)
    _lib.set_param("spmm_split_min", 512)


@pytest.mark.parametrize("dtype,heads", [(np.float32, h) for h in (1, 3, 8, 12, 16, 32)]
                         + [(np.float64, h) for h in (1, 2, 5, 8, 16)])
def test_narrow_softmax_runs_and_chunks(orc, chunk_items, dtype, heads):
    """Items of at most 64 bytes take the lane walk (runs of L lanes, one per
    column vector, each run a stretch of consecutive items; split rows joined
    by a warp scan of run pieces; widths that are not a power-of-two count of
    vectors leave lanes idle); wider
    narrow rows (float32 x 32, float64 x 16) the warp-wide steps.  Hubs span
    many runs and chunks; isolated nodes leave empty rows.  Covers the three
    callers: edge_softmax over all edges (edge-order second pass), a positional
    subset of edge ids and segment_softmax (item-order second pass)."""
    u, v = power_law(3000, 51)
    u = np.concatenate([u, [2999, 2999]])  # two nodes more, one isolated
    v = np.concatenate([v, [3001, 3001]])
    rng = np.random.default_rng(52)
    z = (rng.normal(size=(u.size, heads, 1)) * 3).astype(dtype)
    g, og = dgl.graph((u, v), num_nodes=3003), orc.Graph(u, v, 3003)
    rtol = 2e-5 if dtype == np.float32 else 1e-12
    atol = 1e-7 if dtype == np.float32 else 0
    for norm_by in ("dst", "src"):
        got = ops.edge_softmax(g, z, norm_by=norm_by)
        want = orc.edge_softmax(og, z.astype(np.float64), norm_by=norm_by)
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)
    sel = rng.permutation(u.size)[: u.size // 2]
    got = ops.edge_softmax(g, z, eids=sel)
    want = orc.edge_softmax(og, z.astype(np.float64), eids=sel)
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)
    seglen = np.bincount(v, minlength=3003)
    val = z.reshape(u.size, heads)
    np.testing.assert_allclose(ops.segment_softmax(seglen, val),
                               orc.segment_softmax(seglen, val.astype(np.float64)),
                               rtol=rtol, atol=atol)


def test_split_rows_are_deterministic(small_chunks):
    u, v = power_law(5000, 41)
    x = np.random.default_rng(42).normal(size=(5000, 64)).astype(np.float32)
    g = dgl.graph((u, v))
    a = ops.copy_u_sum(g, x)
    b = ops.copy_u_sum(g, x)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("split", [False, True])
def test_float32_mean_is_the_correctly_rounded_sum_over_degree(split, request):
    """copy_u_mean divides each row's float32 sum by its in-degree once, so it
    must equal copy_u_sum's output divided by the degree in IEEE float32 bit
    for bit -- degrees 0..4000 and a few hundred thousand, values from 2^-110
    to 2^110, zeros, inf and NaN."""
    if split:
        request.getfixturevalue("small_chunks")
    rng = np.random.default_rng(91)
    deg = np.concatenate([np.arange(4001), rng.integers(4001, 300_000, 12),
                          [65536, 65537, 131071]])
    n = deg.size
    v = np.repeat(np.arange(n), deg)
    u = rng.integers(0, 2048, v.size)
    x = rng.normal(size=(n, 64)) * np.exp2(rng.integers(-40, 41, size=(n, 1)))
    x[:64] = rng.normal(size=(64, 64)) * 2.0 ** -110
    x[64:128] = rng.normal(size=(64, 64)) * 2.0 ** 110
    x[128, :8] = 0.0
    x[129, 8] = np.inf
    x[130, 9] = np.nan
    x = x.astype(np.float32)
    g = dgl.graph((u, v), num_nodes=n)
    s = ops.copy_u_sum(g, x)
    m = ops.copy_u_mean(g, x)
    want = s / np.maximum(deg, 1).astype(np.float32)[:, None]
    assert want.dtype == np.float32
    np.testing.assert_array_equal(m, want)


def test_host_result_sliced_path_matches_device_path():
    """A host-bound result of 64 MB or more is computed in destination-row
    slices whose rows are copied back while the next slice runs; it must
    match the device-resident call: max/min bit for bit, sum/mean within the
    float32 gSpMM bound (a hub row may be split at other chunk boundaries)."""
    u, v = power_law(200_000, 91, mean_deg=8)
    rng = np.random.default_rng(92)
    x = rng.normal(size=(200_000, 128)).astype(np.float32)
    w = rng.normal(size=(u.size, 128)).astype(np.float32)
    g = dgl.graph((u, v), num_nodes=200_000)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    for red in ("sum", "mean", "max", "min"):
        got = ops.gspmm(g, "copy_lhs", red, x, None)
        assert isinstance(got, np.ndarray) and got.shape == (200_000, 128)
        want = ops.gspmm(g, "copy_lhs", red, xd, None).cpu().numpy()
        if red in ("max", "min"):
            np.testing.assert_array_equal(got, want)
        else:
            s = ops.gspmm(g, "copy_lhs", "sum" if red == "sum" else "mean", np.abs(x), None)
            within_s(got, want.astype(np.float64), s)
    got = ops.gspmm(g, "mul", "max", torch.from_numpy(x), torch.from_numpy(w))
    assert isinstance(got, torch.Tensor) and got.is_pinned()
    np.testing.assert_array_equal(got.numpy(), ops.gspmm(g, "mul", "max", xd, wd).cpu().numpy())


def test_head_broadcast_gat_layer(orc):
    """BASELINE config 2's pipeline at a small size: u_add_v on (N, H, 1),
    leaky_relu, edge_softmax over (E, H, 1), u_mul_e_sum of (N, H, D) by
    (E, H, 1) -- the head broadcast read in place, no np.repeat."""
    u, v = power_law(3000, 51)
    rng = np.random.default_rng(52)
    H, D = 8, 16
    el = rng.normal(size=(3000, H, 1)).astype(np.float32)
    er = rng.normal(size=(3000, H, 1)).astype(np.float32)
    feat = rng.normal(size=(3000, H, D)).astype(np.float32)
    g, og = dgl.graph((u, v)), orc.Graph(u, v)
    s = ops.u_add_v(g, el, er)
    assert s.shape == (u.size, H, 1)
    s_ref = orc.gsddmm(og, "add", el, er, "u", "v")
    np.testing.assert_allclose(s, s_ref, rtol=1e-6)
    a = np.where(s > 0, s, np.float32(0.2) * s)
    att = ops.edge_softmax(g, a)
    att_ref = orc.edge_softmax(og, a.astype(np.float64))
    np.testing.assert_allclose(att, att_ref, rtol=2e-5, atol=1e-7)
    out = ops.u_mul_e_sum(g, feat, att)
    assert out.shape == (3000, H, D)
    ref = orc.gspmm(og, "mul", "sum", feat, att)
    sb = orc.gspmm_abs_bound(og, "mul", feat, att)
    within_s(out.reshape(3000, -1), ref.reshape(3000, -1), sb.reshape(3000, -1))


def test_csr_build_bit_exact_at_scale():
    n, e = 300_000, 3_000_000
    u, v = rand_graph(n, e, 61)
    v[:500_000] = 7  # a very heavy destination
    g = dgl.graph((u, v))
    ip, nbr, order = g._in_csr()
    want = np.argsort(v, kind="stable")
    np.testing.assert_array_equal(order, want)
    np.testing.assert_array_equal(nbr, u[want])
    np.testing.assert_array_equal(ip[1:], np.cumsum(np.bincount(v, minlength=n)))
    op, onbr, oorder = g._out_csr()
    np.testing.assert_array_equal(oorder, np.argsort(u, kind="stable"))
    np.testing.assert_array_equal(g.out_degrees(), np.bincount(u, minlength=n))


def test_torch_cuda_inputs_stay_on_device(orc):
    u, v = rand_graph(1000, 8000, 71)
    x = torch.randn(1000, 32, device="cuda")
    g = dgl.graph((torch.from_numpy(u).cuda(), torch.from_numpy(v).cuda()))
    out = ops.copy_u_sum(g, x)
    assert isinstance(out, torch.Tensor) and out.is_cuda and out.dtype == torch.float32
    g2 = dgl.graph((u, v))
    np.testing.assert_array_equal(out.cpu().numpy(), ops.copy_u_sum(g2, x.cpu().numpy()))
    deg = g.in_degrees()
    assert isinstance(deg, torch.Tensor)
    np.testing.assert_array_equal(deg.cpu().numpy(), np.bincount(v, minlength=1000))


def test_segment_ops_float32(orc):
    rng = np.random.default_rng(81)
    seglen = rng.geometric(1 / 32, size=3000)
    seglen[::17] = 0
    n = int(seglen.sum())
    val = rng.normal(size=(n, 64)).astype(np.float32)
    ref_sum = orc.segment_reduce(seglen, val, "sum")
    s = orc.segment_reduce(seglen, np.abs(val), "sum")
    within_s(ops.segment_reduce(seglen, val, "sum"), ref_sum, s)
    np.testing.assert_array_equal(ops.segment_reduce(seglen, val, "max"),
                                  orc.segment_reduce(seglen, val, "max"))
    soft = ops.segment_softmax(seglen, val)
    np.testing.assert_allclose(soft, orc.segment_softmax(seglen, val), rtol=2e-5, atol=1e-7)


def test_grouped_mm_float32(orc):
    rng = np.random.default_rng(91)
    r, d1, d2 = 6, 64, 48
    seglen = rng.multinomial(5000, rng.dirichlet(0.5 * np.ones(r)))
    a = rng.normal(0, 0.05, size=(5000, d1)).astype(np.float32)
    b = rng.normal(0, 0.05, size=(r, d1, d2)).astype(np.float32)
    ref = orc.segment_mm(a, b, seglen)
    sbound = orc.segment_mm(np.abs(a), np.abs(b), seglen)
    within_s(ops.segment_mm(a, b, seglen), ref, sbound, tol=1e-2)
    idx = rng.integers(0, r, 5000)
    ref = orc.gather_mm(a, b, idx)
    sbound = orc.gather_mm(np.abs(a), np.abs(b), idx)
    within_s(ops.gather_mm(a, b, idx_b=idx), ref, sbound, tol=1e-2)


# ------------------------------------------------- reference-compatible ABI
def _addr(a):
    return a.ctypes.data


def test_compat_abi_matches_the_oracle(orc):
    """The mdgl_* symbols called exactly as the reference's Python layer
    calls them (python/mojodgl/ops/*.py), on host float64 buffers."""
    L = _lib.lib()
    O = orc.lib()
    u, v = rand_graph(500, 6000, 101)
    og = orc.Graph(u, v)
    rng = np.random.default_rng(102)
    x, e = rng.normal(size=(500, 7)), rng.normal(size=(6000, 7))
    indptr, indices, eid = og.in_csr()
    for red in range(4):
        a = np.empty((500, 7))
        b = np.empty((500, 7))
        args = (_addr(indptr), _addr(indices), _addr(eid), _addr(x), _addr(e))
        L.mdgl_gspmm(*args, _addr(a), 500, 2, 7, 7, 7, red, _addr(og.indeg))
        O.mdgl_gspmm(*args, _addr(b), 500, 2, 7, 7, 7, red, _addr(og.indeg))
        np.testing.assert_array_equal(a, b)
    a, b = np.empty((6000, 1)), np.empty((6000, 1))
    for lib_, out in ((L, a), (O, b)):
        lib_.mdgl_gsddmm(_addr(og.u), _addr(og.v), _addr(x), _addr(e), _addr(out), 6000, 0, 2, 4, 7, 7, 1)
    np.testing.assert_allclose(a, b, rtol=1e-12)
    off = np.array([0, 3, 3, 10, 14, 14], dtype=np.int64)
    val = rng.normal(size=(14, 5))
    for red in range(3):
        a, b = np.empty((5, 5)), np.empty((5, 5))
        L.mdgl_segment_reduce(_addr(off), _addr(val), _addr(a), 5, 5, red, 14)
        O.mdgl_segment_reduce(_addr(off), _addr(val), _addr(b), 5, 5, red, 14)
        np.testing.assert_array_equal(a, b)
    scratch = np.empty(32 * 2 * 5)
    a, b = np.zeros((14, 5)), np.zeros((14, 5))
    L.mdgl_segment_softmax(_addr(off), _addr(val), _addr(a), _addr(scratch), 5, 5, 14)
    O.mdgl_segment_softmax(_addr(off), _addr(val), _addr(b), _addr(scratch), 5, 5, 14)
    np.testing.assert_allclose(a, b, rtol=1e-12)
    logit = rng.normal(size=(6000, 2))
    mask = np.ones(1, dtype=np.int8)
    scratch = np.empty(32 * 2 * 2)
    a, b = np.empty((6000, 2)), np.empty((6000, 2))
    for lib_, out in ((L, a), (O, b)):
        lib_.mdgl_edge_softmax_(_addr(indptr), _addr(indices), _addr(eid), _addr(mask), _addr(logit),
                                _addr(out), _addr(scratch), 500, 1, 2)
    np.testing.assert_allclose(a, b, rtol=1e-12)
    am, bm = rng.normal(size=(40, 5)), rng.normal(size=(3, 5, 4))
    seg = np.array([10, 0, 30], dtype=np.int64)
    a, b = np.zeros((40, 4)), np.zeros((40, 4))
    L.mdgl_segment_mm(_addr(am), _addr(bm), _addr(a), _addr(seg), 40, 5, 3, 4)
    O.mdgl_segment_mm(_addr(am), _addr(bm), _addr(b), _addr(seg), 40, 5, 3, 4)
    np.testing.assert_array_equal(a, b)
    idx = rng.integers(0, 3, 40).astype(np.int64)
    a, b = np.empty((40, 4)), np.empty((40, 4))
    L.mdgl_gather_mm(_addr(am), _addr(bm), _addr(idx), _addr(a), 40, 5, 4)
    O.mdgl_gather_mm(_addr(am), _addr(bm), _addr(idx), _addr(b), 40, 5, 4)
    np.testing.assert_array_equal(a, b)
    src = np.array([3, 1, 4, 1, 5], dtype=np.int64)
    a, b = np.zeros(5, np.int64), np.zeros(5, np.int64)
    L.mdgl_cumsum(_addr(src), _addr(a), 5)
    O.mdgl_cumsum(_addr(src), _addr(b), 5)
    np.testing.assert_array_equal(a, b)
    L.mdgl_clamp_i64(_addr(src), _addr(a), 5, 2, 4)
    np.testing.assert_array_equal(a, np.clip(src, 2, 4))
    f = np.array([1.0, np.inf, -np.inf, -2.0])
    a = np.empty(4)
    L.mdgl_replace_inf_with_zero(_addr(f), _addr(a), 4)
    np.testing.assert_array_equal(a, [1.0, 0.0, 0.0, -2.0])
    assert L.bgl_last_error() == b""


@pytest.mark.parametrize("red", ["sum", "mean", "max", "min"])
def test_accumulate_passes_match_one_pass(orc, red):
    """BGL_ACCUMULATE: the aggregation run as P passes, one per source-owner
    block (as the multi-GPU halo delivers them), equals the single pass --
    float64 sums to rtol 1e-12, max/min and their edge ids exactly."""
    import torch

    L = _lib.lib()
    u, v = power_law(6000, 91)
    rng = np.random.default_rng(92)
    n, d, P = 6000, 8, 3
    x = rng.integers(-4, 5, size=(n, d)).astype(np.float64) + rng.normal(size=(n, d)) * (red in ("sum", "mean"))
    blk = (n + P - 1) // P
    dev = torch.device("cuda")
    code = _lib.REDUCERS[red]
    out = torch.empty((n, d), dtype=torch.float64, device=dev)
    arg_e = torch.empty((n, d), dtype=torch.int64, device=dev)
    deg = torch.from_numpy(np.bincount(v, minlength=n).astype(np.int64)).to(dev)
    xs = torch.from_numpy(x).to(dev)
    for p in range(P):
        m = np.nonzero(u // blk == p)[0]
        order = m[np.argsort(v[m], kind="stable")]
        indptr = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(np.bincount(v[m], minlength=n), out=indptr[1:])
        t_ip = torch.from_numpy(indptr).to(dev)
        t_nbr = torch.from_numpy((u[order] - p * blk).astype(np.int32)).to(dev)
        t_eid = torch.from_numpy(order.astype(np.int32)).to(dev)
        feat = xs[p * blk: (p + 1) * blk].contiguous()
        r = _lib.REDUCE_SUM if (red == "mean" and p < P - 1) else code
        flags = (_lib.BGL_ACCUMULATE if p else 0) | (
            _lib.BGL_ZERO_INF if (p == P - 1 and red in ("max", "min")) else 0)
        nb = L.bgl_gspmm_workspace_size(n, m.size, d, _lib.BGL_F64, r)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
        rc = L.bgl_gspmm(t_ip.data_ptr(), t_nbr.data_ptr(), t_eid.data_ptr(), deg.data_ptr(), n,
                         m.size, feat.data_ptr(), d, 1, None, 1, 1, out.data_ptr(), d, None,
                         arg_e.data_ptr() if red in ("max", "min") else None, _lib.BGL_F64,
                         _lib.OP_COPY_LHS, r, flags, ws.data_ptr(), nb,
                         torch.cuda.current_stream().cuda_stream)
        assert rc == 0, L.bgl_last_error()
    torch.cuda.synchronize()
    og = orc.Graph(u, v, num_nodes=n)
    if red in ("max", "min"):
        want, _, want_e = orc.gspmm(og, "copy_lhs", red, x, None, with_arg=True)
        want = orc.replace_inf_with_zero(want)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        np.testing.assert_array_equal(arg_e.cpu().numpy(), want_e)
    else:
        np.testing.assert_allclose(out.cpu().numpy(), orc.gspmm(og, "copy_lhs", red, x, None),
                                   rtol=1e-12, atol=1e-12)


def test_check_csr_counts_bad_row_pointers_and_ids():
    """bgl_check_csr on a valid CSR reports nothing; with planted faults (a
    neighbour id past the source count, a negative edge id, a decreasing row
    pointer and a wrong last pointer) it counts each and names the first bad
    position.  Only the validator reads the faulty arrays."""
    lib = _lib.lib()
    rng = np.random.default_rng(91)
    n, ne, nsrc = 500, 8000, 700
    v = np.sort(rng.integers(0, n, ne))
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.bincount(v, minlength=n), out=indptr[1:])
    indices = rng.integers(0, nsrc, ne).astype(np.int32)
    eid = rng.permutation(ne).astype(np.int32)
    res = torch.zeros(3, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def check(ip, ind, ed):
        t = [torch.from_numpy(x).cuda() for x in (ip, ind, ed)]
        rc = lib.bgl_check_csr(t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), n, ne, nsrc,
                               ne, res.data_ptr(), stream)
        assert rc == 0, lib.bgl_last_error()
        return res.cpu().tolist()

    assert check(indptr, indices, eid) == [0, 0, -1]
    bad_ind, bad_eid, bad_ptr = indices.copy(), eid.copy(), indptr.copy()
    bad_ind[4321] = nsrc + 5
    bad_eid[777] = -3
    bad_ptr[100] = bad_ptr[101] + 1  # indptr[100] > indptr[101]
    bad_ptr[n] = ne + 1
    assert check(bad_ptr, bad_ind, bad_eid) == [2, 2, 777]
