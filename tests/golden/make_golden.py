"""Generate tests/golden/ref_cases.npz from the reference's own Python package.

Run here (where the reference checkout exists), never on the GPU box:

    python tests/golden/make_golden.py /path/to/mojo-dgl

It imports lee101/mojo-dgl's ``python/mojodgl`` package and points its
``MOJODGL_LIB`` override at ``oracle/_build/libported_ref.so`` -- the C
restatement of ``src/ported.mojo`` exported under the reference's own eleven
``mdgl_*`` symbols (the Mojo toolchain that builds the real library is not in
this image).  Every host-side step -- ``reshape_lhs_rhs``/``_flat``/
``_broadcast``, CSR build by stable argsort, the ``update_all`` fusion rules,
segment mean/inf post-processing, the positional-``eids`` CSR rebuild,
``gather_mm``'s route choice -- is therefore the reference's own code, and only
the kernels are the restatement.  The cases follow the parametrisations of the
reference's tests/test_ops.py, tests/test_function.py,
tests/test_edge_softmax_eids.py and tests/test_parallel.py (same seeds, same
shapes), so the fixtures stand in for the reference suite on a box without it.
"""

from __future__ import annotations

import itertools
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str) -> None:
    sys.path.insert(0, REPO)
    from oracle import oracle as orc

    os.environ["MOJODGL_LIB"] = orc.build()
    sys.path.insert(0, os.path.join(ref_root, "python"))
    import mojodgl as dgl  # the reference package
    import mojodgl.function as fn
    import mojodgl.ops as ops

    assert os.path.realpath(dgl._lib.LIB) == os.path.realpath(orc.LIB_PATH)
    gm_mod = sys.modules["mojodgl.ops.gather_mm"]

    cases = {}

    def put(name, **arrays):
        for k, v in arrays.items():
            cases["{}/{}".format(name, k)] = np.asarray(v)

    # tests/upstream.py:33-37 + tests/test_ops.py:69-76
    rng0 = np.random.default_rng(0)
    U = rng0.integers(0, 64, size=512).astype(np.int64)
    V = rng0.integers(0, 64, size=512).astype(np.int64)
    N = 64
    G = dgl.graph((U, V))
    rng = np.random.default_rng(7)
    X = rng.normal(size=(N, 8))
    E = rng.normal(size=(len(U), 8))
    Y1 = rng.normal(size=(N, 1))
    put("graph0", u=U, v=V, x=X, e=E, y1=Y1,
        indptr=G._in_csr()[0], in_indices=G._in_csr()[1], in_order=G._in_csr()[2],
        outptr=G._out_csr()[0], out_indices=G._out_csr()[1], out_order=G._out_csr()[2],
        indeg=G.in_degrees(), outdeg=G.out_degrees())

    for bop, red in itertools.product(["add", "sub", "mul", "div"], ["sum", "max", "min", "mean"]):
        name = "u_{}_e_{}".format(bop, red)
        put("spmm/" + name, out=getattr(ops, name)(G, X, E))
    for src, red in itertools.product(["copy_u", "copy_e"], ["sum", "max", "min", "mean"]):
        name = "{}_{}".format(src, red)
        put("spmm/" + name, out=getattr(ops, name)(G, X if src == "copy_u" else E))
    put("spmm/u_add_e_sum_bcast", out=ops.u_add_e_sum(G, Y1, E))

    for (lt, rt), bop in itertools.product(itertools.permutations("uve", 2),
                                           ["add", "sub", "mul", "div", "dot"]):
        name = "{}_{}_{}".format(lt, bop, rt)
        data = {"u": X, "v": X, "e": E}
        put("sddmm/" + name, out=getattr(ops, name)(G, data[lt], data[rt]))
    put("sddmm/copy_lhs", out=ops.gsddmm(G, "copy_lhs", X, None))
    put("sddmm/copy_rhs_y1", out=ops.gsddmm(G, "copy_rhs", None, Y1))
    put("sddmm/copy_u", out=ops.copy_u(G, X))
    put("sddmm/copy_v", out=ops.copy_v(G, X))

    # every feature width (tests/test_ops.py:294-335)
    wr = np.random.default_rng(70)
    for d in [1, 2, 3, 5, 7, 8, 16, 33]:
        x = wr.normal(size=(N, d))
        e = wr.normal(size=(len(U), d))
        put("width{}".format(d), x=x, e=e,
            u_add_e_sum=ops.u_add_e_sum(G, x, e), u_div_e_min=ops.u_div_e_min(G, x, e),
            u_mul_e_mean=ops.u_mul_e_mean(G, x, e), copy_u_max=ops.copy_u_max(G, x),
            copy_e_sum=ops.copy_e_sum(G, e), u_mul_v=ops.u_mul_v(G, x, x),
            u_add_e=ops.u_add_e(G, x, e), u_dot_e=ops.u_dot_e(G, x, e))

    # segment ops (tests/test_ops.py:133-181, 324-359; tests/test_function.py:197-207)
    seglen = np.array([3, 0, 5, 4, 2])
    value = np.arange(14 * 3, dtype=np.float64).reshape(14, 3)
    for red in ["sum", "max", "min", "mean"]:
        put("segred/arange/" + red, out=ops.segment_reduce(seglen, value, red))
    put("segred/arange", seglen=seglen, value=value)
    sr = np.random.default_rng(71)
    for d in [1, 3, 5, 8, 33]:
        val = sr.normal(size=(14, d))
        put("segred/w{}".format(d), value=val,
            **{red: ops.segment_reduce(seglen, val, red) for red in ["sum", "max", "min", "mean"]})
    for i, sl in enumerate([[1, 0, 5, 4], [0, 0, 14], [2] * 7, [14]]):
        for d in [1, 3, 4, 32]:
            sl_ = np.asarray(sl, dtype=np.int64)
            val = sr.normal(size=(int(sl_.sum()), d))
            put("segsoft/{}/{}".format(i, d), seglen=sl_, value=val,
                out=ops.segment_softmax(sl_, val))
    seg10 = np.array([1, 0, 5, 4])
    put("segsoft/arange", seglen=seg10, value=np.arange(10.0).reshape(10, 1),
        out=ops.segment_softmax(seg10, np.arange(10.0).reshape(10, 1)))

    # segment_mm / gather_mm (tests/test_ops.py:155-170, 361-413)
    a = np.arange(18 * 4, dtype=np.float64).reshape(18, 4)
    b = np.arange(4 * 4 * 3, dtype=np.float64).reshape(4, 4, 3)
    put("segmm/arange", a=a, b=b, seglen=np.array([10, 5, 0, 3]),
        out=ops.segment_mm(a, b, np.array([10, 5, 0, 3])))
    mr = np.random.default_rng(72)
    for d2 in [1, 3, 4, 5, 8, 9]:
        a = mr.normal(size=(18, 5))
        b = mr.normal(size=(4, 5, d2))
        put("segmm/d2_{}".format(d2), a=a, b=b, out=ops.segment_mm(a, b, np.array([10, 5, 0, 3])))
        a = mr.normal(size=(300, 5))
        b = mr.normal(size=(7, 5, d2))
        idx = mr.integers(0, 7, size=300).astype(np.int64)
        put("gathermm/d2_{}".format(d2), a=a, b=b, idx=idx, out=ops.gather_mm(a, b, idx_b=idx))
    a = np.arange(6 * 4, dtype=np.float64).reshape(6, 4)
    b = np.arange(5 * 4 * 3, dtype=np.float64).reshape(5, 4, 3)
    idx = np.array([0, 3, 1, 1, 4, 2], dtype=np.int64)
    put("gathermm/arange", a=a, b=b, idx=idx, out=ops.gather_mm(a, b, idx_b=idx))
    r3 = np.random.default_rng(3)
    a = r3.normal(size=(1200, 9))
    b = r3.normal(size=(6, 9, 7))
    idx = r3.integers(0, 6, size=1200).astype(np.int64)
    saved = gm_mod._SEGMENT_BLOCK
    gm_mod._SEGMENT_BLOCK = 0
    put("gathermm/segment_route", a=a, b=b, idx=idx, out=ops.gather_mm(a, b, idx_b=idx))
    gm_mod._SEGMENT_BLOCK = saved

    # edge_softmax (tests/test_ops.py:184-218; tests/test_edge_softmax_eids.py)
    er = np.random.default_rng(73)
    lg = er.normal(size=(len(U), 1))
    put("esoft/logits1", logits=lg)
    for nb in ["dst", "src"]:
        put("esoft/" + nb, out=ops.edge_softmax(G, lg, norm_by=nb))
        for h in [1, 3, 8]:
            lh = er.normal(size=(len(U), h, 1))
            put("esoft/{}/h{}".format(nb, h), logits=lh, out=ops.edge_softmax(G, lh, norm_by=nb))
    eids = np.array([0, 5, 17, 30, 100, 511], dtype=np.int64)
    put("esoft/subset", eids=eids, out=ops.edge_softmax(G, lg, eids=eids))
    lh4 = er.normal(size=(len(U), 4, 1))
    put("esoft/subset_h4", logits=lh4, out=ops.edge_softmax(G, lh4, eids=eids))
    eid_rng = np.random.default_rng(2024)
    for case in range(40):
        nn_ = int(eid_rng.integers(2, 40))
        ne_ = int(eid_rng.integers(1, 120))
        u_ = eid_rng.integers(0, nn_, size=ne_).astype(np.int64)
        v_ = eid_rng.integers(0, nn_, size=ne_).astype(np.int64)
        g_ = dgl.graph((u_, v_))
        l_ = eid_rng.normal(size=(ne_, 1))
        size = int(eid_rng.integers(1, ne_ + 1))
        ei = eid_rng.choice(ne_, size=size, replace=False).astype(np.int64)
        nb = "dst" if case % 2 == 0 else "src"
        put("esoft/rand{}".format(case), u=u_, v=v_, logits=l_, eids=ei,
            norm_by=np.array(nb), out=ops.edge_softmax(g_, l_, eids=ei, norm_by=nb))
    ei = np.array([4, 4, 9], dtype=np.int64)
    put("esoft/repeat", eids=ei, out=ops.edge_softmax(G, lg, eids=ei))

    # update_all / pull (tests/test_function.py:13-26, 60-170)
    r1 = np.random.default_rng(1)
    U1 = r1.integers(0, 48, size=400).astype(np.int64)
    V1 = r1.integers(0, 48, size=400).astype(np.int64)
    r11 = np.random.default_rng(11)
    X1 = r11.normal(size=(48, 6))
    E1 = r11.normal(size=(400, 6))
    put("fn", u=U1, v=V1, x=X1, e=E1)

    def pair():
        g = dgl.graph((U1, V1))
        g.ndata["x"] = X1
        g.edata["e"] = E1
        return g

    for name, red in itertools.product(["copy_u", "copy_e"], ["sum", "max", "min", "mean"]):
        g = pair()
        g.update_all(getattr(fn, name)("x" if name == "copy_u" else "e", "m"),
                     getattr(fn, red)("m", "h"))
        put("fn/{}_{}".format(name, red), h=g.ndata["h"])
    for (lt, rt), op in itertools.product(itertools.permutations("uve", 2),
                                          ["add", "sub", "mul", "div", "dot"]):
        name = "{}_{}_{}".format(lt, op, rt)
        for red in ["sum", "max"]:
            g = pair()
            g.update_all(getattr(fn, name)("e" if lt == "e" else "x", "e" if rt == "e" else "x",
                                           "m"), getattr(fn, red)("m", "h"))
            put("fn/{}/{}".format(name, red), h=g.ndata["h"])
    g = pair()
    g.update_all(lambda edges: {"m": edges.src["x"] * edges.data["e"] + 1.0}, fn.mean("m", "h"))
    put("fn/udf_msg_mean", h=g.ndata["h"])
    g = pair()
    g.update_all(fn.copy_u("x", "m"), fn.sum("m", "h"),
                 lambda nodes: {"h": nodes.data["h"] * 0.5 + 2.0})
    put("fn/apply", h=g.ndata["h"])
    g = pair()
    g.update_all(fn.u_mul_e("x", "e", "m"), lambda nodes: {"h": nodes.mailbox["m"] * 2.0})
    put("fn/udf_reduce", h=g.ndata["h"])
    targets = np.array([1, 5, 9, 40], dtype=np.int64)
    g = pair()
    g.pull(targets, fn.u_mul_e("x", "e", "m"), fn.sum("m", "h"),
           apply_node_func=lambda nodes: {"h": nodes.data["h"] + 1.0})
    put("fn/pull", targets=targets, h=g.ndata["h"])
    g = pair()
    g.pull(targets, lambda edges: {"m": edges.src["x"] * edges.data["e"] + 1.0}, fn.mean("m", "h"))
    put("fn/pull_udf", h=g.ndata["h"])

    # zero in-degree / empty graph (tests/test_ops.py:227-260, 452-457)
    zu = np.array([0, 1], dtype=np.int64)
    zv = np.array([1, 2], dtype=np.int64)
    zr = np.random.default_rng(74)
    zx = zr.normal(size=(5, 4))
    ze = zr.normal(size=(2, 4))
    gz = dgl.graph((zu, zv), num_nodes=5)
    put("zero", u=zu, v=zv, x=zx, e=ze, u_add_e_sum=ops.u_add_e_sum(gz, zx, ze),
        u_mul_e_mean=ops.u_mul_e_mean(gz, zx, ze), copy_u_max=ops.copy_u_max(gz, zx),
        copy_e_min=ops.copy_e_min(gz, ze))

    # a larger graph with a hub, both sides of PARALLEL_MIN (tests/test_parallel.py:42-111)
    rl = np.random.default_rng(5)
    nl, el_ = 5000, 12000
    ul = rl.integers(0, nl, size=el_).astype(np.int64)
    vl = rl.integers(0, nl, size=el_).astype(np.int64)
    vl[: 2500] = 17  # one destination with 2500+ in-edges
    xl = rl.normal(size=(nl, 3))
    elf = rl.normal(size=(el_, 3))
    gl = dgl.graph((ul, vl))
    lgl = rl.normal(size=(el_, 2, 1))
    put("large", u=ul, v=vl, x=xl, e=elf, logits=lgl,
        u_mul_e_sum=ops.u_mul_e_sum(gl, xl, elf), u_mul_e_max=ops.u_mul_e_max(gl, xl, elf),
        copy_u_min=ops.copy_u_min(gl, xl), u_sub_e_mean=ops.u_sub_e_mean(gl, xl, elf),
        esoft_dst=ops.edge_softmax(gl, lgl), esoft_src=ops.edge_softmax(gl, lgl, norm_by="src"),
        u_dot_e=ops.u_dot_e(gl, xl, elf))

    out = os.path.join(HERE, "ref_cases.npz")
    np.savez_compressed(out, **cases)
    print("wrote {} arrays to {} ({} bytes)".format(len(cases), out, os.path.getsize(out)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/mojo-dgl")
    main(sys.argv[1])
