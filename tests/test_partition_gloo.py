"""Multi-rank host logic of the destination-row partition, on CPU gloo ranks.

Two ranks split a power-law graph by destination rows (balanced by in-edges),
own equal blocks of the node features, all-gather them (the halo), and each
reduces its own rows with the oracle's copy_u_mean.  The stitched result must
equal the single-process result bit for bit: a shard keeps the global edge
order, so every row folds its messages in the same order.  No GPU is used;
the kernels' own multi-GPU run is the bench's N>1 path.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mojodgl.partition import (DstShard, assemble_gathered, edge_balanced_ranges, owner_blocks,
                               ring_exchange)


def graph(seed=5, n=3000):
    rng = np.random.default_rng(seed)
    w = np.minimum(rng.zipf(2.1, n), 2000).astype(np.float64)
    deg = np.floor(w / w.sum() * n * 10).astype(np.int64)
    v = np.repeat(np.arange(n), deg)
    u = rng.integers(0, n, v.size)
    p = rng.permutation(v.size)
    h = rng.normal(size=(n, 6))
    return u[p], v[p], h, n


def test_edge_balanced_ranges_cover_and_balance():
    u, v, h, n = graph()
    indeg = np.bincount(v, minlength=n)
    for parts in (1, 2, 3, 8):
        b = edge_balanced_ranges(indeg, parts)
        assert b[0] == 0 and b[-1] == n and np.all(np.diff(b) >= 0)
        per = [indeg[b[i]:b[i + 1]].sum() for i in range(parts)]
        assert sum(per) == v.size
        assert max(per) <= v.size / parts + indeg.max()


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_pull_order_is_a_rotation(world):
    """Every rank pulls every peer block once, and at each position of the
    order the ranks read distinct peers."""
    from mojodgl.partition import pull_order

    orders = [pull_order(r, world) for r in range(world)]
    for r, o in enumerate(orders):
        assert sorted(o) == [q for q in range(world) if q != r]
    for k in range(world - 1):
        assert len({o[k] for o in orders}) == world


def test_owner_blocks_tile_the_rows():
    blk, owners = owner_blocks(10, 4)
    assert blk == 3 and owners == [(0, 3), (3, 6), (6, 9), (9, 10)]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import oracle as orc

        u, v, h, n = graph()
        bounds = edge_balanced_ranges(np.bincount(v, minlength=n), world)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        shard = DstShard(u, v, lo, hi)
        blk, owners = owner_blocks(n, world)
        a, b = owners[rank]
        mine = torch.zeros(blk, h.shape[1], dtype=torch.float64)
        mine[: b - a] = torch.from_numpy(h[a:b])
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        full = assemble_gathered([p.numpy() for p in parts], n)
        # the shard's rows: a graph over n source ids whose destinations are local
        og = orc.Graph(shard.u, shard.v_local, num_nodes=max(n, hi - lo))
        out = orc.gspmm(og, "copy_lhs", "mean", full, None)[: hi - lo]
        q.put((rank, lo, hi, out))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reproduce_the_single_process_result():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle as orc

    u, v, h, n = graph()
    want = orc.gspmm(orc.Graph(u, v, num_nodes=n), "copy_lhs", "mean", h, None)
    got = np.zeros_like(want)
    for _, lo, hi, out in results:
        got[lo:hi] = out
    np.testing.assert_array_equal(got, want)


def _ring_rank(rank, world, port, q):
    """The owner-pipelined halo: blocks arrive over the ring and each is
    reduced over the shard's edges whose sources it owns; sums add in owner
    order, max keeps the better value with the smaller edge id on a tie."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import oracle as orc

        u, v, h, n = graph(seed=9)
        bounds = edge_balanced_ranges(np.bincount(v, minlength=n), world)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        blk, owners = owner_blocks(n, world)
        a, b = owners[rank]
        mine = torch.zeros(blk, h.shape[1], dtype=torch.float64)
        mine[: b - a] = torch.from_numpy(h[a:b])
        sel = np.nonzero((v >= lo) & (v < hi))[0]
        sums = np.zeros((hi - lo, h.shape[1]))
        best = np.full((hi - lo, h.shape[1]), -np.inf)
        best_e = np.full((hi - lo, h.shape[1]), -1, dtype=np.int64)
        seen = []

        def on_block(owner, block, first, last):
            seen.append(owner)
            m = sel[(u[sel] // blk) == owner]
            og = orc.Graph(u[m] - owner * blk, v[m] - lo, num_nodes=max(blk, hi - lo))
            x = block.numpy()
            part = orc.gspmm(og, "copy_lhs", "sum", x, None)[: hi - lo]
            sums[:] = part if first else sums + part
            mx, au, ae = orc.gspmm(og, "copy_lhs", "max", x, None, with_arg=True)
            mx, ae = mx[: hi - lo], ae[: hi - lo]
            ge = np.where(ae >= 0, m[np.maximum(ae, 0)], -1)  # global edge ids
            take = (mx > best) | ((mx == best) & (ge >= 0) & ((best_e < 0) | (ge < best_e)))
            best[take] = mx[take]
            best_e[take] = ge[take]

        ring_exchange(mine, None, rank, world, on_block)
        q.put((rank, lo, hi, sums, best, best_e, seen))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_halo_reproduces_the_single_process_result(world):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ring_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle as orc

    u, v, h, n = graph(seed=9)
    og = orc.Graph(u, v, num_nodes=n)
    want_sum = orc.gspmm(og, "copy_lhs", "sum", h, None)
    want_max, _, want_e = orc.gspmm(og, "copy_lhs", "max", h, None, with_arg=True)
    for rank, lo, hi, sums, best, best_e, seen in results:
        assert sorted(seen) == list(range(world)) and seen[0] == rank
        np.testing.assert_allclose(sums, want_sum[lo:hi], rtol=1e-12, atol=1e-12)
        np.testing.assert_array_equal(best, want_max[lo:hi])
        np.testing.assert_array_equal(best_e, want_e[lo:hi])


def _slice_rank(rank, world, port, q, slices):
    """The sliced-gather halo: slice c of every owner block arrives by one
    all-gather and is reduced over the shard's edges whose sources fall in
    it; sums add slice by slice, max keeps the better value with the smaller
    edge id on a tie."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import oracle as orc

        from mojodgl.partition import slice_exchange, slice_of, slice_rows

        u, v, h, n = graph(seed=13)
        bounds = edge_balanced_ranges(np.bincount(v, minlength=n), world)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        blk, owners = owner_blocks(n, world)
        sb = slice_rows(blk, slices)
        a, b = owners[rank]
        mine = torch.zeros(slices * sb, h.shape[1], dtype=torch.float64)
        mine[: b - a] = torch.from_numpy(h[a:b])
        sel = np.nonzero((v >= lo) & (v < hi))[0]
        cc, local = slice_of(u[sel], blk, sb)
        sums = np.zeros((hi - lo, h.shape[1]))
        best = np.full((hi - lo, h.shape[1]), -np.inf)
        best_e = np.full((hi - lo, h.shape[1]), -1, dtype=np.int64)
        seen = []

        def on_slice(c, gathered, first, last):
            seen.append((c, first, last))
            assert gathered.shape[0] == world * sb
            k = np.nonzero(cc == c)[0]
            og = orc.Graph(local[k], v[sel[k]] - lo, num_nodes=max(world * sb, hi - lo))
            x = gathered.numpy()
            part = orc.gspmm(og, "copy_lhs", "sum", x, None)[: hi - lo]
            sums[:] = part if first else sums + part
            mx, au, ae = orc.gspmm(og, "copy_lhs", "max", x, None, with_arg=True)
            mx, ae = mx[: hi - lo], ae[: hi - lo]
            ge = np.where(ae >= 0, sel[k][np.maximum(ae, 0)], -1)  # global edge ids
            take = (mx > best) | ((mx == best) & (ge >= 0) & ((best_e < 0) | (ge < best_e)))
            best[take] = mx[take]
            best_e[take] = ge[take]

        slice_exchange(mine, sb, slices, world, None, on_slice)
        q.put((rank, lo, hi, sums, best, best_e, seen))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,slices", [(2, 3), (3, 4), (4, 4)])
def test_slice_halo_reproduces_the_single_process_result(world, slices):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_slice_rank, args=(r, world, port, q, slices)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle as orc

    u, v, h, n = graph(seed=13)
    og = orc.Graph(u, v, num_nodes=n)
    want_sum = orc.gspmm(og, "copy_lhs", "sum", h, None)
    want_max, _, want_e = orc.gspmm(og, "copy_lhs", "max", h, None, with_arg=True)
    for rank, lo, hi, sums, best, best_e, seen in results:
        assert seen == [(c, c == 0, c == slices - 1) for c in range(slices)]
        np.testing.assert_allclose(sums, want_sum[lo:hi], rtol=1e-12, atol=1e-12)
        np.testing.assert_array_equal(best, want_max[lo:hi])
        np.testing.assert_array_equal(best_e, want_e[lo:hi])


def _other_ops_rank(rank, world, port, q):
    """gSDDMM by destination shards (u features all-gathered), segment_mm by
    relation ranges balanced by rows, gather_mm by row blocks (b replicated):
    each rank runs the oracle on its part only."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import oracle as orc

        from mojodgl.partition import row_block_ranges, segment_balanced_ranges

        # gsddmm u_dot_v and u_add_v on the destination shard's edges
        u, v, h, n = graph(seed=21)
        bounds = edge_balanced_ranges(np.bincount(v, minlength=n), world)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        shard = DstShard(u, v, lo, hi)
        blk, owners = owner_blocks(n, world)
        a, b = owners[rank]
        mine = torch.zeros(blk, h.shape[1], dtype=torch.float64)
        mine[: b - a] = torch.from_numpy(h[a:b])
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        full = assemble_gathered([p.numpy() for p in parts], n)
        og = orc.Graph(shard.u, shard.v_local + lo, num_nodes=n)
        dot = orc.gsddmm(og, "dot", full, full, "u", "v")
        add = orc.gsddmm(og, "add", full, full, "u", "v")

        # segment_mm by relation ranges
        rng = np.random.default_rng(22)
        r, d1, d2 = 7, 5, 3
        seglen = rng.integers(0, 40, r)
        rows = int(seglen.sum())
        am = rng.normal(size=(rows, d1))
        bm = rng.normal(size=(r, d1, d2))
        rb = segment_balanced_ranges(seglen, world)
        off = np.concatenate([[0], np.cumsum(seglen)])
        r0, r1 = int(rb[rank]), int(rb[rank + 1])
        seg_part = orc.segment_mm(am[off[r0]:off[r1]], bm[r0:r1], seglen[r0:r1]) if r1 > r0 else None

        # gather_mm by row blocks
        idx = rng.integers(0, r, 50)
        ga = rng.normal(size=(50, d1))
        gb = row_block_ranges(50, world)
        g0, g1 = int(gb[rank]), int(gb[rank + 1])
        gm_part = orc.gather_mm(ga[g0:g1], bm, idx[g0:g1])
        q.put((rank, shard.eids, dot, add, (off[r0], off[r1], seg_part), (g0, g1, gm_part)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_other_ops_shard_and_stitch_to_the_single_process_result(world):
    from mojodgl.partition import scatter_edge_rows

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_other_ops_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle as orc

    u, v, h, n = graph(seed=21)
    og = orc.Graph(u, v, num_nodes=n)
    np.testing.assert_array_equal(scatter_edge_rows([(t[1], t[2]) for t in results], u.size),
                                  orc.gsddmm(og, "dot", h, h, "u", "v"))
    np.testing.assert_array_equal(scatter_edge_rows([(t[1], t[3]) for t in results], u.size),
                                  orc.gsddmm(og, "add", h, h, "u", "v"))
    rng = np.random.default_rng(22)
    r, d1, d2 = 7, 5, 3
    seglen = rng.integers(0, 40, r)
    am = rng.normal(size=(int(seglen.sum()), d1))
    bm = rng.normal(size=(r, d1, d2))
    want = orc.segment_mm(am, bm, seglen)
    got = np.zeros_like(want)
    for t in results:
        s0, s1, part = t[4]
        if part is not None:
            got[s0:s1] = part
    np.testing.assert_array_equal(got, want)
    idx = rng.integers(0, r, 50)
    ga = rng.normal(size=(50, d1))
    want = orc.gather_mm(ga, bm, idx)
    got = np.concatenate([t[5][2] for t in results])
    np.testing.assert_array_equal(got, want)


def _grid_rank(rank, world, port, q, cols, slices):
    """A rank of an R x C grid: its row group's destinations, its column
    group's feature columns, owner blocks exchanged by sliced all-gathers
    within the column group only."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import oracle as orc

        from mojodgl.partition import (column_group_ranks, column_range, rank_grid,
                                       slice_exchange, slice_of, slice_rows)

        rows, rg, cg = rank_grid(rank, world, cols)
        groups = [dist.new_group(r) for r in column_group_ranks(world, cols)]
        u, v, h, n = graph(seed=17)
        c0, c1 = column_range(h.shape[1], cols, cg)
        hc = np.ascontiguousarray(h[:, c0:c1])
        bounds = edge_balanced_ranges(np.bincount(v, minlength=n), rows)
        lo, hi = int(bounds[rg]), int(bounds[rg + 1])
        blk, owners = owner_blocks(n, rows)
        sb = slice_rows(blk, slices)
        a, b = owners[rg]
        mine = torch.zeros(slices * sb, c1 - c0, dtype=torch.float64)
        mine[: b - a] = torch.from_numpy(hc[a:b])
        sel = np.nonzero((v >= lo) & (v < hi))[0]
        cc, local = slice_of(u[sel], blk, sb)
        sums = np.zeros((hi - lo, c1 - c0))
        best = np.full((hi - lo, c1 - c0), -np.inf)
        best_e = np.full((hi - lo, c1 - c0), -1, dtype=np.int64)

        def on_slice(c, gathered, first, last):
            assert gathered.shape == (rows * sb, c1 - c0)
            k = np.nonzero(cc == c)[0]
            og = orc.Graph(local[k], v[sel[k]] - lo, num_nodes=max(rows * sb, hi - lo))
            x = gathered.numpy()
            part = orc.gspmm(og, "copy_lhs", "sum", x, None)[: hi - lo]
            sums[:] = part if first else sums + part
            mx, _, ae = orc.gspmm(og, "copy_lhs", "max", x, None, with_arg=True)
            mx, ae = mx[: hi - lo], ae[: hi - lo]
            ge = np.where(ae >= 0, sel[k][np.maximum(ae, 0)], -1)
            take = (mx > best) | ((mx == best) & (ge >= 0) & ((best_e < 0) | (ge < best_e)))
            best[take] = mx[take]
            best_e[take] = ge[take]

        slice_exchange(mine, sb, slices, rows, None, on_slice, groups[cg])
        q.put((rank, lo, hi, c0, c1, sums, best, best_e))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cols", [(2, 2), (4, 2), (4, 4)])
def test_rank_grid_reproduces_the_single_process_result(world, cols):
    """Row x column rank grids: the pieces (row range x column range) of all
    ranks tile the single-process result; sums to rtol 1e-12, max and its
    edge ids exactly."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_grid_rank, args=(r, world, port, q, cols, 3))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle as orc

    u, v, h, n = graph(seed=17)
    og = orc.Graph(u, v, num_nodes=n)
    want_sum = orc.gspmm(og, "copy_lhs", "sum", h, None)
    want_max, _, want_e = orc.gspmm(og, "copy_lhs", "max", h, None, with_arg=True)
    covered = np.zeros(want_sum.shape, dtype=np.int64)
    for rank, lo, hi, c0, c1, sums, best, best_e in results:
        np.testing.assert_allclose(sums, want_sum[lo:hi, c0:c1], rtol=1e-12, atol=1e-12)
        np.testing.assert_array_equal(best, want_max[lo:hi, c0:c1])
        np.testing.assert_array_equal(best_e, want_e[lo:hi, c0:c1])
        covered[lo:hi, c0:c1] += 1
    assert np.all(covered == 1)
