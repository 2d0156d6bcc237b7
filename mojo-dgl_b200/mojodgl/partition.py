"""Destination-row partitioning of one graph across the GPUs of a node.

Every output row of gSpMM is independent (the reference splits its 32 CPU
workers the same way, src/ported.mojo:34-39, 442-443), so the graph is cut
into P contiguous destination-row ranges with about E/P in-edges each (a
row-count split would not balance a power-law in-degree).  Node features are
owned in P contiguous, equal row blocks.  With uniform sources a shard
references nearly every source row, so the halo is the whole feature matrix
and a selective exchange would not pay.  DeviceShard runs the local gSpMM on
a gathered matrix (one all-gather, then compute); SlicePipeline overlaps the
two, gathering the blocks slice by slice with one all-gather each and running
an accumulating gSpMM pass per slice as it arrives (OwnerPipeline does the
same over a ring of point-to-point steps, one owner block per step).
Outputs stay sharded by destination row.

The ranks can also form a grid of R row groups x C column groups
(``rank_grid``): a rank owns a block of rows of one column block of the
features, aggregates its row group's destinations for its column block only,
and exchanges owner blocks within its column group (R ranks).  Each rank then
receives (R - 1) / R of N x D / C feature values instead of (P - 1) / P of
N x D -- with C = P (one row group) no exchange at all -- while its gather
rows are D / C wide.

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


def rank_grid(rank: int, world: int, cols: int):
    """Ranks as R = world / cols row groups x `cols` column groups, rank =
    row_group * cols + col_group: a rank aggregates the destination rows of
    its row group for the feature columns of its column group.  Returns
    (R, row_group, col_group)."""
    if cols < 1 or world % cols:
        raise ValueError("{} ranks do not split into {} column groups".format(world, cols))
    return world // cols, rank // cols, rank % cols


def column_group_ranks(world: int, cols: int):
    """The ranks of every column group (the ranks that hold the same feature
    columns for different destination rows, and exchange their owner blocks),
    in column-group order."""
    rows = world // cols
    return [[rg * cols + cg for rg in range(rows)] for cg in range(cols)]


def column_range(d: int, cols: int, col_group: int):
    """Feature columns [c0, c1) of a column group: d split into `cols` near-equal
    contiguous ranges."""
    return d * col_group // cols, d * (col_group + 1) // cols


def segment_balanced_ranges(seglen: np.ndarray, parts: int):
    """segment_mm across ranks: P+1 relation boundaries so each rank's
    contiguous relations hold about the same number of rows; a relation's b
    block lives with the rank that owns it, so no collective is needed."""
    return edge_balanced_ranges(np.asarray(seglen, dtype=np.int64), parts)


def row_block_ranges(n: int, parts: int):
    """gather_mm across ranks: contiguous row blocks of a (b, at 64 x 256 x 256
    values, is replicated or broadcast once)."""
    return np.asarray([lo for lo, _ in owner_blocks(n, parts)[1]] + [n], dtype=np.int64)


def scatter_edge_rows(pieces, num_edges: int):
    """Stitch per-rank gSDDMM results into the (E, ...) output: pieces are
    (global edge ids, rows) pairs, one per rank's destination shard."""
    first = pieces[0][1]
    out = np.zeros((num_edges,) + tuple(first.shape[1:]), dtype=first.dtype)
    for eids, rows in pieces:
        out[eids] = rows
    return out


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
        # the shard holds every in-edge of its rows, so the mean's degree is
        # the CSR row length, which the kernel has in hand (deg = NULL)
        check(lib().bgl_gspmm(T.ptr(self.indptr), T.ptr(self.indices), None, None, n, ne,
                              T.ptr(feat), d, 1, None, 1, 1, T.ptr(out), d, T.ptr(arg_u), None, code,
                              OP_COPY_LHS, red, BGL_ZERO_INF if reduce_op in ("max", "min") else 0,
                              T.ptr(workspace), nbytes, T.stream()), "gspmm")
        return out


class OwnerPipeline:
    """A destination-row shard whose in-edges are split by the owner block of
    their source, so the halo exchange overlaps the aggregation.

    The features arrive over P - 1 ring steps of NCCL send/recv (step k: send
    my block to rank + k, receive the block of rank - k); the gSpMM pass over
    the edges whose sources live in a block runs as soon as that block is in,
    while the next block is in flight.  Each pass after the first folds into
    the output (BGL_ACCUMULATE); the mean divide and the max/min inf->0 are
    applied by the last pass.  Per-owner sub-CSRs keep global edge ids, so
    max/min ties resolve to the smaller edge id, as in the single-GPU result;
    sums are the same messages added in owner-block order (compared with a
    tolerance against the single-GPU order)."""

    def __init__(self, u, v, lo, hi, rank, world, num_nodes):
        import torch

        from . import _tensor as T
        from ._lib import check, lib

        self.rank, self.world = rank, world
        self.lo, self.hi = int(lo), int(hi)
        self.blk, self.owners = owner_blocks(num_nodes, world)
        n = self.hi - self.lo
        sel = np.nonzero((v >= lo) & (v < hi))[0]
        uu = u[sel]
        vv = v[sel] - lo
        owner = uu // self.blk
        dev = T.device()
        self.parts = []
        for p in range(world):
            m = np.nonzero(owner == p)[0]
            ne = int(m.size)
            key = torch.from_numpy(np.ascontiguousarray(vv[m])).to(dev)
            other = torch.from_numpy(np.ascontiguousarray(uu[m] - p * self.blk)).to(dev)
            indptr = torch.empty(n + 1, dtype=torch.int64, device=dev)
            deg = torch.empty(n, dtype=torch.int64, device=dev)
            order = torch.empty(ne, dtype=torch.int32, device=dev)
            indices = torch.empty(ne, dtype=torch.int32, device=dev)
            nbytes = lib().bgl_csr_build_workspace_size(ne, n)
            ws = T.workspace(nbytes)
            check(lib().bgl_csr_build(T.ptr(key), T.ptr(other), ne, n, T.ptr(indptr), T.ptr(deg),
                                      T.ptr(order), T.ptr(indices), T.ptr(ws), nbytes, T.stream()),
                  "bgl_csr_build")
            gid = torch.from_numpy(sel[m].astype(np.int64)).to(dev)
            eid = gid[order.long()].to(torch.int32) if ne else order
            self.parts.append((indptr, indices, eid, ne))
        self.deg = torch.from_numpy(np.bincount(vv, minlength=n).astype(np.int64)).to(dev)
        self.num_rows = n

    def _pass(self, p, feat, out, reduce_op, first, last, arg_e, ws):
        from . import _tensor as T
        from ._lib import (BGL_ACCUMULATE, BGL_ZERO_INF, OP_COPY_LHS, REDUCE_SUM, REDUCERS, check,
                           lib)

        indptr, indices, eid, ne = self.parts[p]
        d = int(feat.shape[1])
        red = REDUCERS[reduce_op]
        if reduce_op == "mean" and not last:
            red = REDUCE_SUM
        flags = (0 if first else BGL_ACCUMULATE)
        if last and reduce_op in ("max", "min"):
            flags |= BGL_ZERO_INF
        code = T.code_of(feat.dtype)
        nbytes = lib().bgl_gspmm_workspace_size(self.num_rows, ne, d, code, red)
        if ws[0] is None or ws[0].numel() < nbytes:
            ws[0] = T.workspace(nbytes)
        check(lib().bgl_gspmm(T.ptr(indptr), T.ptr(indices), T.ptr(eid), T.ptr(self.deg),
                              self.num_rows, ne, T.ptr(feat), d, 1, None, 1, 1, T.ptr(out), d, None,
                              T.ptr(arg_e), code, OP_COPY_LHS, red, flags, T.ptr(ws[0]), nbytes,
                              T.stream()), "gspmm")

    def copy_u(self, my_block, reduce_op, out, arg_e=None, bufs=None, ws=None):
        """out[rows of this shard] = reduce over in-edges of the source
        feature; my_block is this rank's (blk, D) feature block."""
        ws = ws if ws is not None else [None]

        def on_block(owner, block, first, last):
            self._pass(owner, block, out, reduce_op, first, last, arg_e, ws)

        ring_exchange(my_block, bufs, self.rank, self.world, on_block)
        return out


def ring_exchange(my_block, bufs, rank, world, on_block):
    """Hand every rank's feature block to on_block(owner, block, first, last),
    this rank's own block first, then the others as they arrive over P - 1
    ring steps of send/recv (step k: send to rank + k, receive from rank - k).
    Step k + 1 is issued before block k is processed, so the transfer of the
    next block overlaps the work on the current one; the two receive buffers
    alternate, and a buffer is only refilled once the work issued on it is in
    the stream order before the receive (torch orders a collective after the
    work already queued on the current stream)."""
    import torch
    import torch.distributed as dist

    P, r = world, rank
    if P == 1:
        on_block(r, my_block, True, True)
        return
    if bufs is None:
        bufs = [torch.empty_like(my_block), torch.empty_like(my_block)]

    def issue(k):
        ops = [dist.P2POp(dist.isend, my_block, (r + k) % P),
               dist.P2POp(dist.irecv, bufs[k % 2], (r - k) % P)]
        return dist.batch_isend_irecv(ops)

    works = issue(1)
    on_block(r, my_block, True, False)
    for k in range(1, P):
        for w in works:
            w.wait()
        if k + 1 < P:
            works = issue(k + 1)
        on_block((r - k) % P, bufs[k % 2], False, k == P - 1)


def slice_rows(blk: int, slices: int):
    """Rows per slice when each owner block of `blk` rows is cut into
    `slices` equal slices (the last may hold fewer real rows)."""
    return max(1, -(-blk // slices))


def slice_of(u: np.ndarray, blk: int, sb: int):
    """For global source rows u: the slice they fall in and their row in
    that slice's gathered buffer (owners concatenated in rank order, sb rows
    each)."""
    owner = u // blk
    off = u - owner * blk
    c = off // sb
    return c, owner * sb + (off - c * sb)


class SlicePipeline:
    """A destination-row shard whose in-edges are split by the slice of
    their source's owner block, so the halo exchange overlaps the
    aggregation with collectives rather than point-to-point steps.

    Every owner block of features is cut into C equal row slices.  Step c
    gathers slice c of every rank's block with one NCCL all-gather (the
    collective runs at the all-gather bus rate; NCCL's point-to-point
    send/recv moved a third of that in the same box) and runs one gSpMM pass
    over the shard's edges whose sources fall in those slices, while the
    gather of slice c + 1 is in flight.  Passes after the first fold into the
    output (BGL_ACCUMULATE); the mean divide and the max/min inf->0 run on
    the last pass.  The sub-CSRs keep global edge ids, so max/min ties
    resolve to the smaller edge id, as in the single-GPU result; sums add
    the same messages slice by slice (compared with a tolerance against the
    single-GPU order)."""

    def __init__(self, u, v, lo, hi, rank, world, num_nodes, slices=4, group=None):
        import torch

        from . import _tensor as T
        from ._lib import check, lib

        # rank / world / group: this rank's place among the ranks that exchange
        # owner blocks (all ranks, or one column group of a rank grid)
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = int(lo), int(hi)
        self.blk, self.owners = owner_blocks(num_nodes, world)
        self.slices = int(slices)
        self.sb = slice_rows(self.blk, self.slices)
        n = self.hi - self.lo
        sel = np.nonzero((v >= lo) & (v < hi))[0]
        vv = v[sel] - lo
        cc, local = slice_of(u[sel], self.blk, self.sb)
        dev = T.device()
        self.parts = []
        for c in range(self.slices):
            m = np.nonzero(cc == c)[0]
            ne = int(m.size)
            key = torch.from_numpy(np.ascontiguousarray(vv[m])).to(dev)
            other = torch.from_numpy(np.ascontiguousarray(local[m])).to(dev)
            indptr = torch.empty(n + 1, dtype=torch.int64, device=dev)
            deg = torch.empty(n, dtype=torch.int64, device=dev)
            order = torch.empty(ne, dtype=torch.int32, device=dev)
            indices = torch.empty(ne, dtype=torch.int32, device=dev)
            nbytes = lib().bgl_csr_build_workspace_size(ne, n)
            ws = T.workspace(nbytes)
            check(lib().bgl_csr_build(T.ptr(key), T.ptr(other), ne, n, T.ptr(indptr), T.ptr(deg),
                                      T.ptr(order), T.ptr(indices), T.ptr(ws), nbytes, T.stream()),
                  "bgl_csr_build")
            gid = torch.from_numpy(sel[m].astype(np.int64)).to(dev)
            eid = gid[order.long()].to(torch.int32) if ne else order
            self.parts.append((indptr, indices, eid, ne))
        self.deg = torch.from_numpy(np.bincount(vv, minlength=n).astype(np.int64)).to(dev)
        self.num_rows = n

    def block_rows(self):
        """Rows of the (padded) feature block each rank contributes."""
        return self.slices * self.sb

    # the pass is the owner pipeline's: same accumulate / last-pass rules
    _pass = OwnerPipeline._pass

    def copy_u(self, my_block, reduce_op, out, arg_e=None, bufs=None, ws=None):
        """out[rows of this shard] = reduce over in-edges of the source
        feature; my_block is this rank's (block_rows(), D) feature block."""
        ws = ws if ws is not None else [None]

        def on_slice(c, gathered, first, last):
            self._pass(c, gathered, out, reduce_op, first, last, arg_e, ws)

        slice_exchange(my_block, self.sb, self.slices, self.world, bufs, on_slice, self.group)
        return out


def slice_exchange(my_block, sb, slices, world, bufs, on_slice, group=None):
    """Hand on_slice(c, gathered, first, last) every slice c of all ranks'
    blocks, gathered rank-major (world * sb rows), gathering slice c + 1
    while slice c is processed; the two buffers alternate, and a buffer is
    refilled only after the work queued on it (a collective is ordered after
    the work already on the current stream).  NCCL gathers into one tensor
    asynchronously; other backends (gloo, for the CPU tests) gather a list
    and copy it in.  ``group``: the process group of the ranks that exchange
    (None: all ranks)."""
    import torch
    import torch.distributed as dist

    if bufs is None:
        bufs = [my_block.new_empty((world * sb,) + tuple(my_block.shape[1:])) for _ in range(2)]
    nccl = dist.get_backend(group) == "nccl"

    def issue(c):
        part = my_block[c * sb:(c + 1) * sb]
        if nccl:
            return dist.all_gather_into_tensor(bufs[c % 2], part, group=group, async_op=True)
        pieces = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(pieces, part.contiguous(), group=group)
        torch.cat(pieces, out=bufs[c % 2])
        return None

    work = issue(0)
    for c in range(slices):
        if work is not None:
            work.wait()
        if c + 1 < slices:
            work = issue(c + 1)
        on_slice(c, bufs[c % 2], c == 0, c == slices - 1)


def pull_order(rank: int, world: int):
    """The peers whose blocks rank pulls, in order: rank + 1, rank + 2, ...
    (mod world).  At every position of the order the ranks pull from
    distinct peers (a rotation), so each GPU serves one reader at a time."""
    return [(rank + k) % world for k in range(1, world)]


class PeerPipeline(OwnerPipeline):
    """A destination-row shard whose halo arrives by copy-engine pulls
    straight from its peers' memory, overlapped with the aggregation.

    Every rank of the exchange group (all ranks, or one column group of a
    rank grid) holds a halo buffer of world x blk rows in owner order
    (``halo``); its own owner block (``own_block()``) is written there by the
    caller.  The buffers are mapped into every peer's address space once,
    through CUDA IPC.  A call then (1) meets the peers in a one-element NCCL
    all-reduce, which completes once every rank has queued the writes of its
    own block; (2) queues on a side stream one copy-engine copy per peer
    block (``bgl_peer_copy``: a DMA over NVLink, no SM time), in
    ``pull_order``; (3) runs the gSpMM pass over the edges whose sources are
    its own rows at once, and the pass over each peer's edges once that
    peer's copy has landed (an event), accumulating into ``out``; (4) meets
    the peers again after its copies, and the caller's stream waits for that
    before it returns, so no rank overwrites its block while a peer may
    still read it.  The NCCL all-gather schedule (SlicePipeline) needs SMs
    for its kernels while the gSpMM grid holds them all; this one does not.
    The passes, the accumulate rules and the tie-breaking are
    OwnerPipeline's."""

    def __init__(self, u, v, lo, hi, rank, world, num_nodes, dim, dtype=None, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _tensor as T
        from ._lib import check, lib

        super().__init__(u, v, lo, hi, rank, world, num_nodes)
        self.group = group
        dev = T.device()
        dtype = dtype or torch.float32
        self.halo = torch.zeros((world * self.blk, int(dim)), dtype=dtype, device=dev)
        self.row_bytes = int(dim) * self.halo.element_size()
        self.copy_stream = torch.cuda.Stream(device=dev)
        self.landed = [torch.cuda.Event() for _ in range(world)]
        self.fence = torch.zeros(2, dtype=torch.float32, device=dev)
        self.peer = {}
        if world > 1:
            nbytes = self.halo.numel() * self.halo.element_size()
            handle = ctypes.create_string_buffer(64)
            off = ctypes.c_int64(0)
            check(lib().bgl_ipc_export(T.ptr(self.halo), nbytes, handle, ctypes.byref(off)),
                  "bgl_ipc_export")
            mine = (bytes(handle.raw), int(off.value), int(nbytes))
            got = [None] * world
            dist.all_gather_object(got, mine, group=group)
            for q in range(world):
                if q == rank:
                    continue
                h, o, nb = got[q]
                if nb != nbytes:
                    raise RuntimeError(f"PeerPipeline: rank {q} exported {nb} bytes, expected {nbytes}")
                p = ctypes.c_void_p(0)
                check(lib().bgl_ipc_open(h, o, nb, ctypes.byref(p)), "bgl_ipc_open")
                self.peer[q] = int(p.value)
            torch.cuda.synchronize()
            dist.barrier(group=group)

    def own_block(self):
        """This rank's rows of the halo buffer: the caller writes its owner
        block's features here (on the current stream) before a call."""
        lo, hi = self.owners[self.rank]
        return self.halo[self.rank * self.blk:self.rank * self.blk + (hi - lo)]

    def block(self, q):
        """Owner q's rows of the halo buffer."""
        lo, hi = self.owners[q]
        return self.halo[q * self.blk:q * self.blk + (hi - lo)]

    def pull(self, q, stream):
        """Queue the copy of owner q's block from its rank's halo buffer."""
        from . import _tensor as T
        from ._lib import check, lib

        lo, hi = self.owners[q]
        off = q * self.blk * self.row_bytes
        nbytes = (hi - lo) * self.row_bytes
        check(lib().bgl_peer_copy(T.ptr(self.halo) + off, self.peer[q] + off, nbytes,
                                  stream.cuda_stream), "bgl_peer_copy")

    def copy_u(self, reduce_op, out, arg_e=None, ws=None):
        """out[rows of this shard] = reduce over in-edges of the source
        feature, the features being every rank's own_block()."""
        import torch
        import torch.distributed as dist

        ws = ws if ws is not None else [None]
        order = pull_order(self.rank, self.world)
        cur = torch.cuda.current_stream()
        if order:
            ready = dist.all_reduce(self.fence[:1], group=self.group, async_op=True)
            with torch.cuda.stream(self.copy_stream):
                ready.wait()
                for q in order:
                    self.pull(q, self.copy_stream)
                    self.landed[q].record(self.copy_stream)
                done = dist.all_reduce(self.fence[1:], group=self.group, async_op=True)
        self._pass(self.rank, self.block(self.rank), out, reduce_op, True, not order, arg_e, ws)
        for k, q in enumerate(order):
            cur.wait_event(self.landed[q])
            self._pass(q, self.block(q), out, reduce_op, False, k == len(order) - 1, arg_e, ws)
        if order:
            done.wait()
        return out

    def close(self):
        """Unmap the peers' buffers (after every rank's last call)."""
        import torch
        import torch.distributed as dist

        from ._lib import check, lib

        if not self.peer:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for q, p in self.peer.items():
            check(lib().bgl_ipc_close(p), "bgl_ipc_close")
        self.peer = {}
