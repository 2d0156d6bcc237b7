"""One rank of the two-GPU PeerPipeline test (tests/test_gpu_peer.py runs it
under torch.distributed.run).  Each rank aggregates its destination rows of
a seeded graph through PeerPipeline.copy_u -- sum, mean, max with edge ids
-- and saves its rows for the parent test to check against the oracle.
Between calls the ranks overwrite their own blocks with new features, so the
second call's result also shows that no pull read a stale or half-written
block."""

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "mojo-dgl_b200"))
sys.path.insert(0, ROOT)

from mojodgl.partition import PeerPipeline, edge_balanced_ranges, owner_blocks  # noqa: E402


def graph(n=40_000, e=600_000, d=24, seed=5):
    """The test graph: uniform edges plus a hub of 20,000 in-edges (split
    over merge-path chunks), and two feature matrices."""
    rng = np.random.default_rng(seed)
    u = rng.integers(0, n, e)
    v = rng.integers(0, n, e)
    v[rng.choice(e, 20_000, replace=False)] = 1234
    h1 = rng.normal(size=(n, d)).astype(np.float32)
    h2 = rng.normal(size=(n, d)).astype(np.float32)
    # a quarter of owner block 1 repeats owner block 0 (two ranks: blocks of
    # n / 2 rows), so maxima tie across the two passes; the earlier edge wins
    h2[n // 2:n // 2 + n // 4] = h2[:n // 4]
    return u, v, h1, h2


def main(outdir):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    u, v, h1, h2 = graph()
    n, d = h1.shape
    bounds = edge_balanced_ranges(np.bincount(v, minlength=n), world)
    lo, hi = int(bounds[rank]), int(bounds[rank + 1])
    pipe = PeerPipeline(u, v, lo, hi, rank, world, n, d)
    _, owners = owner_blocks(n, world)
    own_lo, own_hi = owners[rank]
    out = torch.empty((hi - lo, d), device="cuda")
    arg_e = torch.empty((hi - lo, d), dtype=torch.int64, device="cuda")
    saved = {"lo": lo, "hi": hi}
    for tag, h in (("h1", h1), ("h2", h2)):
        pipe.own_block().copy_(torch.from_numpy(h[own_lo:own_hi]).cuda())
        for red in ("sum", "mean", "max"):
            pipe.copy_u(red, out, arg_e=arg_e if red == "max" else None)
            saved[f"{tag}_{red}"] = out.cpu().numpy()
            if red == "max":
                saved[f"{tag}_arg_e"] = arg_e.cpu().numpy()
    torch.cuda.synchronize()
    pipe.close()
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), **saved)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
