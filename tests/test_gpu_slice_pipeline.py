"""The multi-GPU halo's device path on one GPU: a one-rank NCCL group runs
SlicePipeline (per-slice sub-CSRs, one accumulating gSpMM pass per gathered
slice, mean and inf->0 on the last pass) and must match the one-pass gSpMM:
max/min bit for bit, sum/mean within the float32 gSpMM bound."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_slice_pipeline_matches_one_pass():
    import torch.distributed as dist

    from mojodgl.partition import DeviceShard, DstShard, SlicePipeline

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        rng = np.random.default_rng(17)
        n, e, d = 20_000, 400_000, 64
        u = rng.integers(0, n, e)
        v = rng.integers(0, n, e)
        v[:5000] = 3  # a hub split over merge-path chunks
        h = torch.from_numpy(rng.normal(size=(n, d)).astype(np.float32)).cuda()
        shard = DeviceShard(DstShard(u, v, 0, n))
        pipe = SlicePipeline(u, v, 0, n, 0, 1, n, slices=3)
        block = torch.zeros((pipe.block_rows(), d), device="cuda")
        block[:n] = h
        for red in ("sum", "mean", "max", "min"):
            want = shard.copy_u(h, red)
            got = torch.empty_like(want)
            pipe.copy_u(block, red, got)
            torch.cuda.synchronize()
            if red in ("max", "min"):
                assert torch.equal(got, want), red
            else:
                s = shard.copy_u(h.abs(), "sum" if red == "sum" else "mean")
                err = (got - want).abs()
                assert bool((err <= 1e-5 * want.abs() + 1e-5 * s).all()), red
    finally:
        dist.destroy_process_group()
