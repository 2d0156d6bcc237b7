"""The copy-engine halo (PeerPipeline, bgl_ipc_* / bgl_peer_copy).

The two-GPU test runs tests/_peer_worker.py on two ranks (skipped on a box
with one GPU) and checks every rank's rows against the oracle: sums and
means within the float32 tolerance (the owner-block passes regroup the sum),
max values and their edge ids exactly.  The range checks of bgl_peer_copy
are host-side and run on one GPU."""

import ctypes
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from _fullsize import within_s

pytestmark = pytest.mark.gpu

from mojodgl import _lib  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BGL_E_INVALID = 1


def test_peer_copy_rejects_ranges_outside_the_allocation():
    lib = _lib.lib()
    a = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    b = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.bgl_peer_copy(a.data_ptr(), b.data_ptr(), 4096, s) == 0
    for dst, src, nb in ((a.data_ptr(), b.data_ptr(), 1 << 40),
                         (a.data_ptr(), b.data_ptr(), -1),
                         (None, b.data_ptr(), 16)):
        assert lib.bgl_peer_copy(dst, src, nb, s) == BGL_E_INVALID
    handle = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(-1)
    assert lib.bgl_ipc_export(a.data_ptr(), 1 << 40, handle, ctypes.byref(off)) == BGL_E_INVALID
    assert lib.bgl_ipc_export(a.data_ptr(), 4096, handle, ctypes.byref(off)) == 0
    assert off.value >= 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_pipeline_two_ranks_match_the_oracle(orc, tmp_path):
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
           str(port), os.path.join(ROOT, "tests", "_peer_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from _peer_worker import graph

    u, v, h1, h2 = graph()
    n = h1.shape[0]
    og = orc.Graph(u, v, num_nodes=n)
    for tag, h in (("h1", h1), ("h2", h2)):
        x = h.astype(np.float64)
        s_ref = orc.gspmm(og, "copy_lhs", "sum", x, None)
        mean_ref = orc.gspmm(og, "copy_lhs", "mean", x, None)
        s_abs = orc.gspmm(og, "copy_lhs", "sum", np.abs(x), None)
        deg = np.maximum(og.indeg, 1)[:, None]
        mx, _, ae = orc.gspmm(og, "copy_lhs", "max", x, None, with_arg=True)
        mx = np.where(np.isinf(mx), 0.0, mx)
        for rank in range(2):
            z = np.load(tmp_path / f"rank{rank}.npz")
            lo, hi = int(z["lo"]), int(z["hi"])
            within_s(z[f"{tag}_sum"], s_ref[lo:hi], s_abs[lo:hi], what=f"{tag} sum rank {rank}")
            within_s(z[f"{tag}_mean"], mean_ref[lo:hi], s_abs[lo:hi] / deg[lo:hi],
                     what=f"{tag} mean rank {rank}")
            np.testing.assert_array_equal(z[f"{tag}_max"], mx[lo:hi].astype(np.float32))
            np.testing.assert_array_equal(z[f"{tag}_arg_e"], ae[lo:hi])
