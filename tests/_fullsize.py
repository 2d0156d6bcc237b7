"""Helpers of the full-size parity tests (test_gpu_full_cfg*.py): device
row fetches and the suite's tolerance checks."""

import numpy as np
import torch


def take(t, ids):
    """Rows ``ids`` of a device tensor, as a host numpy array."""
    idx = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int64)).to(t.device)
    return t[idx].cpu().numpy()


def within_s(got, ref, s, tol=1e-5, what=""):
    """|got - ref| <= tol |ref| + tol S elementwise (S = the row's sum of
    |message|, from the oracle): the suite's bound for float32 sums."""
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    bound = tol * np.abs(ref) + tol * s + 1e-30
    bad = err > bound
    assert not bad.any(), "{}: max excess {} at {}".format(what, (err - bound).max(),
                                                           np.argwhere(bad)[:5])
