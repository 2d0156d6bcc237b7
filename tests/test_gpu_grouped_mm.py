"""The tcgen05 grouped GEMM behind segment_mm / gather_mm (TF32 for float32
inputs, BF16 for bfloat16 tensors) against the float64 oracle.

Tolerance for the tensor-core paths: |ours - ref| <= 1e-2 |ref| + 1e-2 S with
S = |a| @ |b| (the oracle computes it); after every launch the kernel's
device status word (bounded mbarrier waits) must read 0.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import mojodgl.ops as ops  # noqa: E402
from mojodgl import _lib  # noqa: E402


def within_s(got, ref, s, tol=1e-2):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    bound = tol * np.abs(ref) + tol * s + 1e-30
    bad = err > bound
    assert not bad.any(), "max excess {} at {}".format((err - bound).max(), np.argwhere(bad)[:5])


def no_device_error():
    assert _lib.lib().bgl_tc_error() == 0


def segments(rng, n, r, zero=()):
    seglen = rng.multinomial(n, rng.dirichlet(0.5 * np.ones(r)))
    for z in zero:
        seglen[0] += seglen[z]
        seglen[z] = 0
    return seglen


@pytest.mark.parametrize("d1,d2", [(256, 256), (64, 48), (40, 24), (128, 512), (96, 136)])
def test_segment_mm_tf32(orc, d1, d2):
    rng = np.random.default_rng(d1 * 1000 + d2)
    n, r = 9000, 7
    seglen = segments(rng, n - 300, r, zero=(3,))  # 300 trailing rows stay zero
    a = rng.normal(0, 0.05, size=(n, d1)).astype(np.float32)
    b = rng.normal(0, 0.05, size=(r, d1, d2)).astype(np.float32)
    got = ops.segment_mm(a, b, seglen)
    no_device_error()
    within_s(got, orc.segment_mm(a, b, seglen), orc.segment_mm(np.abs(a), np.abs(b), seglen))
    assert np.all(got[n - 300:] == 0)


@pytest.mark.parametrize("d1,d2", [(256, 256), (64, 48), (40, 24)])
def test_gather_mm_tf32(orc, d1, d2):
    rng = np.random.default_rng(d1 + d2)
    n, r = 7000, 9
    a = rng.normal(0, 0.05, size=(n, d1)).astype(np.float32)
    b = rng.normal(0, 0.05, size=(r, d1, d2)).astype(np.float32)
    idx = rng.integers(0, r, n)
    idx[idx == 4] = 5  # one relation with no rows
    got = ops.gather_mm(a, b, idx_b=idx)
    no_device_error()
    within_s(got, orc.gather_mm(a, b, idx), orc.gather_mm(np.abs(a), np.abs(b), idx))


def test_bf16_tensors(orc):
    rng = np.random.default_rng(77)
    n, r, d1, d2 = 6000, 5, 256, 256
    seglen = segments(rng, n, r)
    a = torch.from_numpy(rng.normal(0, 0.05, size=(n, d1))).to(torch.bfloat16).cuda()
    b = torch.from_numpy(rng.normal(0, 0.05, size=(r, d1, d2))).to(torch.bfloat16).cuda()
    got = ops.segment_mm(a, b, seglen)
    no_device_error()
    assert got.dtype == torch.bfloat16 and got.is_cuda
    a64, b64 = a.double().cpu().numpy(), b.double().cpu().numpy()
    within_s(got.float().cpu().numpy(), orc.segment_mm(a64, b64, seglen),
             orc.segment_mm(np.abs(a64), np.abs(b64), seglen))
    idx = rng.integers(0, r, n)
    got = ops.gather_mm(a, b, idx_b=idx)
    no_device_error()
    within_s(got.float().cpu().numpy(), orc.gather_mm(a64, b64, idx),
             orc.gather_mm(np.abs(a64), np.abs(b64), idx))


def test_config4_shape_checksum(orc):
    """BASELINE config 4's shapes at full size (2M x 256 by 64 x 256 x 256):
    a seeded sample of rows against the oracle's segment_mm and gather_mm, and
    a size-independent property -- the column sums of out equal
    sum_r (column sums of a's rows of segment r) @ b[r]."""
    rng = np.random.default_rng(4)
    n, r, d = 2_000_000, 64, 256
    a = torch.empty((n, d), device="cuda").normal_(0, 0.05, generator=torch.Generator("cuda").manual_seed(4))
    b = torch.empty((r, d, d), device="cuda").normal_(0, 0.05, generator=torch.Generator("cuda").manual_seed(5))
    seglen = rng.multinomial(n, rng.dirichlet(0.5 * np.ones(r)))
    out = ops.segment_mm(a, b, seglen)
    no_device_error()
    off = np.concatenate([[0], np.cumsum(seglen)])
    colsum = torch.zeros(d, dtype=torch.float64, device="cuda")
    for i in range(r):
        if seglen[i]:
            colsum += a[off[i]:off[i + 1]].double().sum(0) @ b[i].double()
    np.testing.assert_allclose(out.double().sum(0).cpu().numpy(), colsum.cpu().numpy(),
                               rtol=2e-2, atol=2e-2 * float(colsum.abs().max()))
    # sampled rows, the first and last row of every segment included: the
    # oracle runs segment_mm on the sampled rows grouped by their relation
    edges = np.concatenate([off[:-1][seglen > 0], off[1:][seglen > 0] - 1])
    rows = np.unique(np.concatenate([rng.choice(n, 2000, replace=False), edges]))
    rel = np.searchsorted(off, rows, side="right") - 1
    rows_t = torch.from_numpy(rows).cuda()
    a_s = a[rows_t].double().cpu().numpy()
    b_np = b.double().cpu().numpy()
    seglen_s = np.bincount(rel, minlength=r)
    within_s(out[rows_t].double().cpu().numpy(), orc.segment_mm(a_s, b_np, seglen_s),
             orc.segment_mm(np.abs(a_s), np.abs(b_np), seglen_s))
    del out
    # gather_mm at the same size, uniform relation ids (the reference's
    # segment route at this shape), on the same sample
    idx = rng.integers(0, r, n)
    got = ops.gather_mm(a, b, idx_b=torch.from_numpy(idx).cuda())
    no_device_error()
    within_s(got[rows_t].double().cpu().numpy(), orc.gather_mm(a_s, b_np, idx[rows]),
             orc.gather_mm(np.abs(a_s), np.abs(b_np), idx[rows]))
