"""bgl_gspmm_static_scratch: gSpMM for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc -- a plugin or serving
runtime that owns every device allocation and passes the library only its
input and output buffers, or a request path where an allocation (which can
synchronise the device) is not allowed.  For them the library exports one
entry point that uses a fixed scratch array compiled into the library instead
of a caller workspace.  This test calls it through the C ABI and checks it
against bgl_gspmm with a caller workspace, bit for bit, on two calls in a row
(the second one finds the first one's leftovers in the shared scratch).

The file is named to be collected last, so a run that stops at the first
failure has already run every other test; it passes alone in a fresh process
as well as after the rest of the suite.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from mojodgl import _lib  # noqa: E402


def csr(v, u, n):
    order = np.argsort(v, kind="stable")
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.bincount(v, minlength=n), out=indptr[1:])
    return indptr, u[order].astype(np.int32), order.astype(np.int32)


@pytest.mark.parametrize("reduce_op", ["sum", "max"])
def test_static_scratch_matches_workspace_path(reduce_op):
    lib = _lib.lib()
    rng = np.random.default_rng(2024)
    n, ne, d = 20_000, 300_000, 64
    u = rng.integers(0, n, ne)
    v = rng.integers(0, n, ne)
    v[:6000] = 5  # a hub longer than a merge-path chunk: its row is split into pieces
    indptr, indices, eid = csr(v, u, n)
    h = rng.normal(size=(n, d)).astype(np.float32)
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(a).to(dev) for k, a in
         dict(indptr=indptr, indices=indices, eid=eid, h=h).items()}
    red = _lib.REDUCERS[reduce_op]
    stream = torch.cuda.current_stream().cuda_stream

    def run(static):
        out = torch.full((n, d), float("nan"), device=dev)
        arg = torch.full((n, d), -7, dtype=torch.int64, device=dev) if reduce_op == "max" else None
        argp = arg.data_ptr() if arg is not None else None
        common = (t["indptr"].data_ptr(), t["indices"].data_ptr(), t["eid"].data_ptr(), None, n, ne,
                  t["h"].data_ptr(), d, 1, None, 1, 1, out.data_ptr(), d, argp, None,
                  _lib.BGL_F32, _lib.OP_COPY_LHS, red, 0)
        if static:
            rc = lib.bgl_gspmm_static_scratch(*common, stream)
        else:
            nbytes = lib.bgl_gspmm_workspace_size(n, ne, d, _lib.BGL_F32, red)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            rc = lib.bgl_gspmm(*common, ws.data_ptr(), nbytes, stream)
        assert rc == 0, lib.bgl_last_error()
        torch.cuda.synchronize()
        return out.cpu().numpy(), None if arg is None else arg.cpu().numpy()

    # Both paths run the same plan and kernels, and the split rows' pieces are
    # folded in a fixed order (no float atomics), so the results agree bit for
    # bit; leftovers of the previous call in the shared scratch would show.
    ref, ref_arg = run(static=False)
    for _ in range(2):
        got, got_arg = run(static=True)
        np.testing.assert_array_equal(got, ref)
        if ref_arg is not None:
            np.testing.assert_array_equal(got_arg, ref_arg)


def test_static_scratch_rejects_oversized_calls():
    lib = _lib.lib()
    cap = lib.bgl_static_scratch_bytes()
    assert cap == 64 << 20
    # a plan whose split-row piece buffers exceed the fixed scratch: wide
    # float64 rows with max (values + winning positions per chunk)
    rows, edges, width = 10_000_000, 1_000_000_000, 8192
    need = lib.bgl_gspmm_workspace_size(rows, edges, width, _lib.BGL_F64, _lib.REDUCE_MAX)
    assert need > cap
    rc = lib.bgl_gspmm_static_scratch(None, None, None, None, rows, edges, None, width, 1, None,
                                      1, 1, None, width, None, None, _lib.BGL_F64,
                                      _lib.OP_COPY_LHS, _lib.REDUCE_MAX, 0, None)
    assert rc == 1
    assert b"built-in scratch holds" in lib.bgl_last_error()
