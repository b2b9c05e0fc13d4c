"""swx_scan_bwd_static_scratch: the scan backward for callers that cannot allocate.

Some callers cannot call cudaMalloc -- a process that reserved all of its device memory
at start-up and forbids later allocations, or a binding that only receives ready-made
buffers -- so this entry point takes its scratch from a fixed array inside the library
instead of a caller-provided workspace.  The test calls it through the C ABI, twice in
a row (the second call reuses the array the first one left behind), and checks both
results against the regular swx_scan_bwd with the tolerance of the other scan tests.
It also checks that a problem too large for the array is rejected before any launch.
The file is named to be collected last, so a run that stops at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from swiftx_b200 import _lib
from swiftx_b200.selective_scan import _fill_inputs, _prep, scan_backward, scan_forward
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _static_scratch_backward(lib, inp, ck):
    """Same arguments as scan_backward, but through swx_scan_bwd_static_scratch and with
    no workspace passed."""
    u, delta, A, B, C, D, z, bias, h0, in_dt = _prep(inp["u"], inp["delta"], inp["A"], inp["B"],
                                                     inp["C"], inp["D"], inp["z"], inp["delta_bias"], None)
    b, L, Dm = u.shape
    N = A.shape[1]
    dout = inp["dout"].contiguous()
    e = lambda *s, dt=in_dt: torch.full(s, float("nan"), device=DEV, dtype=dt)  # noqa: E731
    g = {"du": e(b, L, Dm), "ddelta": e(b, L, Dm), "dz": e(b, L, Dm), "dB": e(b, L, N), "dC": e(b, L, N),
         "dA": e(Dm, N, dt=torch.float32), "dD": e(Dm, dt=torch.float32),
         "ddelta_bias": e(Dm, dt=torch.float32)}
    a = _lib.ScanArgs()
    _fill_inputs(a, u, delta, A, B, C, D, z, bias, h0, True, in_dt)
    a.out_dtype = a.in_dtype
    a.checkpoints = ck.data_ptr()
    a.dout, a.dout_sb, a.dout_sl = dout.data_ptr(), dout.stride(0), dout.stride(1)
    for k, v in g.items():
        setattr(a, k, v.data_ptr())
    a.workspace, a.workspace_bytes = None, 0
    status = lib.swx_scan_bwd_static_scratch(ctypes.byref(a), _lib.stream_ptr(torch.device(DEV)))
    assert status == _lib.SWX_OK, lib.swx_status_string(status)
    torch.cuda.synchronize()
    return g


def test_static_scratch_backward_matches_allocating_backward():
    lib = _lib.load()
    b, L, Dm, N = 2, 300, 96, 16
    assert lib.swx_scan_bwd_workspace_bytes(b, L, Dm) <= _lib.SWX_STATIC_SCRATCH_BYTES
    inp = config_inputs(b, L, Dm, N, seed=21, device=DEV)
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    _, ck, _ = scan_forward(*args, checkpoints=True)
    want = scan_backward(*args, None, ck, inp["dout"])
    first = _static_scratch_backward(lib, inp, ck)
    # a second call on a different problem, then the first problem again: the array keeps
    # the last call's contents, which must not leak into the next result
    inp2 = config_inputs(1, 100, 64, N, seed=22, device=DEV)
    args2 = (inp2["u"], inp2["delta"], inp2["A"], inp2["B"], inp2["C"], inp2["D"], inp2["z"],
             inp2["delta_bias"], True)
    _, ck2, _ = scan_forward(*args2, checkpoints=True)
    want2 = scan_backward(*args2, None, ck2, inp2["dout"])
    got2 = _static_scratch_backward(lib, inp2, ck2)
    second = _static_scratch_backward(lib, inp, ck)
    for got, ref in ((first, want), (second, want), (got2, want2)):
        for k, v in ref.items():
            if v is None:
                continue
            np.testing.assert_allclose(got[k].double().cpu().numpy(), v.double().cpu().numpy(),
                                       rtol=1e-4, atol=1e-5, err_msg=k)


def test_static_scratch_rejects_problems_beyond_capacity():
    lib = _lib.load()
    a = _lib.ScanArgs()
    a.batch, a.seqlen, a.dim, a.dstate = 64, 65536, 2048, 16          # needs ~34 GB of scratch
    assert lib.swx_scan_bwd_workspace_bytes(64, 65536, 2048) > _lib.SWX_STATIC_SCRATCH_BYTES
    assert lib.swx_scan_bwd_static_scratch(ctypes.byref(a), None) == _lib.SWX_ERR_INVALID_ARG
