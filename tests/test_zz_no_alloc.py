"""swx_scan_bwd_static_scratch: the scan backward for callers that cannot allocate.

Some callers cannot call cudaMalloc -- a process that reserved all of its device memory
at start-up and forbids later allocations, or a binding that only receives ready-made
buffers -- so this entry point takes its scratch from a fixed array inside the library
instead of a caller-provided workspace.  The test calls it through the C ABI, twice in
a row (the second call reuses the array the first one left behind), and checks every
result against the regular swx_scan_bwd (bit for bit) and against the oracle.
It also checks that a problem too large for the array is rejected before any launch.
The file is named to be collected last, so a run that stops at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
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


def _args(inp):
    return (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)


def _check_vs_oracle(got, inp, rtol, atol_rel):
    """The gradients against the float64 oracle on the same (rounded) inputs."""
    n = lambda t: t.detach().double().cpu().numpy()  # noqa: E731
    want = oracle.scan_bwd(*(n(inp[k]) for k in ("u", "delta", "A", "B", "C")), n(inp["dout"]), D=n(inp["D"]),
                           z=n(inp["z"]), delta_bias=n(inp["delta_bias"]), delta_softplus=True)
    for k, v in want.items():
        np.testing.assert_allclose(n(got[k].float()), v, rtol=rtol, atol=atol_rel * np.abs(v).max() + 1e-5,
                                   err_msg=k)


def test_static_scratch_backward_matches_allocating_backward():
    """Two calls in a row on one problem, a different problem (fp32) in between and a
    bf16 problem with a partial 80-channel block after them: each result equals the
    allocating swx_scan_bwd bit for bit (both are deterministic, fixed-order sums) and
    matches the oracle (fp32 rtol 1e-4; bf16 inputs rtol 2e-2)."""
    lib = _lib.load()
    N = 16
    cases = [config_inputs(2, 300, 96, N, seed=21, device=DEV),
             config_inputs(1, 100, 64, N, seed=22, device=DEV),
             config_inputs(2, 300, 96, N, seed=21, device=DEV),
             config_inputs(2, 130, 80, N, seed=23, device=DEV, dtype=torch.bfloat16)]
    for inp in cases:
        b, L, Dm = inp["u"].shape
        assert lib.swx_scan_bwd_workspace_bytes(b, L, Dm) <= _lib.SWX_STATIC_SCRATCH_BYTES
    results = []
    for inp in cases:
        _, ck, _ = scan_forward(*_args(inp), checkpoints=True)
        want = scan_backward(*_args(inp), None, ck, inp["dout"])
        got = _static_scratch_backward(lib, inp, ck)
        for k, v in want.items():
            if v is not None:
                assert torch.equal(got[k], v), k
        results.append(got)
    for k in results[0]:
        assert torch.equal(results[0][k], results[2][k]), k          # the same problem twice
    _check_vs_oracle(results[0], cases[0], 1e-4, 1e-5)
    _check_vs_oracle(results[3], cases[3], 2e-2, 2e-2)


def test_static_scratch_rejects_problems_beyond_capacity():
    lib = _lib.load()
    a = _lib.ScanArgs()
    a.batch, a.seqlen, a.dim, a.dstate = 64, 65536, 2048, 16          # needs ~34 GB of scratch
    assert lib.swx_scan_bwd_workspace_bytes(64, 65536, 2048) > _lib.SWX_STATIC_SCRATCH_BYTES
    assert lib.swx_scan_bwd_static_scratch(ctypes.byref(a), None) == _lib.SWX_ERR_INVALID_ARG
    # sizes whose product would overflow the workspace arithmetic are rejected up front
    a.batch, a.seqlen, a.dim = 65535, 1 << 30, 1 << 30
    assert lib.swx_scan_bwd_workspace_bytes(a.batch, a.seqlen, a.dim) == -1
    assert lib.swx_scan_bwd_static_scratch(ctypes.byref(a), None) == _lib.SWX_ERR_INVALID_ARG
