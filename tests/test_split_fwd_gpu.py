"""The split forward (SWX_SCAN_SPLIT_FWD): a small batch's long rows cut into segments
scanned in parallel from zero states, the segments' end states combined in order, and
every later segment's output, checkpoints and pre-gate output corrected for its initial
state.  Against the whole-row forward of the same kernels and against the oracle; the
backward run on the split forward's checkpoints must match the oracle as well.

Tolerances: fp32 rtol 1e-4 / atol 1e-5 (sums over many terms scaled by their magnitude,
as in tests/test_scan_gpu.py); bf16 inputs rtol 2e-2 of each quantity's magnitude.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200 import _lib, selective_scan_fn
from swiftx_b200.selective_scan import _fill_inputs, _prep, scan_forward
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def n64(t):
    return None if t is None else t.detach().double().cpu().numpy()


def _split_bytes(inp):
    a = _lib.ScanArgs()
    u, dl, A, Bm, Cm, Dv, z, bias, h0, in_dt = _prep(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"],
                                                     inp["D"], inp["z"], inp["delta_bias"], None)
    _fill_inputs(a, u, dl, A, Bm, Cm, Dv, z, bias, h0, True, in_dt)
    a.out = 16                                       # only its presence matters to the plan
    a.flags |= _lib.SWX_SCAN_SPLIT_FWD
    return _lib.load().swx_scan_fwd_workspace_bytes(a)


def test_plan_splits_only_small_batches_of_long_rows():
    assert _split_bytes(config_inputs(1, 16384, 512, 16, device=DEV)) > 0
    assert _split_bytes(config_inputs(8, 2048, 512, 16, device=DEV)) == 0       # fills the GPU, short
    assert _split_bytes(config_inputs(1, 2048, 512, 16, device=DEV)) == 0       # segments would be short
    assert _split_bytes(config_inputs(1, 16392, 512, 16, device=DEV)) == 0      # no 16-step-aligned cut


def _forward(inp, h0, split, dtype_out=torch.float32):
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32)
    out, ck, hl, ds = scan_forward(*args, h0=h0, out_dtype=dtype_out, checkpoints=True, return_last_state=True,
                                   return_delta_sum=True, pre_out=pre, split=split)
    return out, ck, hl, ds, pre


@pytest.mark.parametrize("with_h0", [False, True])
def test_split_forward_matches_whole_rows_and_oracle(with_h0):
    b, L, D, N = 1, 16384, 256, 16
    inp = config_inputs(b, L, D, N, seed=51, device=DEV)
    assert _split_bytes(inp) > 0
    h0 = (torch.randn(b, D, N, generator=torch.Generator().manual_seed(2)) * 0.5).to(DEV) if with_h0 else None
    got = _forward(inp, h0, True)
    whole = _forward(inp, h0, False)
    names = ("out", "checkpoints", "h_last", "delta_sum", "pre-gate output")
    for g, w, name in zip(got, whole, names):
        w64 = n64(w)
        np.testing.assert_allclose(n64(g), w64, rtol=1e-4, atol=1e-5 * max(1.0, np.abs(w64).max()), err_msg=name)
    want, hl = oracle.scan_fwd(*(n64(inp[k]) for k in ("u", "delta", "A", "B", "C")), D=n64(inp["D"]),
                               z=n64(inp["z"]), delta_bias=n64(inp["delta_bias"]), delta_softplus=True,
                               h0=n64(h0), return_last_state=True)
    np.testing.assert_allclose(n64(got[0]), want, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(n64(got[2]), hl, rtol=1e-4, atol=1e-5)


def test_backward_on_split_forward_vs_oracle():
    """Autograd through selective_scan_fn: the forward splits, the backward reads its
    corrected checkpoints and pre-gate output."""
    b, L, D, N = 1, 8192, 128, 16
    inp = config_inputs(b, L, D, N, seed=52, device=DEV)
    assert _split_bytes(inp) > 0
    keys = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]
    t = {k: inp[k].clone().requires_grad_() for k in keys}
    out = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], z=t["z"],
                            delta_bias=t["delta_bias"], delta_softplus=True)
    out.backward(inp["dout"])
    args = [n64(inp[k]) for k in ("u", "delta", "A", "B", "C")]
    kw = dict(D=n64(inp["D"]), z=n64(inp["z"]), delta_bias=n64(inp["delta_bias"]), delta_softplus=True)
    want = oracle.scan_bwd(*args, n64(inp["dout"]), **kw)
    absargs = [np.abs(x) for x in args]
    absargs[2] = -absargs[2]
    scale = oracle.scan_bwd(*absargs, np.abs(n64(inp["dout"])), D=np.abs(kw["D"]), z=np.abs(kw["z"]),
                            delta_bias=kw["delta_bias"], delta_softplus=True)
    got = {"du": t["u"].grad, "ddelta": t["delta"].grad, "dA": t["A"].grad, "dB": t["B"].grad, "dC": t["C"].grad,
           "dD": t["D"].grad, "dz": t["z"].grad, "ddelta_bias": t["delta_bias"].grad}
    for k, v in want.items():
        tol = 1e-5 + (1e-5 * np.abs(scale[k]) if k in ("dA", "dD", "ddelta_bias", "dB", "dC") else 0.0)
        err = np.abs(n64(got[k]) - v)
        assert (err <= tol + 1e-4 * np.abs(v)).all(), (k, err.max())


def test_split_forward_bf16_and_pathway_mix():
    """bf16 inputs with the SiftX group weights fused into the gate: split against whole rows."""
    b, L, D, N = 2, 8192, 128, 16
    inp = config_inputs(b, L, D, N, seed=53, device=DEV, dtype=torch.bfloat16)
    assert _split_bytes(inp) > 0
    g = torch.Generator().manual_seed(4)
    w = (torch.softmax(torch.randn(b, L, 3, generator=g), -1) * 3).to(DEV)
    gof = torch.tensor([0] * 43 + [1] * 42 + [2] * 43, device=DEV)
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    res = [scan_forward(*args, out_dtype=torch.float32, group_w=w, group_of=gof, split=s)[0] for s in (True, False)]
    want = n64(res[1])
    np.testing.assert_allclose(n64(res[0]), want, rtol=2e-2, atol=2e-2 * np.abs(want).max())


def test_split_forward_partial_block_small_state_a_log():
    """N < 16, a partial 32-channel block and A given as log(-A): split against whole rows
    and the oracle, final state included."""
    b, L, D, N = 1, 8192, 200, 12
    inp = config_inputs(b, L, D, N, seed=54, device=DEV)
    assert _split_bytes(inp) > 0
    A_log = torch.log(-inp["A"])
    h0 = (torch.randn(b, D, N, generator=torch.Generator().manual_seed(5)) * 0.3).to(DEV)
    args = (inp["u"], inp["delta"], A_log, inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    res = [scan_forward(*args, h0=h0, return_last_state=True, A_is_log=True, split=s) for s in (True, False)]
    for g, w, name in zip(res[0], res[1], ("out", "checkpoints", "h_last")):
        if g is not None:
            np.testing.assert_allclose(n64(g), n64(w), rtol=1e-4, atol=1e-5, err_msg=name)
    want, hl = oracle.scan_fwd(*(n64(inp[k]) for k in ("u", "delta", "A", "B", "C")), D=n64(inp["D"]),
                               z=n64(inp["z"]), delta_bias=n64(inp["delta_bias"]), delta_softplus=True,
                               h0=n64(h0), return_last_state=True)
    np.testing.assert_allclose(n64(res[0][0]), want, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(n64(res[0][2]), hl, rtol=1e-4, atol=1e-5)
