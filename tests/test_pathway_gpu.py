"""The SiftX pathway mix fused into the scan's gate, against the float64 oracle.

The reference block (models/sift_block.py:130-142) computes y = scan + D*u, then
y * w[..., group_of] with per-token group weights w = softmax(pathway(x)) * G, then the
SiLU(z) gate.  selective_scan_fn(..., group_w=w, group_of=...) does the mix inside the
kernels.  Expected values: the oracle's ungated scan y, mixed and gated in float64; the
gradients of every scan input from the oracle's backward with dout scaled by the group
weight (the mix multiplies the gate's input), and the group weights' gradient
sum_{d in g} dout * silu(z) * y in float64.  Both backward kernels are covered: the
time-segmented one (fp32 problems) and the whole-row one (bf16 problems whose
32-channel x row grid fills the GPU).

Tolerances: fp32 rtol 1e-4 / atol 1e-5, sums scaled by their magnitude as in
tests/test_scan_gpu.py; bf16 inputs rtol 2e-2, atol 2e-2 of each quantity's magnitude.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200 import selective_scan_fn
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def n64(t):
    return t.detach().double().cpu().numpy()


def _groups(D, G, contiguous, seed):
    if contiguous:                     # the reference's layout: nearly equal consecutive ranges
        edges = [round(i * D / G) for i in range(G + 1)]
        gof = np.concatenate([np.full(edges[i + 1] - edges[i], i) for i in range(G)])
    else:
        gof = np.random.default_rng(seed).integers(0, G, D)
    return torch.from_numpy(gof).to(DEV)


def _expected(inp, w, gof):
    args = [n64(inp[k]) for k in ("u", "delta", "A", "B", "C")]
    kw = dict(D=n64(inp["D"]), delta_bias=n64(inp["delta_bias"]), delta_softplus=True)
    y = oracle.scan_fwd(*args, **kw)                                   # ungated, D skip included
    z = n64(inp["z"])
    silu = z / (1.0 + np.exp(-z))
    wd = n64(w)[..., gof.cpu().numpy()]                                # (b, L, D)
    out = y * wd * silu
    dout = n64(inp["dout"])
    g = oracle.scan_bwd(*args, dout * wd, z=z, **kw)
    G = w.shape[-1]
    contrib = dout * silu * y
    dgw = np.stack([contrib[..., gof.cpu().numpy() == k].sum(-1) for k in range(G)], -1)
    # magnitudes for the sums' tolerances
    absargs = [np.abs(a) for a in args]
    absargs[2] = -absargs[2]
    scale = oracle.scan_bwd(*absargs, np.abs(dout * wd), z=np.abs(z), D=np.abs(kw["D"]),
                            delta_bias=kw["delta_bias"], delta_softplus=True)
    dgw_scale = np.stack([np.abs(contrib)[..., gof.cpu().numpy() == k].sum(-1) for k in range(G)], -1)
    return out, g, dgw, scale, dgw_scale


def _run(inp, w, gof):
    keys = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]
    t = {k: inp[k].clone().requires_grad_() for k in keys}
    wt = w.clone().requires_grad_()
    out = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], z=t["z"],
                            delta_bias=t["delta_bias"], delta_softplus=True, group_w=wt, group_of=gof)
    out.backward(inp["dout"])
    grads = {"du": t["u"].grad, "ddelta": t["delta"].grad, "dA": t["A"].grad, "dB": t["B"].grad,
             "dC": t["C"].grad, "dD": t["D"].grad, "dz": t["z"].grad, "ddelta_bias": t["delta_bias"].grad}
    return out, grads, wt.grad


def _weights(b, L, G, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.softmax(torch.randn(b, L, G, generator=g), -1) * G).to(DEV)


@pytest.mark.parametrize("G,contiguous", [(3, True), (1, True), (8, False)])
def test_mix_fp32_segmented_backward_vs_oracle(G, contiguous):
    b, L, D, N = 2, 300, 96, 16
    inp = config_inputs(b, L, D, N, seed=31, device=DEV)
    w, gof = _weights(b, L, G, 1), _groups(D, G, contiguous, 2)
    out, grads, dgw = _run(inp, w, gof)
    want, g, dgw_want, scale, dgw_scale = _expected(inp, w, gof)
    np.testing.assert_allclose(n64(out), want, rtol=1e-4, atol=1e-5)
    for k, v in g.items():
        tol = 1e-5 + (1e-5 * np.abs(scale[k]) if k in ("dA", "dD", "ddelta_bias", "dB", "dC") else 0.0)
        err = np.abs(n64(grads[k]) - v)
        assert (err <= tol + 1e-4 * np.abs(v)).all(), (k, err.max())
    err = np.abs(n64(dgw) - dgw_want)
    assert (err <= 1e-5 + 1e-5 * dgw_scale + 1e-4 * np.abs(dgw_want)).all(), err.max()


def test_mix_bf16_row_backward_vs_oracle():
    """bf16 with a grid of 16 channel blocks x 10 rows (> 148 SMs): the whole-row kernel."""
    b, L, D, N = 10, 64, 512, 16
    inp = config_inputs(b, L, D, N, seed=32, device=DEV, dtype=torch.bfloat16)
    w, gof = _weights(b, L, 3, 3), _groups(D, 3, True, 0)
    out, grads, dgw = _run(inp, w, gof)
    want, g, dgw_want, _, dgw_scale = _expected(inp, w, gof)
    np.testing.assert_allclose(n64(out), want, rtol=2e-2, atol=2e-2 * np.abs(want).max())
    for k, v in g.items():
        np.testing.assert_allclose(n64(grads[k]), v, rtol=2e-2, atol=2e-2 * np.abs(v).max(), err_msg=k)
    np.testing.assert_allclose(n64(dgw), dgw_want, rtol=2e-2, atol=2e-2 * np.abs(dgw_want).max())


def test_mix_gradients_deterministic():
    b, L, D, N = 2, 200, 80, 16
    inp = config_inputs(b, L, D, N, seed=33, device=DEV)
    w, gof = _weights(b, L, 3, 4), _groups(D, 3, True, 0)
    _, g1, d1 = _run(inp, w, gof)
    _, g2, d2 = _run(inp, w, gof)
    assert torch.equal(d1, d2)
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_mix_with_unit_weights_is_the_plain_gate():
    """w = 1 everywhere (the pathway's initial state) gives exactly the gated scan."""
    b, L, D, N = 2, 130, 64, 16
    inp = config_inputs(b, L, D, N, seed=34, device=DEV)
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"])
    plain = selective_scan_fn(*args, z=inp["z"], delta_bias=inp["delta_bias"], delta_softplus=True)
    mixed = selective_scan_fn(*args, z=inp["z"], delta_bias=inp["delta_bias"], delta_softplus=True,
                              group_w=torch.ones(b, L, 3, device=DEV), group_of=_groups(D, 3, True, 0))
    assert torch.equal(plain, mixed)


@pytest.mark.parametrize("D,N", [(2048, 16), (96, 12)])
def test_decode_step_mix_matches_unfused(D, N):
    """decode_ssm_step with the group weights (the streaming kernel at D=2048, N=16; the
    general kernel at D=96, N=12) equals the step without the gate followed by the mix
    and gate in float64, and updates the state identically."""
    from swiftx_b200.decode import decode_ssm_step
    b, G = 6, 3
    g = torch.Generator().manual_seed(9)
    r = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc).to(DEV)  # noqa: E731
    xc, z, dl = r(b, D), r(b, D), r(b, D, sc=0.5)
    Bm, Cm = r(b, N), r(b, N)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).to(DEV)
    Dsk, bias = r(D), r(D, sc=0.1)
    h = r(b, D, N, sc=0.1)
    w = (torch.softmax(torch.randn(b, G, generator=g), -1) * G).to(DEV)
    gof = _groups(D, G, True, 0)
    h1, h2 = h.clone(), h.clone()
    fused = decode_ssm_step(xc, dl, Bm, Cm, A, h1, Dskip=Dsk, z=z, delta_bias=bias, group_w=w, group_of=gof)
    y = decode_ssm_step(xc, dl, Bm, Cm, A, h2, Dskip=Dsk, delta_bias=bias)
    want = n64(y) * n64(w)[:, gof.cpu().numpy()] * n64(z) / (1.0 + np.exp(-n64(z)))
    np.testing.assert_allclose(n64(fused), want, rtol=1e-5, atol=1e-6)
    assert torch.equal(h1, h2)
