"""Seeded sweep of problem shapes and options through the forward and backward kernels,
against the float64 oracle.

Each case draws (b, L, D, N) -- sequence lengths that are and are not multiples of the
16-step checkpoint chunk, channel counts with partial 32- and 64-channel blocks, state
counts below 16 -- and the options of selective_scan_fn: the SiLU gate, softplus(delta +
bias) or a plain delta, the D skip, an initial state, A given as log(-A), and u / z as
the strided halves of one (b, L, 2D) tensor (the in_proj output of the Sift block,
models/sift_block.py:108-117).  The backward plan (segment count, sub-segment length,
whole-row kernel for bf16 grids that fill the GPU) follows from the shape, so the sweep
crosses many plans.

Tolerances as in tests/test_scan_gpu.py: fp32 rtol 1e-4 / atol 1e-5, sums scaled by the
magnitude of their terms (1e-5 of the oracle's sum over |terms|); bf16 inputs with fp32
state rtol 2e-2 with atol 2e-2 of each quantity's magnitude.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.selective_scan import scan_backward, scan_forward

pytestmark = pytest.mark.gpu
DEV = "cuda"
SUMS = ("dA", "dD", "ddelta_bias", "dB", "dC", "dh0")


def np64(t):
    return None if t is None else t.detach().cpu().double().numpy()


def _case(i):
    r = np.random.default_rng(7000 + i)
    b = int(r.choice([1, 2, 3, 5]))
    L = int(r.choice([1, 7, 16, 33, 129, 257, 640, 1000, 1203]))
    D = int(r.choice([1, 5, 31, 40, 64, 96, 150]))
    N = int(r.choice([1, 4, 12, 16, 16]))
    opts = dict(gate=bool(r.random() < 0.7), softplus=bool(r.random() < 0.7), with_D=bool(r.random() < 0.8),
                h0=bool(r.random() < 0.4), a_log=bool(r.random() < 0.4), strided=bool(r.random() < 0.4))
    return b, L, D, N, opts


def _inputs(b, L, D, N, opts, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s, sc=1.0: torch.randn(*s, generator=g) * sc  # noqa: E731
    if opts["strided"]:                       # u and z: the halves of one (b, L, 2D) tensor
        xz = rn(b, L, 2 * D).to(dtype)
        u, z = xz[..., :D], xz[..., D:]
    else:
        u, z = rn(b, L, D).to(dtype), rn(b, L, D).to(dtype)
    delta = rn(b, L, D, sc=0.5)
    bias = torch.log(torch.expm1(torch.exp(torch.empty(D).uniform_(np.log(1e-3), np.log(1e-1), generator=g))))
    if not opts["softplus"]:                  # a plain, positive delta
        delta = torch.nn.functional.softplus(delta + bias)
    A = -torch.exp(torch.empty(D, N).uniform_(0.0, np.log(16.0), generator=g))
    inp = dict(u=u, delta=delta.to(dtype), A=A, B=rn(b, L, N).to(dtype), C=rn(b, L, N).to(dtype),
               D=rn(D), z=z, delta_bias=bias, dout=rn(b, L, D).to(dtype),
               h0=rn(b, D, N, sc=0.3) if opts["h0"] else None)
    return {k: (v.to(DEV) if v is not None else None) for k, v in inp.items()}


def _oracle(inp, opts):
    kw = dict(D=np64(inp["D"]) if opts["with_D"] else None, z=np64(inp["z"]) if opts["gate"] else None,
              delta_bias=np64(inp["delta_bias"]) if opts["softplus"] else None,
              delta_softplus=opts["softplus"], h0=np64(inp["h0"]))
    args = [np64(inp[k]) for k in ("u", "delta", "A", "B", "C")]
    out, hl = oracle.scan_fwd(*args, return_last_state=True, **kw)
    grads = oracle.scan_bwd(*args, np64(inp["dout"]), **kw)
    absargs = [np.abs(a) for a in args]
    absargs[2] = -absargs[2]
    kwa = dict(kw)
    for k in ("D", "z", "h0"):
        if kwa[k] is not None:
            kwa[k] = np.abs(kwa[k])
    scale = oracle.scan_bwd(*absargs, np.abs(np64(inp["dout"])), **kwa)
    if opts["a_log"]:                         # the kernels return d/dA_log = dA * A
        A = args[2]
        grads["dA"] = grads["dA"] * A
        scale["dA"] = scale["dA"] * np.abs(A)
    return out, hl, grads, scale


def _run(inp, opts):
    A = torch.log(-inp["A"]) if opts["a_log"] else inp["A"]
    Dv = inp["D"] if opts["with_D"] else None
    z = inp["z"] if opts["gate"] else None
    bias = inp["delta_bias"] if opts["softplus"] else None
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32) if z is not None else None
    out, ck, hl = scan_forward(inp["u"], inp["delta"], A, inp["B"], inp["C"], Dv, z, bias, opts["softplus"],
                               h0=inp["h0"], out_dtype=torch.float32, checkpoints=True, return_last_state=True,
                               pre_out=pre, A_is_log=opts["a_log"])
    g = scan_backward(inp["u"], inp["delta"], A, inp["B"], inp["C"], Dv, z, bias, opts["softplus"], inp["h0"], ck,
                      inp["dout"], y_pre=pre, A_is_log=opts["a_log"])
    return out, hl, {k: v for k, v in g.items() if v is not None}


def _check(name, got, want, rtol, atol):
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{name}: {bad.sum()}/{bad.size} out of tolerance, max abs err {err.max():.3g}"


FP32_CASES = [_case(i) for i in range(18)]


@pytest.mark.parametrize("case", FP32_CASES, ids=[f"b{c[0]}-L{c[1]}-D{c[2]}-N{c[3]}" for c in FP32_CASES])
def test_sweep_fp32_vs_oracle(case):
    b, L, D, N, opts = case
    inp = _inputs(b, L, D, N, opts, seed=b * 7919 + L * 31 + D * 7 + N, dtype=torch.float32)
    out_o, hl_o, gr_o, scale = _oracle(inp, opts)
    out, hl, g = _run(inp, opts)
    _check("out", np64(out), out_o, 1e-4, 1e-5)
    _check("h_last", np64(hl), hl_o, 1e-4, 1e-5)
    assert set(g) == set(gr_o), (sorted(g), sorted(gr_o))
    for k, want in gr_o.items():
        atol = 1e-5 + (1e-5 * np.abs(scale[k]) if k in SUMS else 0.0)
        _check(k, np64(g[k]), want, 1e-4, atol)


BF16_CASES = [_case(100 + i) for i in range(6)] + [(12, 96, 512, 16, dict(gate=True, softplus=True, with_D=True,
                                                                           h0=False, a_log=True, strided=True))]


@pytest.mark.parametrize("case", BF16_CASES, ids=[f"b{c[0]}-L{c[1]}-D{c[2]}-N{c[3]}" for c in BF16_CASES])
def test_sweep_bf16_vs_oracle(case):
    """bf16 inputs, fp32 state; the last case is a grid of 16 x 12 row blocks (> 148 SMs),
    which the whole-row backward takes."""
    b, L, D, N, opts = case
    inp = _inputs(b, L, D, N, opts, seed=b * 7919 + L * 31 + D * 7 + N + 1, dtype=torch.bfloat16)
    out_o, hl_o, gr_o, scale = _oracle(inp, opts)
    out, hl, g = _run(inp, opts)
    _check("out", np64(out), out_o, 2e-2, 2e-2 * np.abs(out_o).max())
    _check("h_last", np64(hl), hl_o, 2e-2, 2e-2 * np.abs(hl_o).max())
    for k, want in gr_o.items():
        atol = 2e-2 * np.abs(want).max() + (1e-5 * np.abs(scale[k]).max() if k in SUMS else 0.0)
        _check(k, np64(g[k]), want, 2e-2, atol)
