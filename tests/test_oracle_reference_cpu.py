"""The oracle against the reference's own computation on seeded random problems (CPU, float64).

The golden fixtures pin the oracle on fixed cases; this test draws further shapes and
options and compares the oracle's forward and every gradient with the reference computed
in float64 under autograd: the block's expression around the scan,
out = selective_scan_ref(u, softplus(delta + bias), A, B, C, D) * silu(z)
(models/selective_scan.py:34-60, models/sift_block.py:108,134), with the softplus, the
gate and the D skip each switched on or off (skipped where the reference checkout is not
available; set SWIFTX_REFERENCE to point at one), and the decode oracle against the
reference's own SiftBlock.step over several tokens.  The block's causal conv + SiLU is
torch's depthwise Conv1d in the reference, so its check needs no checkout.
"""
import importlib
import os
import sys

import numpy as np
import pytest
import torch

import oracle

REF = os.environ.get("SWIFTX_REFERENCE", "/root/reference")
needs_reference = pytest.mark.skipif(not os.path.isfile(os.path.join(REF, "models", "selective_scan.py")),
                                     reason="reference checkout not available")

CASES = [((2, 33, 7, 5), dict(gate=True, softplus=True, skip=True)),
         ((1, 50, 16, 16), dict(gate=False, softplus=True, skip=True)),
         ((3, 17, 9, 1), dict(gate=True, softplus=False, skip=False)),
         ((2, 1, 4, 3), dict(gate=True, softplus=True, skip=False)),
         ((1, 64, 3, 12), dict(gate=False, softplus=False, skip=True))]


@pytest.fixture(scope="module")
def reference_models():
    """Importer of the reference checkout's models.* modules, removed afterwards."""
    sys.path.insert(0, REF)
    try:
        yield lambda name: importlib.import_module(f"models.{name}")
    finally:
        sys.path.remove(REF)
        for name in [m for m in sys.modules if m == "models" or m.startswith("models.")]:
            del sys.modules[name]


@pytest.fixture(scope="module")
def reference_scan(reference_models):
    return reference_models("selective_scan").selective_scan_ref


@needs_reference
@pytest.mark.parametrize("shape,opts", CASES, ids=[f"{s}-{''.join(k[0] for k, v in o.items() if v)}" for s, o in CASES])
def test_oracle_matches_reference_expression(reference_scan, shape, opts):
    b, L, D, N = shape
    g = torch.Generator().manual_seed(1000 + b * L * D * N)
    rn = lambda *s, sc=1.0: (torch.randn(*s, generator=g, dtype=torch.float64) * sc)  # noqa: E731
    u, z, dout = rn(b, L, D), rn(b, L, D), rn(b, L, D)
    delta = rn(b, L, D, sc=0.5) if opts["softplus"] else torch.rand(b, L, D, generator=g, dtype=torch.float64) * 0.2
    bias = rn(D, sc=0.5) - 2.0
    A = -torch.exp(torch.rand(D, N, generator=g, dtype=torch.float64) * 2.0)
    Bm, Cm, Dv = rn(b, L, N), rn(b, L, N), rn(D)

    leaves = {k: t.clone().requires_grad_() for k, t in
              dict(u=u, delta=delta, A=A, B=Bm, C=Cm, D=Dv, z=z, bias=bias).items()}
    t = leaves
    dl = t["delta"] + t["bias"]
    dl = torch.nn.functional.softplus(dl) if opts["softplus"] else dl
    y = reference_scan(t["u"], dl, t["A"], t["B"], t["C"], t["D"] if opts["skip"] else None)
    out = y * torch.nn.functional.silu(t["z"]) if opts["gate"] else y
    out.backward(dout)

    n = lambda x: x.detach().numpy()  # noqa: E731
    kw = dict(D=n(Dv) if opts["skip"] else None, z=n(z) if opts["gate"] else None, delta_bias=n(bias),
              delta_softplus=opts["softplus"])
    args = [n(x) for x in (u, delta, A, Bm, Cm)]
    np.testing.assert_allclose(oracle.scan_fwd(*args, **kw), n(out), rtol=1e-10, atol=1e-12)
    got = oracle.scan_bwd(*args, n(dout), **kw)
    want = dict(du="u", ddelta="delta", dA="A", dB="B", dC="C", ddelta_bias="bias")
    if opts["skip"]:
        want["dD"] = "D"
    if opts["gate"]:
        want["dz"] = "z"
    for k, leaf in want.items():
        np.testing.assert_allclose(got[k], n(leaves[leaf].grad), rtol=1e-9, atol=1e-11, err_msg=k)


@pytest.mark.parametrize("b,L,D,K,bias", [(2, 19, 6, 4, True), (1, 3, 5, 4, True), (3, 40, 8, 2, False),
                                          (2, 11, 7, 3, True)])
def test_conv_oracle_matches_block_expression(b, L, D, K, bias):
    """The block's causal conv + SiLU as the reference computes it (models/sift_block.py:
    62-65,117-118: depthwise Conv1d with padding K-1, the first L outputs, then SiLU),
    forward and gradients in float64 under autograd, against oracle.conv1d_fwd / _bwd."""
    g = torch.Generator().manual_seed(2000 + b * L * D * K)
    x = torch.randn(b, L, D, generator=g, dtype=torch.float64, requires_grad=True)
    w = (torch.randn(D, 1, K, generator=g, dtype=torch.float64) * 0.5).requires_grad_()
    cb = torch.randn(D, generator=g, dtype=torch.float64, requires_grad=True) if bias else None
    dout = torch.randn(b, L, D, generator=g, dtype=torch.float64)
    y = torch.nn.functional.conv1d(x.transpose(1, 2), w, cb, padding=K - 1, groups=D)[..., :L].transpose(1, 2)
    y = torch.nn.functional.silu(y)
    y.backward(dout)
    n = lambda t: None if t is None else t.detach().numpy()  # noqa: E731
    np.testing.assert_allclose(oracle.conv1d_fwd(n(x), n(w), n(cb)), n(y), rtol=1e-12, atol=1e-13)
    dx, dw, db = oracle.conv1d_bwd(n(x), n(w), n(cb), n(dout))
    np.testing.assert_allclose(dx, n(x.grad), rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(dw, n(w.grad).reshape(D, K), rtol=1e-11, atol=1e-12)
    if bias:
        np.testing.assert_allclose(db, n(cb.grad), rtol=1e-11, atol=1e-12)
    else:
        assert db is None


@needs_reference
@pytest.mark.parametrize("b,d_model,d_state,d_conv", [(2, 12, 5, 3), (4, 16, 16, 4)])
def test_decode_oracle_matches_block_step(reference_models, b, d_model, d_state, d_conv):
    """oracle.decode_step against the reference's own SiftBlock.step (models/sift_block.py:
    153-175) in float64 over four tokens: the step's inputs to the state update (x, z, the
    dt projection, B, C) are captured from the block as it runs, and the oracle, fed them
    and the previous states, must give the block's gated output and both new states."""
    SiftBlock = reference_models("sift_block").SiftBlock
    torch.manual_seed(b * d_model + d_state)
    blk = SiftBlock(d_model=d_model, d_state=d_state, d_conv=d_conv, expand=2).double()
    conv_state, ssm_state = blk.allocate_state(b, dtype=torch.float64)
    g = torch.Generator().manual_seed(5)
    conv_state.copy_(torch.randn(conv_state.shape, dtype=torch.float64, generator=g))
    ssm_state.copy_(0.1 * torch.randn(ssm_state.shape, dtype=torch.float64, generator=g))
    cap = {}
    fwd = {k: getattr(blk, k).forward for k in ("in_proj", "x_proj", "dt_proj")}
    blk.in_proj.forward = lambda h: cap.setdefault("xz", fwd["in_proj"](h))
    blk.x_proj.forward = lambda t: cap.setdefault("xdbl", fwd["x_proj"](t))
    blk.dt_proj.forward = lambda t: cap.setdefault("dr", fwd["dt_proj"](t))
    blk.out_proj.forward = lambda y: cap.setdefault("y", y)
    A = -torch.exp(blk.A_log.float()).double()                  # as the block forms it
    n = lambda t: t.detach().numpy()  # noqa: E731
    cs, ss = n(conv_state).copy(), n(ssm_state).copy()
    for _ in range(4):
        cap.clear()
        with torch.no_grad():
            blk.step(torch.randn(b, d_model, dtype=torch.float64, generator=g), (conv_state, ssm_state))
        x, z = cap["xz"].chunk(2, dim=-1)
        _, Bm, Cm = torch.split(cap["xdbl"], [blk.dt_rank, d_state, d_state], dim=-1)
        out, cs, ss, _ = oracle.decode_step(n(x), n(z), n(cap["dr"]), n(Bm), n(Cm), n(blk.conv1d.weight.squeeze(1)),
                                            n(blk.conv1d.bias), n(A), n(blk.D), None, cs, ss, delta_softplus=True)
        np.testing.assert_allclose(out, n(cap["y"]), rtol=1e-11, atol=1e-12)
        np.testing.assert_allclose(cs, n(conv_state), rtol=0, atol=0)
        np.testing.assert_allclose(ss, n(ssm_state), rtol=1e-11, atol=1e-12)
