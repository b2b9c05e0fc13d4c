"""The oracle against the reference's own computation on seeded random problems (CPU, float64).

The golden fixtures pin the oracle on fixed cases; this test draws further shapes and
options and compares the oracle's forward and every gradient with the reference computed
in float64 under autograd: the block's expression around the scan,
out = selective_scan_ref(u, softplus(delta + bias), A, B, C, D) * silu(z)
(models/selective_scan.py:34-60, models/sift_block.py:108,134), with the softplus, the
gate and the D skip each switched on or off (skipped where the reference checkout is not
available; set SWIFTX_REFERENCE to point at one).  The block's causal conv + SiLU is
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
def reference_scan():
    """models.selective_scan imported from the reference checkout, removed afterwards."""
    sys.path.insert(0, REF)
    try:
        mod = importlib.import_module("models.selective_scan")
        yield mod.selective_scan_ref
    finally:
        sys.path.remove(REF)
        for name in [m for m in sys.modules if m == "models" or m.startswith("models.")]:
            del sys.modules[name]


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
