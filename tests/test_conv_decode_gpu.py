"""Parity of the conv1d + SiLU and decode-step kernels with the CPU oracle.

Golden fixtures conv.npz / decode.npz come from the reference's own SiftBlock
(models/sift_block.py:117-118, :153-175).  fp32 tolerance rtol 1e-4 / atol 1e-5.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.conv import causal_conv1d_fn, conv1d_backward, conv1d_forward
from swiftx_b200.decode import decode_conv_step, decode_ssm_step, decode_step

pytestmark = pytest.mark.gpu
DEV = "cuda"


def t(a, dtype=torch.float32):
    return torch.tensor(np.asarray(a), device=DEV, dtype=dtype)


def n64(x):
    return x.detach().double().cpu().numpy()


def close(got, want, rtol=1e-4, atol=1e-5):
    np.testing.assert_allclose(n64(got) if torch.is_tensor(got) else got, want, rtol=rtol, atol=atol)


def test_conv_golden(golden):
    g = golden("conv")
    D = g["w"].shape[0]
    xz = t(g["xz"])
    x = xz[..., :D]                                 # strided view, row stride 2D
    assert x.stride(1) == 2 * D
    w = t(g["w"]).reshape(D, 1, -1).requires_grad_()
    b = t(g["bias"]).requires_grad_()
    xr = x.detach().clone().requires_grad_()
    out = causal_conv1d_fn(xr, w, b)
    close(out, g["out"])
    out.backward(t(g["gout"]))
    close(xr.grad, g["dx"])
    close(w.grad.reshape(D, -1), g["dw"], atol=1e-4)
    close(b.grad, g["dbias"], atol=1e-4)


@pytest.mark.parametrize("shape", [(2, 200, 96, 4), (3, 65, 40, 4), (1, 1, 32, 4), (2, 130, 64, 3),
                                   (2, 70, 33, 2)])
def test_conv_vs_oracle(shape):
    b, L, D, K = shape
    g = torch.Generator().manual_seed(L * 7 + D)
    xz = torch.randn(b, L, 2 * D, generator=g).to(DEV)
    x = xz[..., :D]
    w = (torch.randn(D, K, generator=g) * 0.5).to(DEV)
    bias = torch.randn(D, generator=g).to(DEV)
    dout = torch.randn(b, L, D, generator=g).to(DEV)
    out = conv1d_forward(x, w, bias)
    close(out, oracle.conv1d_fwd(n64(x), n64(w), n64(bias)))
    dx, dw, db = conv1d_backward(x, w, bias, dout)
    odx, odw, odb = oracle.conv1d_bwd(n64(x), n64(w), n64(bias), n64(dout))
    close(dx, odx)
    close(dw, odw, atol=1e-3)          # sums over b*L terms
    close(db, odb, atol=1e-3)


def test_conv_causal_impulse():
    """Impulse response of the conv (tests/test_sift_block.py:38-45 in the reference)."""
    D, L = 32, 10
    x = torch.zeros(1, L, D, device=DEV)
    x[:, 5] = 1.0
    w = torch.randn(D, 4, generator=torch.Generator().manual_seed(0)).to(DEV)
    out = conv1d_forward(x, w, None, silu=False)
    assert torch.all(out[:, :5].abs() < 1e-7)
    assert torch.all(out[:, 9:].abs() < 1e-7)
    assert torch.allclose(out[0, 5:9].T, w.flip(1), atol=1e-6)


def test_conv_bf16():
    b, L, D = 2, 96, 64
    x = torch.randn(b, L, D, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    w = torch.randn(D, 4, generator=torch.Generator().manual_seed(2)).to(DEV)
    out = conv1d_forward(x, w, None)
    assert out.dtype == torch.bfloat16
    close(out.float(), oracle.conv1d_fwd(n64(x.float()), n64(w), None), rtol=2e-2, atol=2e-2)


def test_decode_golden(golden):
    g = golden("decode")
    cs, ss = t(g["conv_state0"]), t(g["ssm_state0"])
    # two launches, as in the model (x_proj / dt_proj sit between them)
    xc = decode_conv_step(t(g["x"]), cs, t(g["conv_w"]), t(g["conv_b"]))
    y = decode_ssm_step(xc, t(g["delta_raw"]), t(g["B"]), t(g["C"]), t(g["A"]), ss, Dskip=t(g["D"]),
                        z=t(g["z"]))
    close(y, g["y"])
    close(cs, np.float32(g["conv_state1"]), atol=0, rtol=0)     # a shift + append: exact
    close(ss, g["ssm_state1"])
    # one fused launch
    cs2, ss2 = t(g["conv_state0"]), t(g["ssm_state0"])
    y2 = decode_step(t(g["x"]), cs2, t(g["conv_w"]), t(g["conv_b"]), t(g["delta_raw"]), t(g["B"]),
                     t(g["C"]), t(g["A"]), ss2, Dskip=t(g["D"]), z=t(g["z"]))
    close(y2, g["y"])
    close(ss2, g["ssm_state1"])


@pytest.mark.parametrize("N", [16, 5])
def test_decode_vs_oracle_multi_step(N):
    b, D, K = 4, 96, 4
    g = torch.Generator().manual_seed(N)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1)
    cw, cb = torch.randn(D, K, generator=g) * 0.5, torch.randn(D, generator=g)
    Dskip, dbias = torch.ones(D), torch.randn(D, generator=g) * 0.5 - 3
    cs = torch.randn(b, D, K, generator=g)
    ss = torch.randn(b, D, N, generator=g) * 0.1
    cs_o, ss_o = cs.double().numpy(), ss.double().numpy()
    csd, ssd = cs.to(DEV), ss.to(DEV)
    for step in range(5):
        x, z, dr = (torch.randn(b, D, generator=g) for _ in range(3))
        Bm, Cm = torch.randn(b, N, generator=g), torch.randn(b, N, generator=g)
        y = decode_step(x.to(DEV), csd, cw.to(DEV), cb.to(DEV), dr.to(DEV), Bm.to(DEV), Cm.to(DEV),
                        A.to(DEV), ssd, Dskip=Dskip.to(DEV), z=z.to(DEV), delta_bias=dbias.to(DEV))
        yo, cs_o, ss_o, _ = oracle.decode_step(x, z, dr, Bm, Cm, cw, cb, A, Dskip, dbias, cs_o, ss_o)
        close(y, yo)
        close(csd, cs_o)
        close(ssd, ss_o)


def _stream_case(b, D, seed):
    N, K = 16, 4
    g = torch.Generator().manual_seed(seed)
    p = {"A": -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1), "cw": torch.randn(D, K, generator=g) * 0.5,
         "cb": torch.randn(D, generator=g), "Dskip": torch.randn(D, generator=g),
         "dbias": torch.randn(D, generator=g) * 0.5 - 3}
    st = {"cs": torch.randn(b, D, K, generator=g), "ss": torch.randn(b, D, N, generator=g) * 0.1}
    steps = [{k: torch.randn(b, n, generator=g) for k, n in (("x", D), ("z", D), ("dr", D), ("B", N), ("C", N))}
             for _ in range(4)]
    return p, st, steps


def _padded(t):
    """The same values with a row stride that is not a multiple of 4 elements, which
    sends the launch to the per-CTA kernel instead of the streaming one."""
    buf = torch.zeros(t.shape[0], t.shape[1] + 1, device=t.device, dtype=t.dtype)
    buf[:, :t.shape[1]] = t
    return buf[:, :t.shape[1]]


@pytest.mark.parametrize("b,D,gate", [(5, 128, True), (3, 256, False), (19, 64, True)])
def test_decode_streaming_path(b, D, gate):
    """D a multiple of 64, N=16, K=4, aligned rows: the persistent streaming kernel.  It
    matches the float64 oracle over several steps (fused launch), matches the per-CTA
    kernel bit for bit on the same values, and the split launch (conv kernel, then the
    state update alone, which also streams) gives the same result."""
    p, st, steps = _stream_case(b, D, seed=b + D)
    dv = {k: v.to(DEV) for k, v in p.items()}
    cs_s, ss_s = st["cs"].to(DEV), st["ss"].to(DEV)            # streaming, fused
    cs_r, ss_r = st["cs"].to(DEV), st["ss"].to(DEV)            # per-CTA kernel, fused
    cs_2, ss_2 = st["cs"].to(DEV), st["ss"].to(DEV)            # streaming, split
    cs_o, ss_o = st["cs"].double().numpy(), st["ss"].double().numpy()
    for s in steps:
        d = {k: v.to(DEV) for k, v in s.items()}
        z = d["z"] if gate else None
        kw = dict(Dskip=dv["Dskip"], delta_bias=dv["dbias"])
        y_s = decode_step(d["x"], cs_s, dv["cw"], dv["cb"], d["dr"], d["B"], d["C"], dv["A"], ss_s, z=z, **kw)
        y_r = decode_step(_padded(d["x"]), cs_r, dv["cw"], dv["cb"], d["dr"], d["B"], d["C"], dv["A"], ss_r,
                          z=z, **kw)
        xc = decode_conv_step(d["x"], cs_2, dv["cw"], dv["cb"])
        y_2 = decode_ssm_step(xc, d["dr"], d["B"], d["C"], dv["A"], ss_2, z=z, **kw)
        yo, cs_o, ss_o, _ = oracle.decode_step(s["x"], s["z"] if gate else None, s["dr"], s["B"], s["C"], p["cw"],
                                               p["cb"], p["A"], p["Dskip"], p["dbias"], cs_o, ss_o)
        close(y_s, yo)
        close(ss_s, ss_o)
        close(cs_s, cs_o)
        assert torch.equal(y_s, y_r) and torch.equal(ss_s, ss_r) and torch.equal(cs_s, cs_r)
        close(y_2, yo)
        assert torch.equal(ss_2, ss_s) and torch.equal(cs_2, cs_s)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("L,K", [(300, 4), (37, 3)])
def test_conv_vector_and_scalar_paths_agree(dtype, L, K):
    """D a multiple of 4 with aligned rows runs the 4-channel forward; the same values in
    a view whose row stride is odd run the one-channel forward.  Outputs are identical
    (same per-channel arithmetic), and so are the gradients of the two layouts."""
    b, D = 3, 128
    g = torch.Generator().manual_seed(L + K)
    x = torch.randn(b, L, D, generator=g).to(DEV, dtype)
    odd = torch.zeros(b, L, D + 1, device=DEV, dtype=dtype)
    odd[..., :D] = x
    xo = odd[..., :D]
    assert xo.stride(1) % 4 != 0
    w = (torch.randn(D, K, generator=g) * 0.5).to(DEV)
    bias = torch.randn(D, generator=g).to(DEV)
    dout = torch.randn(b, L, D, generator=g).to(DEV, dtype)
    assert torch.equal(conv1d_forward(x, w, bias), conv1d_forward(xo, w, bias))
    for got, want in zip(conv1d_backward(x, w, bias, dout), conv1d_backward(xo, w, bias, dout)):
        assert torch.equal(got, want)


@pytest.mark.parametrize("b,D,N", [(5, 128, 16), (3, 96, 16), (4, 64, 5)])
def test_decode_a_log_formed_in_kernel(b, D, N):
    """A_is_log=True (the kernel forms A = -exp(A_log), SiftBlock.step's call) against the
    block's torch expression A = -torch.exp(A_log) passed as A: the same values (the
    kernel's expf is the function torch.exp evaluates), on the streaming kernel (D a
    multiple of 64, N=16), the per-CTA kernel (D=96) and the N < 16 path, over three
    steps of the fused conv + state update."""
    g = torch.Generator().manual_seed(b * D + N)
    A_log = (torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(D, 1)
             + 0.1 * torch.randn(D, N, generator=g)).to(DEV)
    cw, cb = (torch.randn(D, 4, generator=g) * 0.5).to(DEV), torch.randn(D, generator=g).to(DEV)
    Dsk, dbias = torch.randn(D, generator=g).to(DEV), (torch.randn(D, generator=g) * 0.5 - 3).to(DEV)
    cs0, ss0 = torch.randn(b, D, 4, generator=g), torch.randn(b, D, N, generator=g) * 0.1
    states = [(cs0.clone().to(DEV), ss0.clone().to(DEV)) for _ in range(2)]
    for _ in range(3):
        x, z, dr = (torch.randn(b, D, generator=g).to(DEV) for _ in range(3))
        B, C = torch.randn(b, N, generator=g).to(DEV), torch.randn(b, N, generator=g).to(DEV)
        outs = []
        for (cs, ss), in_kernel in zip(states, (False, True)):
            A = A_log if in_kernel else -torch.exp(A_log)
            outs.append(decode_step(x, cs, cw, cb, dr, B, C, A, ss, Dskip=Dsk, z=z, delta_bias=dbias,
                                    A_is_log=in_kernel))
        close(outs[1], n64(outs[0]), rtol=1e-6, atol=1e-7)
        close(states[1][1], n64(states[0][1]), rtol=1e-6, atol=1e-7)
        assert torch.equal(states[1][0], states[0][0])


@pytest.mark.parametrize("D,N,R", [(2048, 16, 64), (96, 12, 20), (512, 16, 128)])
def test_decode_dt_proj_folded(D, N, R):
    """decode_ssm_step with dt_proj folded in (dt_in, dt_weight) against the block's step
    recurrence (models/sift_block.py:167-174) in float64, fed delta = dt_in @ dt_weight.T
    (the streaming kernel for D a multiple of 64 with N=16, the general kernel otherwise);
    dt_in, B and C are strided column slices of an x_proj-like output, as in the block."""
    b = 7
    g = torch.Generator().manual_seed(41)
    r = lambda *s, sc=1.0: torch.randn(*s, generator=g) * sc  # noqa: E731
    xc, z = r(b, D), r(b, D)
    x_dbl = r(b, R + 2 * N, sc=0.3)
    W = r(D, R, sc=R ** -0.5)
    Bm, Cm = x_dbl[:, R:R + N], x_dbl[:, R + N:]
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1)
    Dsk, bias = r(D), r(D, sc=0.1)
    h = r(b, D, N, sc=0.1)
    dev = lambda t: t.to(DEV)  # noqa: E731
    hd = dev(h)
    xd = dev(x_dbl)
    y = decode_ssm_step(dev(xc), None, xd[:, R:R + N], xd[:, R + N:], dev(A), hd, Dskip=dev(Dsk), z=dev(z),
                        delta_bias=dev(bias), dt_in=xd[:, :R], dt_weight=dev(W))
    delta = x_dbl[:, :R].double() @ W.double().T
    dte = torch.nn.functional.softplus(delta + bias.double())
    a = torch.exp(dte[..., None] * A.double())
    hn = a * h.double() + (dte * xc.double())[..., None] * Bm.double()[:, None, :]
    yo = (hn * Cm.double()[:, None, :]).sum(-1) + Dsk.double() * xc.double()
    yo = yo * z.double() * torch.sigmoid(z.double())
    np.testing.assert_allclose(y.double().cpu().numpy(), yo.numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(hd.double().cpu().numpy(), hn.numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("b,D,R", [(1, 128, 8), (7, 2048, 64), (40, 512, 128)])
def test_decode_layer_step_folds_both_projections(b, D, R):
    """swx_decode_layer_step (conv + x_proj + dt_proj + state update + gate, both
    projections inside the kernels) against the block's step in float64
    (models/sift_block.py:160-175): conv window roll, xc = silu(conv + bias),
    dt | B | C = x_proj(xc), delta = softplus(dt_proj(dt) + bias), the recurrence, readout,
    D skip and gate.  Batch 40 gives the state-update CTAs more than one row each."""
    from swiftx_b200.decode import decode_layer_step
    N, K = 16, 4
    g = torch.Generator().manual_seed(43)
    r = lambda *s, sc=1.0: torch.randn(*s, generator=g) * sc  # noqa: E731
    xz = r(b, 2 * D)
    cw, cb = r(D, 1, K, sc=0.5), r(D, sc=0.1)
    Wx, Wdt = r(R + 2 * N, D, sc=D ** -0.5), r(D, R, sc=R ** -0.5)
    A_log = torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(D, 1)
    Dsk, bias = r(D), r(D, sc=0.1) - 4.0
    cs, h = r(b, D, K), r(b, D, N, sc=0.1)
    dev = lambda t: t.to(DEV)  # noqa: E731
    xzd, csd, hd = dev(xz), dev(cs), dev(h)
    y = decode_layer_step(xzd[:, :D], csd, dev(cw), dev(cb), dev(Wx), dev(Wdt), dev(A_log), hd, Dskip=dev(Dsk),
                          z=xzd[:, D:], delta_bias=dev(bias), A_is_log=True)
    assert y is not None
    d = lambda t: t.double()  # noqa: E731
    x, z = d(xz[:, :D]), d(xz[:, D:])
    win = torch.cat([d(cs)[..., 1:], x[..., None]], -1)
    xc = torch.nn.functional.silu((win * d(cw)[:, 0, :]).sum(-1) + d(cb))
    x_dbl = xc @ d(Wx).T
    dt, Bm, Cm = x_dbl[:, :R], x_dbl[:, R:R + N], x_dbl[:, R + N:]
    dte = torch.nn.functional.softplus(dt @ d(Wdt).T + d(bias))
    hn = torch.exp(dte[..., None] * -torch.exp(d(A_log))) * d(h) + (dte * xc)[..., None] * Bm[:, None, :]
    yo = ((hn * Cm[:, None, :]).sum(-1) + d(Dsk) * xc) * torch.nn.functional.silu(z)
    np.testing.assert_allclose(y.double().cpu().numpy(), yo.numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(hd.double().cpu().numpy(), hn.numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(csd.double().cpu().numpy(), win.numpy(), rtol=0, atol=0)


def test_decode_layer_step_declines_other_shapes():
    """D not a multiple of 64 (or d_state != 16): None, and the states are untouched."""
    from swiftx_b200.decode import decode_layer_step
    b, D, N, R = 3, 96, 16, 8
    xz = torch.randn(b, 2 * D, device=DEV)
    cs, h = torch.randn(b, D, 4, device=DEV), torch.randn(b, D, N, device=DEV)
    cs0, h0 = cs.clone(), h.clone()
    y = decode_layer_step(xz[:, :D], cs, torch.randn(D, 1, 4, device=DEV), None,
                          torch.randn(R + 2 * N, D, device=DEV), torch.randn(D, R, device=DEV),
                          -torch.ones(D, N, device=DEV), h, z=xz[:, D:])
    assert y is None and torch.equal(cs, cs0) and torch.equal(h, h0)


def test_conv_empty_sequence_zero_weight_grads():
    """An empty sequence: empty output, and zero weight / bias gradients (no step
    contributes), as torch's conv1d gives."""
    x = torch.randn(2, 0, 64, device=DEV, requires_grad=True)
    w = torch.randn(64, 1, 4, device=DEV, requires_grad=True)
    bias = torch.randn(64, device=DEV, requires_grad=True)
    y = causal_conv1d_fn(x, w, bias, "silu")
    assert y.shape == (2, 0, 64)
    y.sum().backward()
    assert torch.equal(w.grad, torch.zeros_like(w)) and torch.equal(bias.grad, torch.zeros_like(bias))
