"""The fused RMSNorm (swiftx_b200.norm) against the reference's expression
(models/sift_model.py:25-26), forward and backward, evaluated in float64 by torch
autograd.  Tolerances: fp32 rtol 1e-5 / atol 1e-6 (dweight, a sum over rows: atol 1e-4);
bf16 rtol 2e-2."""
import numpy as np
import pytest
import torch

from swiftx_b200.norm import rms_norm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def reference(x, w, eps=1e-5):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


@pytest.mark.parametrize("shape", [(3, 7, 256), (1000, 96), (2, 5, 1024), (9, 40), (1, 1, 32)])
def test_forward_backward_fp32(shape):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(shape, generator=g) * 3
    w = torch.randn(shape[-1], generator=g)
    dy = torch.randn(shape, generator=g)
    xd, wd = x.to(DEV).requires_grad_(), w.to(DEV).requires_grad_()
    y = rms_norm(xd, wd)
    y.backward(dy.to(DEV))
    x64, w64 = x.double().requires_grad_(), w.double().requires_grad_()
    y64 = reference(x64, w64)
    y64.backward(dy.double())
    np.testing.assert_allclose(y.detach().double().cpu().numpy(), y64.detach().numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(xd.grad.double().cpu().numpy(), x64.grad.numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(wd.grad.double().cpu().numpy(), w64.grad.numpy(), rtol=1e-5, atol=1e-4)


def test_bf16_and_determinism():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(64, 128, 256, generator=g)).to(DEV)
    w = torch.randn(256, generator=g).to(DEV)
    yb = rms_norm(x.bfloat16(), w)
    assert yb.dtype == torch.bfloat16
    np.testing.assert_allclose(yb.float().cpu().numpy(), reference(x.bfloat16().float(), w).cpu().numpy(),
                               rtol=2e-2, atol=2e-2)
    dy = torch.randn(64, 128, 256, device=DEV)
    grads = []
    for _ in range(2):
        xr, wr = x.clone().requires_grad_(), w.clone().requires_grad_()
        rms_norm(xr, wr).backward(dy)
        grads.append((xr.grad, wr.grad))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])


def test_rejects_unsupported():
    with pytest.raises(ValueError):
        rms_norm(torch.randn(2, 2048, device=DEV), torch.ones(2048, device=DEV))


def test_bf16_output_is_the_rounded_fp32_result():
    """out_dtype=bf16 gives the fp32 result rounded once, and its backward (bf16 upstream
    gradient) equals the fp32 backward fed the same gradient values."""
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(40, 256, generator=g) * 2).to(DEV)
    w = torch.randn(256, generator=g).to(DEV)
    dy = torch.randn(40, 256, generator=g).to(DEV).bfloat16()
    x1, w1 = x.clone().requires_grad_(), w.clone().requires_grad_()
    yb = rms_norm(x1, w1, out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16 and x1.grad is None
    x2, w2 = x.clone().requires_grad_(), w.clone().requires_grad_()
    yf = rms_norm(x2, w2)
    assert torch.equal(yb, yf.bfloat16())
    yb.backward(dy)
    yf.backward(dy.float())
    assert torch.equal(x1.grad, x2.grad) and torch.equal(w1.grad, w2.grad)


@pytest.mark.parametrize("res_dtype,out_dtype,with_ds", [
    (torch.bfloat16, torch.bfloat16, True),       # the LM under autocast: bf16 mixer output, bf16 norm output
    (torch.float32, None, True),
    (torch.bfloat16, None, False),                # the final norm: nothing else reads the sum
])
def test_add_rms_norm_equals_separate_add_and_norm(res_dtype, out_dtype, with_ds):
    # Residual form against the separate ops on the same kernels: x + res (torch), then
    # rms_norm; backward through autograd's add (gradient sum, cast to res's dtype).  With
    # an fp32 residual stream every value must agree bit for bit.
    from swiftx_b200.norm import add_rms_norm
    g = torch.Generator().manual_seed(11)
    shape = (4, 300, 256)
    x = (torch.randn(shape, generator=g) * 2).to(DEV)
    res = torch.randn(shape, generator=g).to(DEV).to(res_dtype)
    w = torch.randn(256, generator=g).to(DEV)
    dy = torch.randn(shape, generator=g).to(DEV).to(out_dtype or torch.float32)
    ds = torch.randn(shape, generator=g).to(DEV) if with_ds else None

    def run(fused):
        xa, ra, wa = x.clone().requires_grad_(), res.clone().requires_grad_(), w.clone().requires_grad_()
        if fused:
            s, y = add_rms_norm(xa, ra, wa, 1e-5, out_dtype)
        else:
            s = xa + ra
            y = rms_norm(s, wa, 1e-5, out_dtype)
        outs, grads = [y], [dy]
        if with_ds:
            outs.append(s)
            grads.append(ds)
        torch.autograd.backward(outs, grads)
        return s.detach(), y.detach(), xa.grad, ra.grad, wa.grad

    for a, b, name in zip(run(True), run(False), ("sum", "y", "dx", "dres", "dweight")):
        assert a.dtype == b.dtype, name
        assert torch.equal(a, b), name


def test_backbone_fused_residual_norm_matches_per_layer_form():
    # SiftBackbone folds each residual add into the next norm; the per-layer form
    # (ResidualBlock.forward) must give the same logits and gradients, bit for bit,
    # under bf16 autocast as in the LM training step.
    from swiftx_b200.sift import SiftConfig, SiftLM
    torch.manual_seed(0)
    m = SiftLM(SiftConfig(vocab_size=64, d_model=128, n_layers=3, d_state=16)).to(DEV)
    tok = torch.randint(0, 64, (2, 97), device=DEV)

    def run(fuse):
        m.backbone.fuse_residual_norm = fuse
        m.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, loss = m(tok[:, :-1], tok[:, 1:])
        loss.backward()
        return logits.detach().float(), [p.grad.clone() for p in m.parameters()]

    l1, g1 = run(True)
    l0, g0 = run(False)
    assert torch.equal(l1, l0)
    for a, b in zip(g1, g0):
        assert torch.equal(a, b)


def test_no_rows_zero_weight_grad():
    """No rows: an empty output and a zero weight gradient (no row contributes)."""
    x = torch.randn(0, 256, device="cuda", requires_grad=True)
    w = torch.randn(256, device="cuda", requires_grad=True)
    y = rms_norm(x, w)
    assert y.shape == (0, 256)
    y.sum().backward()
    assert torch.equal(w.grad, torch.zeros_like(w))
