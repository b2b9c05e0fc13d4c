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
