"""parallel_scan / sequential_scan (h_t = a_t * h_{t-1} + x_t along dim 1) on the sm_100a
linear-scan kernel, against the reference's own outputs (linscan.npz, made by importing
models/selective_scan.py) and the float64 oracle.

Tolerances: fp32 atol 1e-5 against the reference (its own parallel-vs-loop pin,
tests/test_selective_scan.py:64); fp32 rtol 1e-5 / atol 1e-6 against the oracle; fp64
rtol 1e-10.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200 import parallel_scan, sequential_scan

pytestmark = pytest.mark.gpu
DEV = "cuda"


def n64(t):
    return t.detach().double().cpu().numpy()


@pytest.mark.parametrize("L", [1, 2, 5, 8, 33, 128])
def test_matches_reference_outputs(golden, L):
    g = golden("linscan")
    a, x = torch.from_numpy(g[f"a_{L}"]).to(DEV), torch.from_numpy(g[f"x_{L}"]).to(DEV)
    for fn in (parallel_scan, sequential_scan):
        h = fn(a, x)
        assert h.shape == a.shape and h.dtype == torch.float32
        np.testing.assert_allclose(n64(h), g[f"hp_{L}"], atol=1e-5, rtol=0)
        np.testing.assert_allclose(n64(h), g[f"hs_{L}"], atol=1e-5, rtol=0)


def test_fp64_gradients_match_reference_autograd(golden):
    g = golden("linscan")
    a = torch.from_numpy(g["ga"]).to(DEV).requires_grad_()
    x = torch.from_numpy(g["gx"]).to(DEV).requires_grad_()
    h = parallel_scan(a, x)
    assert h.dtype == torch.float64
    (h * torch.from_numpy(g["gw"]).to(DEV)).sum().backward()
    np.testing.assert_allclose(n64(h), g["gh"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(n64(a.grad), g["gda"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(n64(x.grad), g["gdx"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("shape", [(1, 1, 1), (2, 7, 3), (3, 8, 130), (2, 9, 4, 5), (4, 100, 64, 16),
                                   (1, 1000, 33)])
def test_vs_oracle_fp32_with_grads(shape):
    gen = torch.Generator().manual_seed(sum(shape))
    a = torch.rand(shape, generator=gen)
    x = torch.randn(shape, generator=gen)
    w = torch.randn(shape, generator=gen)
    ad, xd = a.to(DEV).requires_grad_(), x.to(DEV).requires_grad_()
    h = sequential_scan(ad, xd)
    (h * w.to(DEV)).sum().backward()
    ho = oracle.linear_scan(a, x)
    np.testing.assert_allclose(n64(h), ho, rtol=1e-5, atol=1e-6)
    da, dx = oracle.linear_scan_bwd(a, ho, w)
    np.testing.assert_allclose(n64(ad.grad), da, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n64(xd.grad), dx, rtol=1e-5, atol=1e-6)


def test_strided_inputs_and_other_dtypes():
    gen = torch.Generator().manual_seed(5)
    base_a = torch.rand(3, 40, 2, 6, generator=gen)
    base_x = torch.randn(3, 40, 2, 6, generator=gen)
    a, x = base_a.to(DEV)[:, ::2], base_x.to(DEV)[:, ::2]          # every other step: strided
    want = oracle.linear_scan(base_a[:, ::2], base_x[:, ::2])
    np.testing.assert_allclose(n64(parallel_scan(a, x)), want, rtol=1e-5, atol=1e-6)
    hb = parallel_scan(a.bfloat16(), x.bfloat16())                   # computed in fp32
    assert hb.dtype == torch.bfloat16
    np.testing.assert_allclose(n64(hb), oracle.linear_scan(a.bfloat16(), x.bfloat16()), rtol=2e-2, atol=2e-2)
    with pytest.raises(ValueError):
        parallel_scan(a, x[:, :3])


def test_large_recurrence():
    """(b, L, D, N) = (2, 2048, 512, 16): the layout the reference feeds its _scan."""
    gen = torch.Generator(device=DEV).manual_seed(7)
    a = torch.rand(2, 2048, 512, 16, device=DEV, generator=gen) * 0.2 + 0.8
    x = torch.randn(2, 2048, 512, 16, device=DEV, generator=gen)
    h = parallel_scan(a, x)
    want = oracle.linear_scan(a[:, :, :64], x[:, :, :64])             # a slice of the channels
    np.testing.assert_allclose(n64(h[:, :, :64]), want, rtol=1e-4, atol=1e-4)
