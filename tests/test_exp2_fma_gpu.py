"""The FMA-pipe 2^x used for part of the backward's decays, against a float64 reference:
over the decay range [-125, 0] (and a little above 0) its relative error stays within
4 units in the last place of fp32 (2^-22; the polynomial itself is a 7.5e-8 minimax fit),
the order of CUDA's exp2f / ex2.approx error bounds; below -125 it is 0, as
ex2.approx.ftz flushes results under 2^-126."""
import numpy as np
import pytest
import torch

from swiftx_b200 import _lib

pytestmark = pytest.mark.gpu


def _eval(x):
    y = torch.empty_like(x)
    assert _lib.load().swx_exp2_fma_eval(x.data_ptr(), y.data_ptr(), x.numel(),
                                         _lib.stream_ptr(x.device)) == _lib.SWX_OK
    torch.cuda.synchronize()
    return y


def test_exp2_fma_relative_error():
    x = torch.linspace(-124.99, 4.0, 2_000_001, device="cuda", dtype=torch.float32)
    x = torch.cat([x, torch.rand(1_000_000, device="cuda") * -20.0])
    y = _eval(x).double().cpu().numpy()
    ref = np.exp2(x.double().cpu().numpy())
    rel = np.abs(y - ref) / ref
    assert rel.max() < 2.0 ** -22, rel.max()
    # CUDA's own fp32 exp2 for context: the same order of error
    rel_cuda = np.abs(torch.exp2(x).double().cpu().numpy() - ref) / ref
    assert rel.max() < 8 * max(rel_cuda.max(), 2.0 ** -24)


def test_exp2_fma_special_points():
    x = torch.tensor([0.0, -1.0, -0.5, 0.5, -125.0, -200.0, 1.0, 126.5], device="cuda")
    y = _eval(x).double().cpu().numpy()
    assert y[5] == 0.0                        # flushed like ex2.approx.ftz
    keep = [0, 1, 2, 3, 4, 6, 7]
    np.testing.assert_allclose(y[keep], np.exp2(x.cpu().double().numpy()[keep]), rtol=2.0 ** -22)
