"""Host side of the conv wrappers (swiftx_b200.conv), on CPU with the launches stubbed.

The conv kernels read x, the weight, the bias and the output gradient through bare
pointers sized by x, so the wrappers check them first.  Without a GPU this tests that
well-formed forward and backward calls (including the strided x half of a (b, L, 2D)
tensor, as the Sift block passes it) reach the library, and that a bias, weight or
output gradient of the wrong size raises before any launch.  The launch entry points
are a stub that records them; size queries go to the real library; the CUDA-device
check is lifted so CPU tensors stand in for device ones.
"""
import pytest
import torch

from swiftx_b200 import _lib, conv


class _LaunchStub:
    def __init__(self, real):
        self.real, self.calls = real, []

    def __getattr__(self, name):
        if name in ("swx_conv1d_fwd", "swx_conv1d_bwd"):
            return lambda a, stream: self.calls.append((name, a.batch, a.seqlen, a.dim, a.width)) or 0
        return getattr(self.real, name)


@pytest.fixture
def stub(monkeypatch):
    lib = _LaunchStub(_lib.load())
    monkeypatch.setattr(_lib, "load", lambda: lib)
    monkeypatch.setattr(_lib, "stream_ptr", lambda dev: None)
    monkeypatch.setattr(conv, "_require_cuda", lambda *ts: None)
    return lib


def test_block_shaped_calls_reach_the_library(stub):
    b, L, D, K = 2, 19, 6, 4
    xz = torch.randn(b, L, 2 * D)
    w, cb = torch.randn(D, 1, K), torch.randn(D)
    x = xz[..., :D]                                        # the strided x half, row stride 2D
    y = conv.causal_conv1d_fn(x, w, cb)
    assert y.shape == (b, L, D)
    dxz = torch.empty_like(xz)
    conv.conv1d_backward(x, w, cb, torch.randn(b, L, D), True, dx_out=dxz[..., :D])
    conv.conv1d_backward(x, w.view(D, K), None, torch.randn(b, L, D), True)
    assert [c[0] for c in stub.calls] == ["swx_conv1d_fwd", "swx_conv1d_bwd", "swx_conv1d_bwd"]
    assert all(c[1:] == (b, L, D, K) for c in stub.calls)


@pytest.mark.parametrize("what", ["bias", "weight", "dout"])
def test_wrong_sizes_are_refused(stub, what):
    b, L, D, K = 2, 19, 6, 4
    x, w, cb, dout = torch.randn(b, L, D), torch.randn(D, 1, K), torch.randn(D), torch.randn(b, L, D)
    if what == "bias":
        cb = torch.randn(D - 1)
    elif what == "weight":
        w = torch.randn(D + 1, 1, K)
    else:
        dout = torch.randn(b, L + 1, D)
    with pytest.raises(ValueError, match=what):
        if what == "dout":
            conv.conv1d_backward(x, w, cb, dout, True)
        else:
            conv.conv1d_forward(x, w, cb)
    assert stub.calls == []
