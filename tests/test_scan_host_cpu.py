"""Host side of the scan wrappers (swiftx_b200.selective_scan), on CPU with the launches stubbed.

The kernels read every operand through a bare pointer, so the wrappers check shapes,
dtypes and layouts first.  Without a GPU this tests that the calls the autograd Function
makes (forward with checkpoints and the pre-gate output, backward reading them) pass
those checks and reach the library, and that mis-shaped operands raise before any
launch.  The launch entry points are replaced by a stub that records them; the size
queries (host arithmetic only) go to the real library; the CUDA-device check is lifted
so CPU tensors stand in for device ones.
"""
import pytest
import torch

from swiftx_b200 import _lib, selective_scan


class _LaunchStub:
    def __init__(self, real):
        self.real, self.calls = real, []

    def __getattr__(self, name):
        if name in ("swx_scan_fwd", "swx_scan_bwd"):
            return lambda a, stream: self.calls.append((name, a.batch, a.seqlen, a.dim, a.dstate)) or 0
        if name == "swx_scan_fwd_workspace_bytes":
            return lambda a: 0
        return getattr(self.real, name)


@pytest.fixture
def stub(monkeypatch):
    lib = _LaunchStub(_lib.load())
    monkeypatch.setattr(_lib, "load", lambda: lib)
    monkeypatch.setattr(_lib, "stream_ptr", lambda dev: None)
    monkeypatch.setattr(selective_scan, "_require_cuda", lambda *ts: None)
    return lib


def _problem(b=2, L=37, D=12, N=5, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    return dict(u=r(b, L, D), delta=r(b, L, D), A=-torch.rand(D, N, generator=g) - 0.1, B=r(b, L, N), C=r(b, L, N),
                D=r(D), z=r(b, L, D), delta_bias=r(D), h0=r(b, D, N))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
def test_autograd_calls_pass_the_checks(stub, dtype):
    p = {k: v.to(dtype if k in ("u", "delta", "B", "C", "z") else v.dtype).requires_grad_() for k, v in _problem().items()}
    out = selective_scan.selective_scan_fn(p["u"], p["delta"], p["A"], p["B"], p["C"], p["D"], z=p["z"],
                                           delta_bias=p["delta_bias"], delta_softplus=True, h0=p["h0"])
    out.float().sum().backward()
    assert [c[0] for c in stub.calls] == ["swx_scan_fwd", "swx_scan_bwd"]
    assert stub.calls[1][1:] == (2, 37, 12, 5)


@pytest.mark.parametrize("name,shape", [("D", (11,)), ("delta_bias", (13,)), ("h0", (2, 12, 6)),
                                        ("h0", (1, 12, 5))])
def test_mis_shaped_parameters_are_refused(stub, name, shape):
    p = _problem()
    p[name] = torch.randn(*shape)
    with pytest.raises(ValueError, match=name):
        selective_scan.scan_forward(p["u"], p["delta"], p["A"], p["B"], p["C"], p["D"], p["z"], p["delta_bias"],
                                    True, h0=p["h0"], checkpoints=True)
    assert stub.calls == []


def test_backward_refuses_a_mis_shaped_output_gradient(stub):
    p = _problem()
    args = (p["u"], p["delta"], p["A"], p["B"], p["C"], p["D"], p["z"], p["delta_bias"], True)
    _, ck, _ = selective_scan.scan_forward(*args, checkpoints=True)
    assert len(stub.calls) == 1
    with pytest.raises(ValueError, match="dout"):
        selective_scan.scan_backward(*args, None, ck, torch.randn(2, 37, 13))
    assert len(stub.calls) == 1
    selective_scan.scan_backward(*args, None, ck, torch.randn(2, 37, 12))
    assert [c[0] for c in stub.calls] == ["swx_scan_fwd", "swx_scan_bwd"]


def test_backward_refuses_checkpoints_and_pre_output_it_cannot_index(stub):
    """The backward kernels read the forward's checkpoints and pre-gate output through bare
    pointers, so scan_backward checks them first: a missing, short, mistyped or strided
    buffer raises before any kernel is launched (as does a mis-shaped pre_out given to
    the forward)."""
    g = torch.Generator().manual_seed(0)
    b, L, D, N = 2, 40, 8, 4
    u, dl, z, dout = (torch.randn(b, L, D, generator=g) for _ in range(4))
    A, Bm, Cm = -torch.rand(D, N, generator=g) - 0.1, torch.randn(b, L, N, generator=g), torch.randn(b, L, N, generator=g)
    args = (u, dl.abs(), A, Bm, Cm, torch.randn(D, generator=g), z, None, False)
    need = stub.swx_scan_checkpoint_floats(b, L, D)
    assert need > 0
    ck = torch.empty(need)
    for bad_ck in (None, torch.empty(need - 1), torch.empty(need, dtype=torch.float64),
                   torch.empty(2 * need)[::2]):
        with pytest.raises(ValueError, match="ck must be"):
            selective_scan.scan_backward(*args, None, bad_ck, dout)
    for bad_pre in (torch.empty(b, L, D - 1), torch.empty(b, L, D, dtype=torch.bfloat16),
                    torch.empty(b, D, L).transpose(1, 2)):
        with pytest.raises(ValueError, match="y_pre must be"):
            selective_scan.scan_backward(*args, None, ck, dout, y_pre=bad_pre)
        with pytest.raises(ValueError, match="pre_out must be"):
            selective_scan.scan_forward(*args, checkpoints=True, pre_out=bad_pre)
    assert stub.calls == []
