"""The two staging paths of the scan kernels give the same bits.

Tiles reach shared memory by TMA (one thread, bulk tensor copies, mbarrier completion)
when every input's base and strides are 16-byte aligned, and by per-thread loads
otherwise.  The arithmetic after staging is the same, so a problem run once on aligned
tensors and once on copies offset by one element (never 16-byte aligned) must give
identical outputs, checkpoints, final states and gradients: the forward, the
time-segmented backward (fp32) and the whole-row backward (a bf16 grid that fills the
GPU), each with partial tiles at the sequence end and a partial channel block.
"""
import pytest
import torch

from swiftx_b200.selective_scan import scan_backward, scan_forward
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
KEYS = ("u", "delta", "B", "C", "z", "dout")


def _offset_copy(t):
    """A copy of t whose storage starts one element past a fresh allocation."""
    buf = torch.empty(t.numel() + 8, dtype=t.dtype, device=t.device)
    v = buf[1:1 + t.numel()].view(t.shape)
    v.copy_(t)
    assert v.data_ptr() % 16 != 0
    return v


def _run(inp, h0):
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32)
    out, ck, hl = scan_forward(*args, h0=h0, out_dtype=torch.float32, checkpoints=True, return_last_state=True,
                               pre_out=pre)
    g = scan_backward(*args, h0, ck, inp["dout"], y_pre=pre)
    return {"out": out, "ck": ck, "h_last": hl, "pre": pre, **{k: v for k, v in g.items() if v is not None}}


@pytest.mark.parametrize("shape,dtype", [((2, 301, 96, 16), torch.float32),      # segmented backward
                                         ((1, 2000, 200, 16), torch.float32),    # several segments
                                         ((16, 77, 520, 16), torch.bfloat16)],   # whole-row backward
                         ids=["fp32-short", "fp32-long", "bf16-rows"])
def test_tma_and_per_thread_staging_agree(shape, dtype):
    b, L, D, N = shape
    inp = config_inputs(b, L, D, N, seed=61, device=DEV, dtype=dtype)
    h0 = (torch.randn(b, D, N, generator=torch.Generator().manual_seed(6)) * 0.2).to(DEV)
    aligned = _run(inp, h0)
    shifted = dict(inp)
    for k in KEYS:
        shifted[k] = _offset_copy(inp[k])
    unaligned = _run(shifted, h0)
    assert set(aligned) == set(unaligned)
    for k in aligned:
        assert torch.equal(aligned[k], unaligned[k]), k


def _segments(inp):
    """swx_scan_bwd_segments for these inputs: 0 = the whole-row kernel, else the segment count."""
    from swiftx_b200 import _lib
    from swiftx_b200.selective_scan import _fill_inputs, _prep
    a = _lib.ScanArgs()
    u, dl, A, Bm, Cm, Dv, z, bias, h0, in_dt = _prep(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"],
                                                     inp["D"], inp["z"], inp["delta_bias"], None)
    _fill_inputs(a, u, dl, A, Bm, Cm, Dv, z, bias, h0, True, in_dt)
    a.out_pre = 16                                    # only its presence matters here
    return _lib.load().swx_scan_bwd_segments(a)


@pytest.mark.parametrize("shape,dtype,rows", [((2, 301, 96, 16), torch.float32, False),
                                              ((3, 67, 37, 16), torch.float32, False),
                                              ((16, 77, 520, 16), torch.bfloat16, True),
                                              ((16, 77, 519, 16), torch.bfloat16, True)],
                         ids=["fp32-segmented", "fp32-segmented-odd", "bf16-rows", "bf16-rows-odd"])
def test_strided_gradient_outputs_equal_dense(shape, dtype, rows):
    """dz written into the z half and the conv's dx into the x half of one (b, L, 2D)
    buffer (row stride 2D, as the in_proj output's gradient) equal the dense outputs bit
    for bit: the segmented and the whole-row backward, and the conv backward.  With an odd
    D the z half starts 4 (fp32) or 2 (bf16) bytes past an aligned address and every other
    row is misaligned, so the segmented kernel's paired dz stores give way to single ones."""
    from swiftx_b200.conv import conv1d_backward
    b, L, D, N = shape
    inp = config_inputs(b, L, D, N, seed=62, device=DEV, dtype=dtype)
    assert (_segments(inp) == 0) == rows
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32)
    _, ck, _ = scan_forward(*args, checkpoints=True, pre_out=pre)
    dense = scan_backward(*args, None, ck, inp["dout"], y_pre=pre)
    dxz = torch.full((b, L, 2 * D), float("nan"), device=DEV, dtype=dtype)
    strided = scan_backward(*args, None, ck, inp["dout"], y_pre=pre, dz_out=dxz[..., D:])
    assert strided["dz"].data_ptr() == dxz[..., D:].data_ptr()
    for k in dense:
        if dense[k] is not None:
            assert torch.equal(dense[k], strided[k]), k
    w = (torch.randn(D, 4, generator=torch.Generator().manual_seed(7)) * 0.3).to(DEV)
    bias = torch.zeros(D, device=DEV)
    dx0, dw0, db0 = conv1d_backward(inp["u"], w, bias, inp["dout"], True)
    dx1, dw1, db1 = conv1d_backward(inp["u"], w, bias, inp["dout"], True, dx_out=dxz[..., :D])
    assert dx1.data_ptr() == dxz.data_ptr()
    assert torch.equal(dx0, dx1) and torch.equal(dw0, dw1) and torch.equal(db0, db1)
    assert torch.equal(dxz[..., D:], dense["dz"])
