"""The status path of the bounded device-side waits.

The time-segmented backward waits for its TMA tiles with an iteration limit; when a
wait runs out it records SWX_ERR_TIMEOUT in the library's status word and returns.  No
real failure is provoked here: swx_diag_wait_timeout runs one thread that waits a few
hundred tries for an mbarrier phase nothing completes and records the timeout the same
way.  The status must read back once, clear, and leave the context usable (a backward
afterwards runs on the TMA path and matches the one before)."""
import pytest
import torch

from swiftx_b200 import _lib
from swiftx_b200.selective_scan import scan_backward, scan_forward
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu


def _backward(inp):
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    _, ck, _ = scan_forward(*args, checkpoints=True)
    return scan_backward(*args, None, ck, inp["dout"])


def test_status_ok_after_backward_and_timeout_reported():
    lib = _lib.load()
    inp = config_inputs(2, 640, 128, 16, seed=5, device="cuda")       # fp32: segmented, TMA staging
    before = _backward(inp)
    assert lib.swx_device_wait_status() == _lib.SWX_OK
    assert lib.swx_diag_wait_timeout(256, _lib.stream_ptr(torch.device("cuda"))) == _lib.SWX_OK
    assert lib.swx_device_wait_status() == _lib.SWX_ERR_TIMEOUT
    assert lib.swx_device_wait_status() == _lib.SWX_OK                  # read once, then cleared
    after = _backward(inp)
    assert lib.swx_device_wait_status() == _lib.SWX_OK
    for k, v in before.items():
        if v is not None:
            assert torch.equal(after[k], v), k
