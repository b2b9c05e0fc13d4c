"""HostScanPipeline: forward + backward of pinned host batches streamed through the GPU
in row chunks over several streams.

Rows of the scan are independent, so every per-row result (out, du, ddelta, dz, dB, dC)
must equal, bit for bit, the whole-batch kernel call on device tensors (the sequences
here are short enough that every chunk gets the whole batch's backward segment plan).  dA, dD and
d(delta_bias) are sums over the batch that the pipeline adds per chunk and then across
chunks; they match the whole-batch sums to fp32 re-association (rtol 1e-5, atol 1e-6 of
the largest entry).  One case is also checked against the float64 oracle.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.host_pipeline import HostScanPipeline
from swiftx_b200.selective_scan import scan_backward, scan_forward
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROW_KEYS = ("out", "du", "ddelta", "dz", "dB", "dC")
SUM_KEYS = ("dA", "dD", "ddelta_bias")


def _device_reference(inp, has_z, has_D, has_bias):
    z = inp["z"] if has_z else None
    D = inp["D"] if has_D else None
    bias = inp["delta_bias"] if has_bias else None
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32) if has_z else None
    out, ck, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], D, z, bias, True,
                              checkpoints=True, pre_out=pre)
    g = scan_backward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], D, z, bias, True, None, ck,
                      inp["dout"], y_pre=pre)
    g["out"] = out
    return {k: v for k, v in g.items() if v is not None}


def _run_pipeline(inp, dtype, rows, nbuf, n_compute, has_z=True, has_D=True, has_bias=True, reps=1):
    b, L, Dm = inp["u"].shape
    N = inp["A"].shape[1]
    pipe = HostScanPipeline(b, L, Dm, N, dtype=dtype, has_z=has_z, has_D=has_D, has_bias=has_bias,
                            rows_per_chunk=rows, nbuf=nbuf, n_compute=n_compute)
    host = {k: v.cpu().pin_memory() for k, v in inp.items()}
    res = pipe.allocate_host_outputs()
    for _ in range(reps):
        for t in res.values():
            t.fill_(float("nan"))
        pipe.forward_backward(host["u"], host["delta"], host["A"], host["B"], host["C"], host["dout"],
                              D=host["D"] if has_D else None, z=host["z"] if has_z else None,
                              delta_bias=host["delta_bias"] if has_bias else None, out=res)
        torch.cuda.synchronize()
    return res


def _compare(res, ref):
    assert set(res) == set(ref)
    for k in ROW_KEYS:
        if k in ref:
            assert torch.equal(res[k], ref[k].cpu()), k
    for k in SUM_KEYS:
        if k in ref:
            want = ref[k].double().cpu().numpy()
            np.testing.assert_allclose(res[k].double().numpy(), want, rtol=1e-5,
                                       atol=1e-6 * np.abs(want).max(), err_msg=k)


@pytest.mark.parametrize("b,rows,nbuf,n_compute", [(8, 2, 3, 2), (5, 2, 2, 1), (3, 1, 3, 3), (4, 4, 3, 2)])
def test_pipeline_matches_whole_batch_call(b, rows, nbuf, n_compute):
    inp = config_inputs(b, 300, 96, 16, seed=31, device=DEV)
    _compare(_run_pipeline(inp, torch.float32, rows, nbuf, n_compute), _device_reference(inp, True, True, True))


def test_pipeline_bf16():
    inp = config_inputs(4, 200, 64, 16, seed=32, device=DEV)
    inp = {k: (v.bfloat16() if k in ("u", "delta", "z", "B", "C", "dout") else v) for k, v in inp.items()}
    _compare(_run_pipeline(inp, torch.bfloat16, 1, 3, 2), _device_reference(inp, True, True, True))


def test_pipeline_without_optional_operands():
    inp = config_inputs(4, 130, 64, 8, seed=33, device=DEV)
    res = _run_pipeline(inp, torch.float32, 2, 3, 2, has_z=False, has_D=False, has_bias=False)
    _compare(res, _device_reference(inp, False, False, False))
    assert "dz" not in res and "dD" not in res and "ddelta_bias" not in res


def test_pipeline_rerun_reuses_buffers():
    inp = config_inputs(6, 160, 64, 16, seed=34, device=DEV)
    _compare(_run_pipeline(inp, torch.float32, 1, 2, 2, reps=3), _device_reference(inp, True, True, True))


def test_pipeline_matches_oracle():
    inp = config_inputs(3, 70, 32, 16, seed=35, device=DEV)
    res = _run_pipeline(inp, torch.float32, 1, 3, 2)
    a = {k: v.double().cpu().numpy() for k, v in inp.items()}
    y = oracle.scan_fwd(a["u"], a["delta"], a["A"], a["B"], a["C"], D=a["D"], z=a["z"],
                        delta_bias=a["delta_bias"], delta_softplus=True)
    g = oracle.scan_bwd(a["u"], a["delta"], a["A"], a["B"], a["C"], a["dout"], D=a["D"], z=a["z"],
                        delta_bias=a["delta_bias"], delta_softplus=True)
    np.testing.assert_allclose(res["out"].double().numpy(), y, rtol=1e-4, atol=1e-5)
    for k in ("du", "ddelta", "dz"):
        np.testing.assert_allclose(res[k].double().numpy(), g[k], rtol=1e-4, atol=1e-5, err_msg=k)
    for k in ("dB", "dC", "dA", "dD", "ddelta_bias"):
        want = g[k]
        np.testing.assert_allclose(res[k].double().numpy(), want, rtol=1e-4,
                                   atol=1e-4 * max(1.0, np.abs(want).max()), err_msg=k)


def test_pipeline_rejects_bad_arguments():
    inp = config_inputs(2, 40, 32, 16, seed=36, device=DEV)
    pipe = HostScanPipeline(2, 40, 32, 16, rows_per_chunk=1)
    host = {k: v.cpu() for k, v in inp.items()}
    args = [host[k] for k in ("u", "delta", "A", "B", "C", "dout")]
    kw = {"D": host["D"], "z": host["z"], "delta_bias": host["delta_bias"]}
    with pytest.raises(ValueError, match="host tensor"):
        pipe.forward_backward(inp["u"], *args[1:], **kw)
    with pytest.raises(ValueError, match="expected contiguous"):
        pipe.forward_backward(host["u"][:, :20], *args[1:], **kw)
    with pytest.raises(ValueError, match="required"):
        pipe.forward_backward(*args, D=host["D"], z=None, delta_bias=host["delta_bias"])


@pytest.mark.parametrize("rows,nbuf,n_compute", [(1, 3, 2), (2, 2, 2), (1, 4, 3)])
def test_chained_calls_overlap_without_mixing_batches(rows, nbuf, n_compute):
    # Four calls queued back to back (no host sync) on two different problems -- other
    # inputs, other A / D / delta_bias -- so that the next call's copies in run while the
    # previous call's kernels and copies out finish; each result set must be its own
    # problem's whole-batch result.
    b, L, Dm, N = 5, 150, 64, 16
    inps = [config_inputs(b, L, Dm, N, seed=41 + i, device=DEV) for i in range(2)]
    refs = [_device_reference(x, True, True, True) for x in inps]
    hosts = [{k: v.cpu().pin_memory() for k, v in x.items()} for x in inps]
    pipe = HostScanPipeline(b, L, Dm, N, rows_per_chunk=rows, nbuf=nbuf, n_compute=n_compute, chain_calls=True)
    results = []
    for i in range(4):
        h = hosts[i % 2]
        res = pipe.allocate_host_outputs()
        for t in res.values():
            t.fill_(float("nan"))
        pipe.forward_backward(h["u"], h["delta"], h["A"], h["B"], h["C"], h["dout"], D=h["D"], z=h["z"],
                              delta_bias=h["delta_bias"], out=res)
        results.append(res)
    torch.cuda.synchronize()
    for i, res in enumerate(results):
        _compare(res, refs[i % 2])
