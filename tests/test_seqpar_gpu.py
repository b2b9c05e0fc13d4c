"""Sequence-parallel scan on one GPU: chunks scanned as separate 'ranks' (pass 1 without
output -> boundary values -> prefix combine -> pass 2 from the true initial state) must
reproduce the one-pass scan of the whole sequence and the oracle."""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.selective_scan import scan_forward
from swiftx_b200.seqpar import combine_prefix
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def chunked_scan(inp, bounds, out_dtype=torch.float32):
    keys = ("u", "delta", "z", "B", "C")
    ends, sums = [], []
    for s, e in zip(bounds[:-1], bounds[1:]):
        ch = {k: inp[k][:, s:e] for k in keys}
        out, _, h_end, dsum = scan_forward(ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], inp["D"], ch["z"],
                                           inp["delta_bias"], True, return_last_state=True,
                                           return_delta_sum=True, write_out=False)
        assert out is None
        ends.append(h_end)
        sums.append(dsum)
    outs = []
    for g, (s, e) in enumerate(zip(bounds[:-1], bounds[1:])):
        ch = {k: inp[k][:, s:e] for k in keys}
        h0 = combine_prefix(ends, sums, inp["A"].float(), g) if g > 0 else None
        out, _, _ = scan_forward(ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], inp["D"], ch["z"],
                                 inp["delta_bias"], True, h0=h0, out_dtype=out_dtype)
        outs.append(out)
    return torch.cat(outs, 1)


def test_delta_sum_output():
    inp = config_inputs(2, 77, 40, 16, seed=1, device=DEV)
    _, _, _, ds = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                               inp["delta_bias"], True, return_delta_sum=True, write_out=False)
    want = torch.nn.functional.softplus(inp["delta"].double() + inp["delta_bias"].double()).sum(1)
    np.testing.assert_allclose(ds.double().cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("bounds", [[0, 130, 300], [0, 64, 100, 229, 300], [0, 1, 2, 300]])
def test_chunked_equals_whole(bounds):
    inp = config_inputs(2, 300, 96, 16, seed=2, device=DEV)
    whole, _, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                               inp["delta_bias"], True)
    got = chunked_scan(inp, bounds)
    want = oracle.scan_fwd(*(inp[k].double().cpu().numpy() for k in ("u", "delta", "A", "B", "C")),
                           D=inp["D"].double().cpu().numpy(), z=inp["z"].double().cpu().numpy(),
                           delta_bias=inp["delta_bias"].double().cpu().numpy(), delta_softplus=True)
    np.testing.assert_allclose(got.double().cpu().numpy(), want, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(got.cpu().numpy(), whole.cpu().numpy(), rtol=1e-4, atol=1e-5)


def test_long_sequence_bf16_eight_chunks():
    """The long-sequence configuration's layout (bf16 u/delta/B/C/z, fp32 state and
    output) at reduced size, split like 8 ranks, against the oracle run on the same
    bf16-rounded values (rtol 2e-2, bf16 inputs with fp32 state)."""
    b, L, D = 2, 8 * 512, 256
    inp = config_inputs(b, L, D, 16, seed=4, device=DEV, dtype=torch.bfloat16)
    got = chunked_scan(inp, list(range(0, L + 1, 512)))
    n = lambda t: t.double().cpu().numpy()  # noqa: E731
    want = oracle.scan_fwd(*(n(inp[k]) for k in ("u", "delta", "A", "B", "C")), D=n(inp["D"]), z=n(inp["z"]),
                           delta_bias=n(inp["delta_bias"]), delta_softplus=True)
    np.testing.assert_allclose(n(got), want, rtol=2e-2, atol=1e-3 * np.abs(want).max())
