"""Parity at the full sizes of the long-sequence and decode workloads, against the oracle.

* Long-sequence scan: b=4, L=65536, D=2048, N=16, bf16 u/delta/B/C/z, fp32 state and
  fp32 output, gated, softplus(delta + bias).  The kernel runs on all 2048 channels;
  channels are independent, so a slice of them is compared with the float64 oracle run
  on the same bf16-rounded values of that slice alone (exact, no sampling of steps).
  The same slice is checked for the sequence-parallel form (eight chunks: each chunk's
  forward from a zero state, prefix combine of the boundary values, initial-state
  correction).
  Tolerance: rtol 2e-2 for bf16 inputs with fp32 state, with atol 1e-3 * max|y|.
* Decode: batch 256, D=2048, N=16, d_conv=4, state h ~ N(0, 0.1), one layer stepped
  several tokens on the persistent streaming kernel, against oracle.decode_step
  (models/sift_block.py:153-175); fp32, rtol 1e-4 / atol 1e-5.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.decode import decode_step
from swiftx_b200.selective_scan import scan_correct, scan_forward
from swiftx_b200.seqpar import combine_prefix

pytestmark = pytest.mark.gpu
DEV = "cuda"
SLICE = slice(0, 64)          # channels compared with the oracle (all 4 rows, all 65536 steps)


def n64(t):
    return t.detach().float().cpu().double().numpy()


def _long_inputs():
    """Long-sequence workload inputs, drawn like the benchmark (seeded)."""
    b, L, D, N = 4, 65536, 2048, 16
    g = torch.Generator(device=DEV).manual_seed(1000)
    bf = torch.bfloat16
    u = torch.randn(b, L, D, generator=g, device=DEV).to(bf)
    dr = (torch.randn(b, L, D, generator=g, device=DEV) * 0.5).to(bf)
    z = torch.randn(b, L, D, generator=g, device=DEV).to(bf)
    Bm = torch.randn(b, L, N, generator=g, device=DEV).to(bf)
    Cm = torch.randn(b, L, N, generator=g, device=DEV).to(bf)
    gc = torch.Generator().manual_seed(0)
    dt = torch.exp(torch.rand(D, generator=gc) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    bias = (dt + torch.log(-torch.expm1(-dt))).to(DEV)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).to(DEV)
    Dsk = torch.ones(D, device=DEV)
    return dict(u=u, delta=dr, z=z, B=Bm, C=Cm, delta_bias=bias, A=A, D=Dsk)


@pytest.fixture(scope="module")
def long_case():
    inp = _long_inputs()
    s = SLICE
    want = oracle.scan_fwd(n64(inp["u"][:, :, s]), n64(inp["delta"][:, :, s]), n64(inp["A"][s]),
                           n64(inp["B"]), n64(inp["C"]), D=n64(inp["D"][s]), z=n64(inp["z"][:, :, s]),
                           delta_bias=n64(inp["delta_bias"][s]), delta_softplus=True)
    return inp, want


def _check_slice(got, want):
    """got: the kernel's output restricted to the compared channels; want: the oracle's."""
    got = n64(got)
    tol = 2e-2 * np.abs(want) + 1e-3 * np.abs(want).max()
    bad = np.abs(got - want) > tol
    assert not bad.any(), (f"{bad.sum()} of {bad.size} outside rtol 2e-2; max abs err "
                           f"{np.abs(got - want).max():.3g} (max |y| {np.abs(want).max():.3g})")


def test_long_sequence_full_size_vs_oracle(long_case):
    inp, want = long_case
    out, _, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                             inp["delta_bias"], True, out_dtype=torch.float32)
    assert out.dtype == torch.float32 and out.shape == (4, 65536, 2048)
    _check_slice(out[:, :, SLICE], want)
    assert torch.isfinite(out).all()


def test_long_sequence_eight_chunks_vs_oracle(long_case):
    """The sequence-parallel decomposition at eight chunks, each chunk the calls one rank
    makes: its forward from a zero state (output, final state, sum of delta), the prefix
    combine of the earlier chunks' boundary values, then the initial-state correction."""
    inp, want = long_case
    L = inp["u"].shape[1]
    bounds = list(range(0, L + 1, L // 8))
    keys = ("u", "delta", "z", "B", "C")
    ends, sums, outs = [], [], []
    for s, e in zip(bounds[:-1], bounds[1:]):
        ch = {k: inp[k][:, s:e] for k in keys}
        out, _, h_end, dsum = scan_forward(ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], inp["D"], ch["z"],
                                           inp["delta_bias"], True, out_dtype=torch.float32,
                                           return_last_state=True, return_delta_sum=True)
        if s > 0:
            h_in = combine_prefix(ends, sums, inp["A"], len(ends))
            scan_correct(out, h_in, ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], z=ch["z"],
                         delta_bias=inp["delta_bias"], delta_softplus=True)
        ends.append(h_end)
        sums.append(dsum)
        outs.append(out[:, :, SLICE].clone())
        del out
    _check_slice(torch.cat(outs, 1), want)


def test_decode_batch256_d2048_vs_oracle():
    """One decode layer at the decode workload's size (batch 256, D=2048, N=16, K=4), four
    tokens on the persistent streaming kernel, state and output against the oracle."""
    b, D, N, K = 256, 2048, 16, 4
    g = torch.Generator().manual_seed(77)
    dt = torch.exp(torch.rand(D, generator=g) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    p = {"cw": torch.randn(D, K, generator=g) * 0.5, "cb": torch.randn(D, generator=g),
         "A": -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1), "Dskip": torch.ones(D),
         "dbias": dt + torch.log(-torch.expm1(-dt))}
    cs = torch.randn(b, D, K, generator=g)
    ss = torch.randn(b, D, N, generator=g) * 0.1
    dv = {k: v.to(DEV) for k, v in p.items()}
    cs_d, ss_d = cs.to(DEV), ss.to(DEV)
    cs_o, ss_o = cs.double().numpy(), ss.double().numpy()
    for _ in range(4):
        x, z = torch.randn(b, D, generator=g), torch.randn(b, D, generator=g)
        dr = torch.randn(b, D, generator=g) * 0.5
        Bm, Cm = torch.randn(b, N, generator=g), torch.randn(b, N, generator=g)
        y = decode_step(x.to(DEV), cs_d, dv["cw"], dv["cb"], dr.to(DEV), Bm.to(DEV), Cm.to(DEV), dv["A"], ss_d,
                        Dskip=dv["Dskip"], z=z.to(DEV), delta_bias=dv["dbias"])
        yo, cs_o, ss_o, _ = oracle.decode_step(x, z, dr, Bm, Cm, p["cw"], p["cb"], p["A"], p["Dskip"], p["dbias"],
                                               cs_o, ss_o)
        torch.cuda.synchronize()
        for got, want, name in ((y, yo, "y"), (ss_d, ss_o, "ssm_state"), (cs_d, cs_o, "conv_state")):
            np.testing.assert_allclose(n64(got), want, rtol=1e-4, atol=1e-5, err_msg=name)
