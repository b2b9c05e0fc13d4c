"""Sequence-parallel scan on one GPU: chunks scanned as separate 'ranks' (each chunk's
forward from a zero state -> boundary values -> prefix combine -> the initial-state
correction swx_scan_correct) must reproduce the one-pass scan of the whole sequence and
the oracle."""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.selective_scan import scan_correct, scan_forward
from swiftx_b200.seqpar import combine_prefix
from swiftx_b200.workloads import config_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def chunked_scan(inp, bounds, out_dtype=torch.float32):
    keys = ("u", "delta", "z", "B", "C")
    outs, ends, sums = [], [], []
    for s, e in zip(bounds[:-1], bounds[1:]):
        ch = {k: inp[k][:, s:e] for k in keys}
        out, _, h_end, dsum = scan_forward(ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], inp["D"], ch["z"],
                                           inp["delta_bias"], True, out_dtype=out_dtype, return_last_state=True,
                                           return_delta_sum=True)
        outs.append(out)
        ends.append(h_end)
        sums.append(dsum)
    for g, (s, e) in enumerate(zip(bounds[:-1], bounds[1:])):
        if g == 0:
            continue
        ch = {k: inp[k][:, s:e] for k in keys}
        h_in = combine_prefix(ends, sums, inp["A"].float(), g)
        scan_correct(outs[g], h_in, ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], z=ch["z"],
                     delta_bias=inp["delta_bias"], delta_softplus=True)
    return torch.cat(outs, 1)


@pytest.mark.parametrize("dtype,out_dtype,gate,N", [(torch.float32, torch.float32, True, 16),
                                                    (torch.float32, torch.float32, False, 5),
                                                    (torch.bfloat16, torch.float32, True, 16),
                                                    (torch.bfloat16, torch.bfloat16, True, 12)])
def test_correct_equals_scan_from_initial_state(dtype, out_dtype, gate, N):
    """swx_scan_correct turns the forward from a zero state into the forward from h_in:
    against the kernel's own forward with h0 = h_in and against the oracle (D not a
    multiple of the 128-channel block, L not a multiple of the 256-step block)."""
    b, L, D = 2, 700, 200
    inp = config_inputs(b, L, D, N, seed=13, gate=gate, device=DEV, dtype=dtype)
    h_in = (torch.randn(b, D, N, generator=torch.Generator().manual_seed(1)) * 0.5).to(DEV)
    z = inp["z"] if gate else None
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], z, inp["delta_bias"], True)
    out0, _, _ = scan_forward(*args, out_dtype=out_dtype)
    want_k, _, _ = scan_forward(*args, h0=h_in, out_dtype=out_dtype)
    got = scan_correct(out0, h_in, inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], z=z,
                       delta_bias=inp["delta_bias"], delta_softplus=True)
    n = lambda t: None if t is None else t.double().cpu().numpy()  # noqa: E731
    want = oracle.scan_fwd(*(n(inp[k]) for k in ("u", "delta", "A", "B", "C")), D=n(inp["D"]), z=n(z),
                           delta_bias=n(inp["delta_bias"]), delta_softplus=True, h0=n(h_in))
    tol = dict(rtol=1e-4, atol=1e-5) if (dtype, out_dtype) == (torch.float32, torch.float32) else \
        dict(rtol=2e-2, atol=2e-2 * np.abs(want).max())
    np.testing.assert_allclose(n(got), want, **tol)
    np.testing.assert_allclose(n(got), n(want_k), **tol)


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


def test_correct_after_the_decays_underflow():
    """A long chunk whose decays exp(A S_t) underflow for whole warps part way (large dt,
    so S_t grows fast): the kernel stops evaluating those state pairs once every lane's
    decay is 0 in fp32, which must leave the result equal to the float64 formula
    out_t += silu(z_t) sum_n C_t[n] exp(A[:, n] S_t) h_in[n] (the skipped terms are
    exactly zero in fp32).  Half the channels decay slowly (dt 1e-3), so some pairs stay
    live to the end."""
    b, L, D, N = 2, 4096, 256, 16
    g = torch.Generator().manual_seed(21)
    dt = torch.where(torch.arange(D) % 64 < 32, torch.full((D,), 0.2), torch.full((D,), 1e-3))
    bias = (dt + torch.log(-torch.expm1(-dt))).to(DEV)
    delta = (torch.randn(b, L, D, generator=g) * 0.3).to(DEV)
    C = torch.randn(b, L, N, generator=g).to(DEV)
    z = torch.randn(b, L, D, generator=g).to(DEV)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).to(DEV)
    h_in = (torch.randn(b, D, N, generator=g) * 0.5).to(DEV)
    u, Bm = torch.zeros(b, L, D, device=DEV), torch.zeros(b, L, N, device=DEV)
    out0 = torch.randn(b, L, D, generator=g).to(DEV)
    got = scan_correct(out0.clone(), h_in, u, delta, A, Bm, C, z=z, delta_bias=bias, delta_softplus=True)
    S = torch.cumsum(torch.nn.functional.softplus(delta.double() + bias.double()), 1)       # (b, L, D)
    P = torch.exp(A.double()[None, None] * S[..., None])                                     # (b, L, D, N)
    corr = torch.einsum("bln,bldn,bdn->bld", C.double(), P, h_in.double()) * torch.nn.functional.silu(z.double())
    want = out0.double() + corr
    np.testing.assert_allclose(got.double().cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-5)
