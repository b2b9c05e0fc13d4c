"""Seeded synthetic workloads of the benchmark configurations (also used by the tests).

``config_inputs`` draws the benchmark value distributions (u ~ N(0,1);
delta_raw ~ N(0, 0.5); delta_bias = inverse-softplus(dt) with dt log-uniform in
[1e-3, 0.1] as in the reference's init_dt_proj (models/ssm.py:54-71); A = -(1..N)
as in init_A_log (models/ssm.py:43-51); B, C ~ N(0,1); D = 1; z ~ N(0,1)),
drawn in (b, D, L) / (b, N, L) order and transposed to the reference layout.
"""
import math

import torch


def config_inputs(b, L, D, N, seed=0, gate=True, device="cpu", dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(b, D, L, generator=g).transpose(1, 2)
    dr = (torch.randn(b, D, L, generator=g) * 0.5).transpose(1, 2)
    dt = torch.exp(torch.rand(D, generator=g) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    bias = dt + torch.log(-torch.expm1(-dt))
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1)
    Bm = torch.randn(b, N, L, generator=g).transpose(1, 2)
    Cm = torch.randn(b, N, L, generator=g).transpose(1, 2)
    Dskip = torch.ones(D)
    z = torch.randn(b, D, L, generator=g).transpose(1, 2) if gate else None
    dout = torch.randn(b, L, D, generator=g)
    to = lambda t, dt=dtype: None if t is None else t.contiguous().to(device=device, dtype=dt)  # noqa: E731
    return dict(u=to(u), delta=to(dr), delta_bias=to(bias, torch.float32), A=to(A, torch.float32),
                B=to(Bm), C=to(Cm), D=to(Dskip, torch.float32), z=to(z), dout=to(dout))


def reference_test_inputs(b, L, D, N, seed=0, device="cpu"):
    """The reference test suite's generator (tests/test_selective_scan.py:14-22)."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(b, L, D, generator=g)
    delta = torch.rand(b, L, D, generator=g) * 0.5 + 0.01
    A = -torch.rand(D, N, generator=g) - 0.1
    B = torch.randn(b, L, N, generator=g)
    C = torch.randn(b, L, N, generator=g)
    Dskip = torch.randn(D, generator=g)
    return [t.to(device) for t in (u, delta, A, B, C, Dskip)]
