"""Host logic of the sequence-parallel scan on CPU ranks (gloo, world sizes 2 and 3).

Each rank runs sequence_parallel_scan on its chunk; the two kernel calls are replaced
through the hooks: the chunk's scan from a zero state by the CPU oracle, and the
initial-state correction by a float64 NumPy restatement of its formula
(out_t += silu(z_t) sum_n C_t[n] exp(A[:, n] S_t) h_in[n]).  What is tested is the
peer-to-peer boundary exchange, the prefix combine and the correction's mathematics:
the concatenated outputs must equal the oracle's scan of the whole sequence, also when
a rank's chunk is empty (chunk_bounds gives short sequences to rank 0 alone): its
boundary passes the earlier ranks' state through unchanged."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from swiftx_b200.seqpar import chunk_bounds, combine_prefix, sequence_parallel_scan
from swiftx_b200.workloads import config_inputs

B_, L_, D_, N_ = 2, 90, 12, 16


def oracle_local_scan(u, delta, A, B, C, D, z, delta_bias, softplus, out_dtype):
    n = lambda t: None if t is None else t.double().numpy()  # noqa: E731
    out, h_end = oracle.scan_fwd(n(u), n(delta), n(A), n(B), n(C), n(D), z=n(z), delta_bias=n(delta_bias),
                                 delta_softplus=softplus, return_last_state=True)
    return torch.from_numpy(out), torch.from_numpy(h_end), _delta_eff(delta, delta_bias, softplus).sum(1)


def _delta_eff(delta, delta_bias, softplus):
    bias = delta_bias.double() if delta_bias is not None else 0.0
    return torch.nn.functional.softplus(delta.double() + bias) if softplus else delta.double() + bias


def numpy_correct(out, h_in, u, delta, A, B, C, z, delta_bias, softplus):
    """out_t += silu(z_t) * sum_n C_t[n] * exp(A[d, n] * S_t) * h_in[d, n], S_t = sum_{s<=t} delta_eff."""
    S = torch.cumsum(_delta_eff(delta, delta_bias, softplus), 1).numpy()           # (b, L, D)
    P = np.exp(A.double().numpy()[None, None] * S[..., None])                       # (b, L, D, N)
    corr = np.einsum("bln,bldn,bdn->bld", C.double().numpy(), P, h_in.double().numpy())
    if z is not None:
        zz = z.double().numpy()
        corr = corr * zz / (1.0 + np.exp(-zz))
    return out + torch.from_numpy(corr)


def _worker(rank, world, port, bounds, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inp = config_inputs(B_, L_, D_, N_, seed=3)
        s, e = bounds[rank], bounds[rank + 1]
        ch = {k: inp[k][:, s:e] for k in ("u", "delta", "z", "B", "C")}
        out = sequence_parallel_scan(ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], inp["D"], ch["z"],
                                     inp["delta_bias"], True, local_scan=oracle_local_scan,
                                     correct=numpy_correct)
        q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("bounds", [[0, 41, 90], [0, 30, 31, 90], chunk_bounds(90, 3, correction_offset=0, multiple=1),
                                    [0, 90, 90], [0, 60, 60, 90]])
def test_sequence_parallel_matches_whole_sequence(bounds):
    world = len(bounds) - 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, bounds, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out = np.concatenate([got[r] for r in range(world)], axis=1)
    inp = config_inputs(B_, L_, D_, N_, seed=3)
    want = oracle.scan_fwd(*(inp[k] for k in ("u", "delta", "A", "B", "C")), D=inp["D"], z=inp["z"],
                           delta_bias=inp["delta_bias"], delta_softplus=True)
    np.testing.assert_allclose(out, want, rtol=1e-9, atol=1e-10)


def test_combine_prefix_is_the_chained_recurrence():
    g = torch.Generator().manual_seed(0)
    b, D, N = 2, 3, 4
    A = -torch.rand(D, N, generator=g, dtype=torch.float64) - 0.1
    h_ends = [torch.randn(b, D, N, generator=g, dtype=torch.float64) for _ in range(4)]
    dsums = [torch.rand(b, D, generator=g, dtype=torch.float64) for _ in range(4)]
    h = torch.zeros(b, D, N, dtype=torch.float64)
    for k in range(3):
        h = torch.exp(A * dsums[k][..., None]) * h + h_ends[k]
    assert torch.allclose(combine_prefix(h_ends, dsums, A, 3), h)
    assert torch.equal(combine_prefix(h_ends, dsums, A, 0), torch.zeros(b, D, N, dtype=torch.float64))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_chunk_bounds_balance(world):
    L, c, c0 = 65536, 0.73, 950
    b = chunk_bounds(L, world, correction_cost=c, correction_offset=c0)
    assert b[0] == 0 and b[-1] == L and len(b) == world + 1
    lens = [b[r + 1] - b[r] for r in range(world)]
    assert all(n > 0 and n % 256 == 0 for n in lens)
    # every rank's modelled time (forward, plus the correction on ranks > 0) within one
    # rounding unit of the others
    cost = [lens[0]] + [(1 + c) * n + c0 for n in lens[1:]]
    assert max(cost) - min(cost) <= 2 * 256 * (1 + c)


def test_chunk_bounds_short_sequence():
    """A sequence too short for the correction's fixed cost: rank 0 takes it whole."""
    assert chunk_bounds(512, 4) == [0, 512, 512, 512, 512]
