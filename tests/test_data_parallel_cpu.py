"""Data-parallel gradient plumbing (swiftx_b200.data_parallel) on CPU ranks over gloo.

Two ranks start from rank 0's parameters (broadcast), train a small MLP for three steps
on their halves of a global batch with every gradient a view into one flat buffer that
is averaged across the ranks each step, then clip and SGD.  Both ranks must end with
identical parameters, equal (to fp32 re-association) to one process training on the
whole batch.  The same class drives the GPU LM's data-parallel step over NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from swiftx_b200.data_parallel import FlatGradients, broadcast_parameters

STEPS, ROWS_PER_RANK, WORLD = 3, 6, 2


def _data():
    g = torch.Generator().manual_seed(5)
    return torch.randn(WORLD * ROWS_PER_RANK, 10, generator=g), torch.randn(WORLD * ROWS_PER_RANK, 3, generator=g)


def _train(x, y, seed):
    torch.manual_seed(seed)                   # ranks other than 0 start elsewhere until the broadcast
    m = torch.nn.Sequential(torch.nn.Linear(10, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3))
    params = list(m.parameters())
    broadcast_parameters(params)
    grads = FlatGradients(params)
    opt = torch.optim.SGD(params, lr=0.2)
    for _ in range(STEPS):
        grads.zero_()
        torch.nn.functional.mse_loss(m(x), y).backward()
        grads.all_reduce_()
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
    assert all(p.grad._base is grads.flat for p in params)      # autograd kept the views
    return torch.cat([p.detach().reshape(-1) for p in params]).numpy()


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        x, y = _data()
        rows = slice(rank * ROWS_PER_RANK, (rank + 1) * ROWS_PER_RANK)
        q.put((rank, _train(x[rows], y[rows], seed=rank)))
    finally:
        dist.destroy_process_group()


def test_flat_gradients_average_over_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got[1], got[0]), "ranks diverged"
    x, y = _data()
    whole = _train(x, y, seed=0)               # one process, whole batch, no process group
    np.testing.assert_allclose(got[0], whole, rtol=1e-5, atol=1e-6)


def test_flat_gradients_bind_views_and_reject_mixed_dtypes():
    a = torch.nn.Parameter(torch.randn(3, 4))
    b = torch.nn.Parameter(torch.randn(5))
    fg = FlatGradients([a, b])
    assert fg.flat.numel() == 17
    (a.sum() * 2 + (b * b).sum()).backward()
    np.testing.assert_allclose(fg.flat[:12].numpy(), 2.0)
    np.testing.assert_allclose(fg.flat[12:].numpy(), (2 * b).detach().numpy())
    fg.zero_()
    assert a.grad.abs().sum() == 0 and b.grad.abs().sum() == 0
    fg.all_reduce_()                           # no process group: a no-op
    with pytest.raises(ValueError, match="dtype"):
        FlatGradients([torch.nn.Parameter(torch.randn(2, dtype=torch.float64))])
    with pytest.raises(ValueError, match="at least one"):
        FlatGradients([])
