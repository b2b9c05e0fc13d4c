"""Data-parallel gradient plumbing (swiftx_b200.data_parallel) on CPU ranks over gloo.

Two ranks start from rank 0's parameters (broadcast), train a small MLP for three steps
on their halves of a global batch with every gradient in one flat buffer that is
averaged across the ranks each step, then clip and SGD -- with the gradients accumulated
into the buffer's views, and with them assigned by the backward and packed into the
buffer.  Both ranks must end with identical parameters, equal (to fp32 re-association)
to one process training on the whole batch.  The same class drives the GPU LM's
data-parallel step over NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from swiftx_b200.data_parallel import FlatGradients, FlatParameters, broadcast_parameters

STEPS, ROWS_PER_RANK, WORLD = 3, 6, 2


def _data():
    g = torch.Generator().manual_seed(5)
    return torch.randn(WORLD * ROWS_PER_RANK, 10, generator=g), torch.randn(WORLD * ROWS_PER_RANK, 3, generator=g)


def _train(x, y, seed, accumulate=True):
    torch.manual_seed(seed)                   # ranks other than 0 start elsewhere until the broadcast
    m = torch.nn.Sequential(torch.nn.Linear(10, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3))
    unused = torch.nn.Parameter(torch.randn(4))   # no gradient reaches it: packed as zeros
    params = list(m.parameters()) + [unused]
    broadcast_parameters(params)
    grads = FlatGradients(params, accumulate=accumulate)
    opt = torch.optim.SGD(params, lr=0.2)
    for _ in range(STEPS):
        grads.zero_()
        torch.nn.functional.mse_loss(m(x), y).backward()
        grads.pack_()
        grads.all_reduce_()
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
    if accumulate or (dist.is_initialized() and dist.get_world_size() > 1):
        assert all(p.grad._base is grads.flat for p in params)  # the optimizer read the buffer
    return torch.cat([p.detach().reshape(-1) for p in params]).numpy()


def _worker(rank, port, accumulate, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        x, y = _data()
        rows = slice(rank * ROWS_PER_RANK, (rank + 1) * ROWS_PER_RANK)
        q.put((rank, _train(x[rows], y[rows], seed=rank, accumulate=accumulate)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("accumulate", [True, False], ids=["accumulate", "assign"])
def test_flat_gradients_average_over_gloo_ranks(accumulate):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, accumulate, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got[1], got[0]), "ranks diverged"
    x, y = _data()
    whole = _train(x, y, seed=0, accumulate=accumulate)    # one process, whole batch, no process group
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


def test_assign_mode_leaves_gradients_to_autograd_on_one_rank():
    a = torch.nn.Parameter(torch.randn(3, 4))
    b = torch.nn.Parameter(torch.randn(5))
    fg = FlatGradients([a, b], accumulate=False)
    assert a.grad is None and b.grad is None
    for k in range(2):                         # no accumulation across steps
        fg.zero_()
        assert a.grad is None
        ((k + 1) * a.sum() + (b * b).sum()).backward()
        fg.pack_()                             # one rank: the assigned gradients stay
        np.testing.assert_allclose(a.grad.numpy(), k + 1.0)
        np.testing.assert_allclose(b.grad.numpy(), (2 * b).detach().numpy())
        assert a.grad._base is not fg.flat


def test_flat_parameters_keep_values_and_update_like_separate_tensors():
    """FlatParameters re-homes the parameters into one buffer per group without changing
    their values, and AdamW over the two flat Parameters (gradients bound to the packed
    gradient buffer) makes bit for bit the update of AdamW over the separate tensors."""
    g = torch.Generator().manual_seed(3)
    shapes = [(4, 3), (5,), (2, 2, 2), (7,)]
    ps_a = [torch.nn.Parameter(torch.randn(s, generator=g)) for s in shapes]
    ps_b = [torch.nn.Parameter(p.detach().clone()) for p in ps_a]
    decay_b, nodecay_b = [ps_b[0], ps_b[2]], [ps_b[1], ps_b[3]]
    flat = FlatParameters([decay_b, nodecay_b])
    for a, b in zip(ps_a, ps_b):
        assert torch.equal(a.detach(), b.detach())
    assert ps_b[2].data.data_ptr() == flat.flats[0].data_ptr() + 12 * 4       # a view of the buffer
    grads = FlatGradients(decay_b + nodecay_b, accumulate=False)
    flat.bind_gradients(grads)
    kw = dict(lr=1e-2, betas=(0.9, 0.95), foreach=False)
    opt_a = torch.optim.AdamW([{"params": [ps_a[0], ps_a[2]], "weight_decay": 0.1},
                               {"params": [ps_a[1], ps_a[3]], "weight_decay": 0.0}], **kw)
    opt_b = torch.optim.AdamW([{"params": [flat.flats[0]], "weight_decay": 0.1},
                               {"params": [flat.flats[1]], "weight_decay": 0.0}], **kw)
    for _ in range(3):
        gs = [torch.randn(s, generator=g) for s in shapes]
        for p, gr in zip(ps_a, gs):
            p.grad = gr.clone()
        grads.zero_()
        for p, gr in zip(ps_b, gs):
            p.grad = gr.clone()
        grads.pack_(always=True)
        opt_a.step()
        opt_b.step()
        for a, b in zip(ps_a, ps_b):
            assert torch.equal(a.detach(), b.detach())
    with pytest.raises(ValueError):
        flat.bind_gradients(FlatGradients(list(reversed(decay_b + nodecay_b)), accumulate=False))


def test_flat_parameters_reject_empty_groups_and_mixed_dtypes():
    with pytest.raises(ValueError):
        FlatParameters([[torch.nn.Parameter(torch.zeros(3))], []])
    with pytest.raises(ValueError):
        FlatParameters([[torch.nn.Parameter(torch.zeros(3)), torch.nn.Parameter(torch.zeros(2, dtype=torch.float64))]])
