"""Data-parallel training of the Sift LM over NCCL on 2+ GPUs (skipped with fewer), the
way bench.py's LM workload runs it: the gradients land in one flat buffer (accumulated
into its views, or assigned by the backward and packed into it) that is all-reduced
(average) once per step, then the clip and the optimizer step.  After three
steps on their halves of a global batch the ranks must hold identical parameters, equal
(to fp32 re-association) to one GPU training on the whole batch.  The optimizer here is
plain SGD, whose update is linear in the gradient, so rounding-level gradient
differences stay rounding-level in the parameters (Adam's first steps move each
parameter by about +-lr whatever the gradient's size)."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
STEPS, ROWS_PER_RANK, SEQ = 3, 2, 24


def _batch(world):
    g = torch.Generator().manual_seed(7)
    return torch.randint(0, 11, (world * ROWS_PER_RANK, SEQ + 1), generator=g)


def _train(tok, dev, accumulate=True):
    from swiftx_b200.data_parallel import FlatGradients, broadcast_parameters
    from swiftx_b200.sift import SiftConfig, SiftLM
    torch.manual_seed(0)
    m = SiftLM(SiftConfig(vocab_size=11, d_model=32, n_layers=2, d_state=8)).to(dev)
    params = list(m.parameters())
    broadcast_parameters(params)
    grads = FlatGradients(params, accumulate=accumulate)
    opt = torch.optim.SGD(params, lr=0.1)
    tok = tok.to(dev)
    for _ in range(STEPS):
        grads.zero_()
        _, loss = m(tok[:, :-1], tok[:, 1:])
        loss.backward()
        grads.pack_()
        grads.all_reduce_()
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
    torch.cuda.synchronize()
    return torch.cat([p.detach().reshape(-1) for p in params]).cpu().numpy()


def _worker(rank, world, port, accumulate, q):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        tok = _batch(world)[rank * ROWS_PER_RANK:(rank + 1) * ROWS_PER_RANK]
        out = _train(tok, torch.device("cuda", rank), accumulate)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("accumulate", [True, False], ids=["accumulate", "assign"])
def test_data_parallel_training_over_nccl(accumulate):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, accumulate, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(1, world):
        assert np.array_equal(got[r], got[0]), f"rank {r} diverged from rank 0"
    whole = _train(_batch(world), torch.device("cuda", 0), accumulate)
    np.testing.assert_allclose(got[0], whole, rtol=1e-4, atol=1e-5)
