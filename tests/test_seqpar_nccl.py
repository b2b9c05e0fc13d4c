"""Sequence-parallel scan over NCCL on 2+ GPUs (skipped with fewer): every rank scans
its chunk (the balanced split of seqpar.chunk_bounds) from a zero state, the boundary
values go peer to peer to the later ranks, each later rank corrects its output for its
initial state, and the rank outputs concatenated along the sequence must match a
one-pass scan of the whole sequence on one GPU."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from swiftx_b200.seqpar import chunk_bounds, sequence_parallel_scan
    from swiftx_b200.workloads import config_inputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        b, L, D = 2, 600, 64
        inp = config_inputs(b, L, D, 16, seed=5, device=f"cuda:{rank}")
        bounds = chunk_bounds(L, world, correction_offset=0, multiple=8)
        s, e = bounds[rank], bounds[rank + 1]
        ch = {k: inp[k][:, s:e] for k in ("u", "delta", "z", "B", "C")}
        out = sequence_parallel_scan(ch["u"], ch["delta"], inp["A"], ch["B"], ch["C"], inp["D"], ch["z"],
                                     inp["delta_bias"], True)
        torch.cuda.synchronize()
        q.put((rank, out.cpu().numpy()))
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_over_nccl():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    from swiftx_b200.selective_scan import scan_forward
    from swiftx_b200.workloads import config_inputs
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inp = config_inputs(2, 600, 64, 16, seed=5, device="cuda:0")
    whole, _, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                               inp["delta_bias"], True)
    out = np.concatenate([got[r] for r in range(world)], axis=1)
    np.testing.assert_allclose(out, whole.cpu().numpy(), rtol=1e-4, atol=1e-5)
