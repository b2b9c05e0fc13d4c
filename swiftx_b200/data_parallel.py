"""Data-parallel gradient plumbing for training on one process per GPU.

The reference trains on one device (training/train.py:133-172).  Data parallelism across
GPUs adds one exchange per step: every parameter's gradient is a view into one flat fp32
buffer, so a single all-reduce (average over the ranks) replaces per-parameter
collectives, and the clip and the optimizer step that follow see the averaged gradient
through the ordinary ``p.grad`` attributes.  With equal per-rank batches, averaging the
ranks' mean-loss gradients gives the gradient of the mean loss over the global batch.

The buffer is allocated once, so CUDA-graph captures of the forward + backward keep
writing into the same memory, and the all-reduce can run between two graph replays.
"""
import torch
import torch.distributed as dist


def broadcast_parameters(params, src=0, group=None):
    """Give every rank the parameters of rank ``src`` (an identical start)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        for p in params:
            dist.broadcast(p.data, src=src, group=group)


class FlatGradients:
    """One flat buffer holding every parameter's gradient as a view.

    params: the parameters, in a fixed order (the same on every rank).  After
    construction ``p.grad`` of each is a view into ``self.flat``; autograd accumulates
    into those views in place, so ``zero_()`` (not ``optimizer.zero_grad``, which would
    drop the views) clears them between steps."""

    def __init__(self, params, device=None, dtype=torch.float32):
        self.params = list(params)
        if not self.params:
            raise ValueError("FlatGradients needs at least one parameter")
        dev = device if device is not None else self.params[0].device
        n = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(n, device=dev, dtype=dtype)
        off = 0
        for p in self.params:
            if p.dtype != dtype:
                raise ValueError(f"parameter dtype {p.dtype} differs from the gradient buffer's {dtype}")
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()

    def zero_(self):
        self.flat.zero_()

    def all_reduce_(self, group=None):
        """Average the gradient buffer over the ranks of ``group`` (no-op on one rank)."""
        if not (dist.is_available() and dist.is_initialized()):
            return
        world = dist.get_world_size(group)
        if world == 1:
            return
        if dist.get_backend(group) == "nccl":
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=group)
        else:                                   # gloo has no AVG: sum, then scale
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
            self.flat.div_(world)
