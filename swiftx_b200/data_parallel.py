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

    params: the parameters, in a fixed order (the same on every rank).  Two ways to fill it:

    * accumulate=True: ``p.grad`` of each parameter is a view into ``self.flat`` from
      construction on; autograd accumulates into those views in place, so ``zero_()``
      (not ``optimizer.zero_grad``, which would drop the views) clears them between steps.
    * accumulate=False: ``zero_()`` drops every ``p.grad``, so the backward assigns each
      parameter its gradient as computed -- no zero fill of the buffer and no
      per-parameter accumulation kernel (one elementwise add per parameter per step
      otherwise).  ``pack_()`` then copies them into the buffer with one multi-tensor copy
      and points ``p.grad`` at its views, when there is an all-reduce to feed.

    In both modes, after ``zero_()``, a backward, ``pack_()`` and ``all_reduce_()``, every
    ``p.grad`` holds the gradient averaged over the ranks."""

    def __init__(self, params, device=None, dtype=torch.float32, accumulate=True):
        self.params = list(params)
        if not self.params:
            raise ValueError("FlatGradients needs at least one parameter")
        dev = device if device is not None else self.params[0].device
        n = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(n, device=dev, dtype=dtype)
        self.accumulate = accumulate
        self.views = []
        off = 0
        for p in self.params:
            if p.dtype != dtype:
                raise ValueError(f"parameter dtype {p.dtype} differs from the gradient buffer's {dtype}")
            self.views.append(self.flat[off:off + p.numel()].view_as(p))
            off += p.numel()
        if accumulate:
            for p, v in zip(self.params, self.views):
                p.grad = v

    def zero_(self):
        """Before a backward: clear the buffer (accumulate mode) or drop every p.grad."""
        if self.accumulate:
            self.flat.zero_()
        else:
            for p in self.params:
                p.grad = None

    def pack_(self, group=None, always=False):
        """After a backward (accumulate=False): when the process group has more than one
        rank, or ``always`` (an optimizer that reads the flat buffer itself, see
        FlatParameters), copy every p.grad into the buffer (a parameter without a gradient
        gets zeros) and point p.grad at the buffer's views.  Otherwise, and in accumulate
        mode, the gradients are already where the optimizer reads them: nothing to do."""
        if self.accumulate or (_world(group) == 1 and not always):
            return
        have = [(v, p.grad) for v, p in zip(self.views, self.params) if p.grad is not None]
        for v, p in zip(self.views, self.params):
            if p.grad is None:
                v.zero_()
        if have:
            torch._foreach_copy_([v for v, _ in have], [g for _, g in have])
        for p, v in zip(self.params, self.views):
            p.grad = v

    def all_reduce_(self, group=None):
        """Average the gradient buffer over the ranks of ``group`` (no-op on one rank)."""
        world = _world(group)
        if world == 1:
            return
        if dist.get_backend(group) == "nccl":
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=group)
        else:                                   # gloo has no AVG: sum, then scale
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
            self.flat.div_(world)


def _world(group=None):
    """Ranks in ``group``: 1 without an initialised process group."""
    if not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


class FlatParameters:
    """The parameters re-homed into one contiguous buffer per group.

    groups: lists of parameters (e.g. those with and without weight decay).  Each
    parameter's ``.data`` becomes a view of its group's buffer, in the given order, with
    its values kept; ``flats[i]`` is a Parameter over the whole buffer of group i.  With a
    FlatGradients built over the same parameters in the same order, ``bind_gradients``
    points each flat Parameter's ``.grad`` at the matching slice of the gradient buffer,
    so an optimizer given ``flats`` updates every parameter in one pass per group instead
    of one per tensor.  The optimizer's arithmetic is element-wise, so the update is the
    one it would make over the separate tensors."""

    def __init__(self, groups, dtype=torch.float32):
        self.groups = [list(g) for g in groups]
        self.flats = []
        for ps in self.groups:
            if not ps:
                raise ValueError("FlatParameters needs a non-empty group")
            n = sum(p.numel() for p in ps)
            buf = torch.empty(n, device=ps[0].device, dtype=dtype)
            off = 0
            for p in ps:
                if p.dtype != dtype:
                    raise ValueError(f"parameter dtype {p.dtype} differs from the buffer's {dtype}")
                v = buf[off:off + p.numel()].view_as(p)
                v.copy_(p.data)
                p.data = v
                off += p.numel()
            self.flats.append(torch.nn.Parameter(buf))

    def bind_gradients(self, grads):
        """Point each flat Parameter's .grad at its slice of ``grads.flat`` (FlatGradients
        over the concatenated groups, same order).  Call once; the slices stay valid."""
        order = [p for g in self.groups for p in g]
        if len(order) != len(grads.params) or any(a is not b for a, b in zip(order, grads.params)):
            raise ValueError("the gradient buffer must hold the groups' parameters in the same order")
        off = 0
        for flat in self.flats:
            flat.grad = grads.flat[off:off + flat.numel()]
            off += flat.numel()
