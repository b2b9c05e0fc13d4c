"""Sequence-parallel selective scan across the ranks of a process group.

A long sequence is split into contiguous chunks, one per rank in rank order.  The
recurrence h_t = a_t h_{t-1} + x_t is affine in the initial state, so with h0 = 0 each
rank's chunk ends in a local state h_end and carries the decay P = prod_t a_t =
exp(A * sum_t delta_eff_t) (per batch row, channel and state).  The true initial state
of chunk g is the prefix  h_in_g = P_{g-1} h_in_{g-1} + h_end_{g-1},  h_in_0 = 0.

  pass 1: local scan without output -> (h_end, sum_t delta_eff)       [kernel, WR=false]
  exchange: all_gather of the 2*b*D*N fp32 boundary values over NCCL (NVLink)
  combine: the prefix above for the ranks before this one (tiny, on the GPU)
  pass 2: full scan of the chunk from h_in (gate, D skip, output)     [kernel]

The two passes are the cost of chunking: both walk every element's decay.
"""
import torch
import torch.distributed as dist

from .selective_scan import scan_forward


def _kernel_local_scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0, write_out, out_dtype):
    if not write_out:
        _, _, h_end, dsum = scan_forward(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0=h0,
                                         out_dtype=out_dtype, return_last_state=True,
                                         return_delta_sum=True, write_out=False)
        return None, h_end, dsum
    out, _, _ = scan_forward(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0=h0,
                             out_dtype=out_dtype)
    return out, None, None


def combine_prefix(h_end_all, dsum_all, A, rank):
    """Initial state of chunk `rank` from the boundary values of chunks 0..rank-1.

    h_end_all[k]: (b, D, N) final state of chunk k scanned from zero;
    dsum_all[k]:  (b, D) sum over chunk k of delta_eff;  A: (D, N)."""
    h = torch.zeros_like(h_end_all[0])
    A = A.to(h.dtype)
    for k in range(rank):
        h = torch.exp(A.unsqueeze(0) * dsum_all[k].unsqueeze(-1)) * h + h_end_all[k]
    return h


def sequence_parallel_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=True,
                           group=None, out_dtype=torch.float32, local_scan=None):
    """Forward selective scan of a sequence split across the ranks of `group`.

    Each rank passes its own chunk (b, L_rank, D) / (b, L_rank, N) of u, delta, z, B, C,
    in rank order along the sequence; A, D, delta_bias are replicated.  Returns this
    rank's (b, L_rank, D) output.  `local_scan` replaces the per-chunk kernel call (the
    tests use it to drive the host logic on CPU ranks)."""
    scan = local_scan or _kernel_local_scan
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, _, Dm = u.shape
    N = A.shape[1]
    h0 = None
    if world > 1:
        _, h_end, dsum = scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, None, False, out_dtype)
        pack = torch.cat([h_end.reshape(-1), dsum.reshape(-1).to(h_end.dtype)])
        parts = [torch.empty_like(pack) for _ in range(world)]
        dist.all_gather(parts, pack, group=group)
        nh = b * Dm * N
        h_ends = [q[:nh].view(b, Dm, N) for q in parts]
        dsums = [q[nh:].view(b, Dm) for q in parts]
        if rank > 0:
            h0 = combine_prefix(h_ends, dsums, A, rank)
    out, _, _ = scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0, True, out_dtype)
    return out
