"""Sequence-parallel selective scan across the ranks of a process group.

A long sequence is split into contiguous chunks, one per rank in rank order.  The scan
is linear in its initial state: with h0 = 0 each rank's chunk ends in a local state
h_end and carries the decay P = exp(A * sum_t delta_eff_t) (per batch row, channel and
state), and the true initial state of chunk g is the prefix
    h_in_g = P_{g-1} h_in_{g-1} + h_end_{g-1},   h_in_0 = 0.

  pass 1: the chunk's full forward from h0 = 0 (gated output, h_end, sum of delta_eff)
  exchange: each rank sends its 2 b D N-sized boundary values peer to peer to every later
            rank (NCCL send/recv over NVLink, grouped; no collective over all ranks)
  combine: the prefix above over the earlier ranks, in rank order (tiny, on the GPU)
  correct: out_t += silu(z_t) sum_n C_t[n] exp(A[:, n] S_t) h_in[n], S_t the running
           sum of delta_eff (swx_scan_correct) -- no step waits for the previous one
           except through S_t, so it runs at the throughput of its exponentials, not as
           a second serial walk of the chunk.
Rank 0 needs no correction, so an even split leaves it idle while the later ranks
correct; chunk_bounds() gives rank 0 the longer chunk that evens out the ranks' times.
"""
import torch
import torch.distributed as dist

from .selective_scan import scan_correct, scan_forward


def _kernel_local_scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, out_dtype):
    out, _, h_end, dsum = scan_forward(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                                       out_dtype=out_dtype, return_last_state=True, return_delta_sum=True)
    return out, h_end, dsum


def _kernel_correct(out, h_in, u, delta, A, B, C, z, delta_bias, delta_softplus):
    return scan_correct(out, h_in, u, delta, A, B, C, z=z, delta_bias=delta_bias,
                        delta_softplus=delta_softplus)


def chunk_bounds(L, world, correction_cost=0.73, correction_offset=950, multiple=256):
    """Chunk boundaries [0, e_0, ..., L] that balance the ranks' work: rank 0 runs only the
    forward of its chunk, every later rank the forward and the correction.  In units of
    one forward step, a chunk of n steps costs n to scan and correction_offset +
    correction_cost * n to correct.  The defaults are fitted to one B200 at b=4, D=2048,
    N=16, bf16 in / fp32 out: the forward at 73.5 ns a step, the correction 1.83 ms at
    32768 steps and 0.51 ms at 8192.  With rank 0's length x and the others' y:
    x = (1 + cost) y + offset and x + (world - 1) y = L.  Lengths are rounded to
    `multiple` steps; the last rank takes the remainder."""
    if world <= 1:
        return [0, L]
    y = max(0.0, (L - correction_offset) / (world + correction_cost))
    x = L - (world - 1) * y
    lens = [x] + [y] * (world - 1)
    bounds, acc = [0], 0.0
    for r in range(world - 1):
        acc += lens[r]
        e = int(round(acc / multiple)) * multiple
        bounds.append(min(max(e, bounds[-1]), L))
    bounds.append(L)
    return bounds


def combine_prefix(h_end_all, dsum_all, A, rank):
    """Initial state of chunk `rank` from the boundary values of chunks 0..rank-1.

    h_end_all[k]: (b, D, N) final state of chunk k scanned from zero;
    dsum_all[k]:  (b, D) sum over chunk k of delta_eff;  A: (D, N)."""
    h = torch.zeros_like(h_end_all[0])
    A = A.to(h.dtype)
    for k in range(rank):
        h = torch.exp(A.unsqueeze(0) * dsum_all[k].unsqueeze(-1)) * h + h_end_all[k]
    return h


def exchange_boundaries(h_end, dsum, group=None):
    """Peer-to-peer exchange of the boundary values: this rank's (h_end, dsum) go to every
    later rank and the earlier ranks' come back.  Returns the lists (h_end, dsum) of
    ranks 0..rank (this rank's own last)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    pack = torch.cat([h_end.reshape(-1), dsum.reshape(-1).to(h_end.dtype)])
    recv = [torch.empty_like(pack) for _ in range(rank)]
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
    ops = [dist.P2POp(dist.isend, pack, ranks[d], group) for d in range(rank + 1, world)]
    ops += [dist.P2POp(dist.irecv, recv[s], ranks[s], group) for s in range(rank)]
    if ops:
        for r in dist.batch_isend_irecv(ops):
            r.wait()
    nh = h_end.numel()
    packs = recv + [pack]
    return ([q[:nh].view_as(h_end) for q in packs], [q[nh:].view_as(dsum) for q in packs])


def sequence_parallel_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=True,
                           group=None, out_dtype=torch.float32, local_scan=None, correct=None):
    """Forward selective scan of a sequence split across the ranks of `group`.

    Each rank passes its own chunk (b, L_rank, D) / (b, L_rank, N) of u, delta, z, B, C,
    in rank order along the sequence; A, D, delta_bias are replicated.  Returns this
    rank's (b, L_rank, D) output.  `local_scan` and `correct` replace the two kernel calls
    (the tests use them to drive the host logic on CPU ranks)."""
    scan = local_scan or _kernel_local_scan
    fix = correct or _kernel_correct
    out, h_end, dsum = scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, out_dtype)
    if dist.get_world_size(group) > 1:
        rank = dist.get_rank(group)
        h_ends, dsums = exchange_boundaries(h_end, dsum, group)
        if rank > 0:
            h_in = combine_prefix(h_ends, dsums, A, rank)
            out = fix(out, h_in, u, delta, A, B, C, z, delta_bias, delta_softplus)
    return out
