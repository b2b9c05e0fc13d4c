"""Embedding weight gradient (swx_embedding_bwd) against the exact (fp64) sums and
torch's fp32 embedding backward.

Each gradient entry is a sum of k fp32 terms (k = how often the id occurs).  Any
summation order in fp32 stays within (k - 1) * 2^-24 * sum|terms| of the exact sum, so
that is the tolerance against the fp64 sum, entry by entry.  torch's result (sorted
segments, another order) obeys the same bound; it is checked to it as well.
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from swiftx_b200 import _lib
from swiftx_b200.embedding import embedding

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _assert_within_summation_bound(got, idx, dy, vocab):
    ids, d = idx.reshape(-1), dy.shape[-1]
    dy64 = dy.reshape(-1, d).double()
    exact = torch.zeros(vocab, d, device=DEV, dtype=torch.float64).index_add_(0, ids, dy64)
    mag = torch.zeros(vocab, d, device=DEV, dtype=torch.float64).index_add_(0, ids, dy64.abs())
    k = torch.bincount(ids, minlength=vocab).double().unsqueeze(1)
    u = 2.0 ** -24
    bound = (k - 1).clamp(min=0) * u / (1 - k * u) * mag + 1e-30     # gamma_{k-1} * sum|x|
    err = (got.double() - exact).abs()
    assert bool((err <= bound).all()), f"max err / bound {float((err / bound).max()):.3g}"


def _torch_grad(idx, w, dy):
    w = w.detach().clone().requires_grad_()
    F.embedding(idx, w).backward(dy)
    return w.grad


@pytest.mark.parametrize("ntok,vocab,dim,dist", [
    (16 * 512, 256, 256, "uniform"),      # the LM's training step
    (1000, 65, 72, "uniform"),            # ragged: a partial column block and token batch
    (3000, 1024, 64, "uniform"),          # largest vocabulary held in shared memory
    (2048, 256, 32, "one"),               # every token the same id
    (5, 7, 3, "uniform"),                 # fewer tokens than one batch
])
def test_matches_torch(ntok, vocab, dim, dist):
    g = torch.Generator(device=DEV).manual_seed(ntok + vocab + dim)
    if dist == "one":
        idx = torch.full((ntok,), 3, device=DEV, dtype=torch.int64)
    else:
        idx = torch.randint(0, vocab, (ntok,), device=DEV, generator=g)
    w = torch.randn(vocab, dim, device=DEV, generator=g)
    dy = torch.randn(ntok, dim, device=DEV, generator=g)
    wt = w.clone().requires_grad_()
    embedding(idx, wt).backward(dy)
    _assert_within_summation_bound(wt.grad, idx, dy, vocab)
    _assert_within_summation_bound(_torch_grad(idx, w, dy), idx, dy, vocab)


def test_batched_ids_and_determinism():
    g = torch.Generator(device=DEV).manual_seed(1)
    idx = torch.randint(0, 256, (16, 512), device=DEV, generator=g)
    w = torch.randn(256, 256, device=DEV, generator=g)
    dy = torch.randn(16, 512, 256, device=DEV, generator=g)
    grads = []
    for _ in range(2):
        wt = w.clone().requires_grad_()
        embedding(idx, wt).backward(dy)
        grads.append(wt.grad)
    assert torch.equal(grads[0], grads[1])
    _assert_within_summation_bound(grads[0], idx, dy, 256)


def test_no_tokens_gives_zero_gradient():
    w = torch.randn(10, 8, device=DEV).requires_grad_()
    idx = torch.empty(0, device=DEV, dtype=torch.int64)
    embedding(idx, w).sum().backward()
    assert torch.count_nonzero(w.grad) == 0


def test_out_of_range_ids_are_flagged_and_skipped():
    # The kernel bounds-checks every id: an id outside [0, vocab) is skipped and sets
    # the status word; the in-range ids still sum as usual.
    lib = _lib.load()
    vocab, dim = 16, 40
    idx = torch.tensor([0, 5, vocab, 5, -1, 15], device=DEV, dtype=torch.int64)
    dy = torch.randn(idx.numel(), dim, device=DEV)
    dw = torch.full((vocab, dim), float("nan"), device=DEV)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    wsb = lib.swx_embedding_bwd_workspace_bytes(idx.numel(), vocab, dim)
    ws = torch.empty(wsb, device=DEV, dtype=torch.uint8)
    a = _lib.EmbeddingArgs()
    a.ntok, a.vocab, a.dim = idx.numel(), vocab, dim
    a.idx, a.dy, a.dweight, a.status = idx.data_ptr(), dy.data_ptr(), dw.data_ptr(), status.data_ptr()
    a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
    assert lib.swx_embedding_bwd(a, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    assert status.item() == 1
    ok = (idx >= 0) & (idx < vocab)
    _assert_within_summation_bound(dw, idx[ok], dy[ok], vocab)
    # a short workspace is refused on the host
    a.workspace_bytes = wsb - 4
    assert lib.swx_embedding_bwd(a, None) == _lib.SWX_ERR_INVALID_ARG
