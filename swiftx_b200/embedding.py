"""Token embedding of the language model with a deterministic, sort-free backward.

The reference's LM embeds tokens with ``nn.Embedding`` (models/sift_model.py), whose CUDA
backward sorts the token ids and reduces segments (a radix sort plus several launches).
``embedding`` keeps torch's gather for the forward and computes the weight gradient
with ``swx_embedding_bwd``: per (32-column block, token slice) partial sums held in
shared memory, then a fixed-order sum over slices.  Supported: fp32 weight with at most
1024 rows on CUDA, int64 ids, no padding_idx / max_norm / sparse options.
"""
import torch
import torch.nn.functional as F

from . import _lib

MAX_VOCAB = 1024


def supported(idx, weight):
    return (idx.is_cuda and weight.is_cuda and idx.dtype == torch.int64 and weight.dtype == torch.float32
            and weight.dim() == 2 and 0 < weight.shape[0] <= MAX_VOCAB)


class EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, weight):
        if not supported(idx, weight):
            raise ValueError(f"embedding: CUDA int64 ids and an fp32 (vocab <= {MAX_VOCAB}, dim) weight "
                             f"expected, got {idx.dtype} ids and {weight.dtype} {tuple(weight.shape)}")
        ctx.save_for_backward(idx)
        ctx.vocab = weight.shape[0]
        return F.embedding(idx, weight)

    @staticmethod
    def backward(ctx, dy):
        (idx,) = ctx.saved_tensors
        d = dy.shape[-1]
        lib = _lib.load()
        ids = idx.contiguous().view(-1)
        dyf = dy.float().contiguous().view(-1, d)
        dw = torch.empty(ctx.vocab, d, device=dy.device, dtype=torch.float32)
        wsb = lib.swx_embedding_bwd_workspace_bytes(ids.numel(), ctx.vocab, d)
        ws = torch.empty(max(wsb, 1), device=dy.device, dtype=torch.uint8)
        a = _lib.EmbeddingArgs()
        a.ntok, a.vocab, a.dim = ids.numel(), ctx.vocab, d
        a.idx, a.dy, a.dweight = ids.data_ptr(), dyf.data_ptr(), dw.data_ptr()
        a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
        _lib.check(lib.swx_embedding_bwd(a, _lib.stream_ptr(dy.device)), "swx_embedding_bwd")
        return None, dw


def embedding(idx, weight):
    """``F.embedding(idx, weight)`` whose weight gradient runs on ``swx_embedding_bwd``."""
    return EmbeddingFn.apply(idx, weight)
