"""Causal depthwise conv1d + SiLU on B200 (the conv segment of the Sift block).

Replaces ``F.silu(self.conv1d(x.transpose(1, 2))[..., :L].transpose(1, 2))`` in
SiftBlock.forward (models/sift_block.py:62-65, 117-118) with one fused kernel that reads
x in the (b, L, D) layout directly -- including the strided x half of the in_proj
output -- and writes a dense (b, L, D) activation.  Backward recomputes the
pre-activation; dweight / dbias are deterministic.
"""
import torch

from . import _lib


def _dtype_code(t):
    if t.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"conv1d: unsupported dtype {t.dtype}")
    return _lib.DTYPE_CODES[t.dtype]


def _fill(a, x, weight, bias, silu):
    b, L, D = x.shape
    a.batch, a.seqlen, a.dim, a.width = b, L, D, weight.shape[-1]
    a.dtype = _dtype_code(x)
    a.silu = 1 if silu else 0
    a.x, a.x_sb, a.x_sl = x.data_ptr(), x.stride(0), x.stride(1)
    a.weight = weight.data_ptr()
    a.bias = bias.data_ptr() if bias is not None else None


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("swiftx_b200 conv1d runs on CUDA tensors only (no CPU path)")


def _prep(x, weight, bias):
    _require_cuda(x, weight)
    if x.dim() != 3:
        raise ValueError("expected x of shape (b, L, D)")
    if x.dtype == torch.float64:
        raise ValueError("conv1d: the kernels take float32 or bfloat16 x (no float64 form)")
    if x.dtype not in _lib.DTYPE_CODES:
        x = x.float()
    if x.stride(-1) != 1:
        x = x.contiguous()
    w = weight.detach().reshape(weight.shape[0], -1).float().contiguous()
    bb = bias.detach().float().contiguous() if bias is not None else None
    if w.shape[0] != x.shape[-1]:
        raise ValueError(f"weight has {w.shape[0]} channels, x has {x.shape[-1]}")
    if bb is not None and bb.numel() != x.shape[-1]:
        raise ValueError(f"bias has {bb.numel()} values, x has {x.shape[-1]} channels")
    return x, w, bb


def conv1d_forward(x, weight, bias=None, silu=True):
    lib = _lib.load()
    x, w, bb = _prep(x, weight, bias)
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    a = _lib.ConvArgs()
    _fill(a, x, w, bb, silu)
    a.out = out.data_ptr()
    _lib.check(lib.swx_conv1d_fwd(a, _lib.stream_ptr(x.device)), "swx_conv1d_fwd")
    return out


def conv1d_backward(x, weight, bias, dout, silu=True, dx_out=None):
    """dx, dweight, dbias of conv1d_forward.  dx_out: optional (b, L, D) tensor with unit
    channel stride (e.g. the x half of a (b, L, 2D) gradient) that receives dx in place of
    a new tensor; its dtype is x's for fp32 / bf16 x, fp32 for x of another dtype (which
    the kernels compute in fp32)."""
    lib = _lib.load()
    x, w, bb = _prep(x, weight, bias)
    if dout.shape != x.shape:
        raise ValueError(f"dout: expected shape {tuple(x.shape)}, got {tuple(dout.shape)}")
    dout = dout.to(x.dtype)
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    b, L, D = x.shape
    K = w.shape[1]
    if dx_out is not None:
        if dx_out.shape != x.shape or dx_out.dtype != x.dtype or dx_out.stride(-1) != 1 or dx_out.device != x.device:
            raise ValueError("dx_out must be a (b, L, D) tensor of x's dtype with unit channel stride")
        dx = dx_out
    else:
        dx = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    dw = torch.empty((D, K), device=x.device, dtype=torch.float32)
    db = torch.empty(D, device=x.device, dtype=torch.float32) if bias is not None else None
    wsb = lib.swx_conv1d_bwd_workspace_bytes(b, L, D, K)
    ws = torch.empty(max(wsb, 1), device=x.device, dtype=torch.uint8)
    a = _lib.ConvArgs()
    _fill(a, x, w, bb, silu)
    a.dout, a.dout_sb, a.dout_sl = dout.data_ptr(), dout.stride(0), dout.stride(1)
    a.dx, a.dweight = dx.data_ptr(), dw.data_ptr()
    a.dbias = db.data_ptr() if db is not None else None
    a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
    if dx_out is not None:
        a.dx_sb, a.dx_sl = dx.stride(0), dx.stride(1)
    _lib.check(lib.swx_conv1d_bwd(a, _lib.stream_ptr(x.device)), "swx_conv1d_bwd")
    return dx, dw, db


class CausalConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, silu):
        ctx.save_for_backward(x, weight, bias)
        ctx.silu = silu
        return conv1d_forward(x, weight, bias, silu)

    @staticmethod
    def backward(ctx, dout):
        x, weight, bias = ctx.saved_tensors
        dx, dw, db = conv1d_backward(x, weight, bias, dout, ctx.silu)
        dw = dw.reshape(weight.shape).to(weight.dtype)
        db = db.to(bias.dtype) if db is not None else None
        return dx.to(x.dtype), dw, db, None


def causal_conv1d_fn(x, weight, bias=None, activation="silu"):
    """x: (b, L, D) (any row strides, unit channel stride); weight (D, 1, K) or (D, K);
    bias (D,).  Returns silu(causal_conv(x) + bias) of shape (b, L, D)."""
    if activation not in (None, "silu"):
        raise ValueError(f"unsupported activation {activation!r}")
    return CausalConv1dFn.apply(x, weight, bias, activation == "silu")
