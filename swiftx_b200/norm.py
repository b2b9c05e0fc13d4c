"""RMSNorm of the language model on one fused kernel each way.

The reference's RMSNorm (models/sift_model.py:17-26) is
``x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight``: six launches forward
and about ten backward.  ``rms_norm`` computes the same expression, in fp32 and in the
same order ((x * r) * w), with one launch forward and one (plus a fixed-order weight
gradient sum) backward.  x: (..., d) fp32 or bf16 with d <= 1024; weight (d,) fp32.
``add_rms_norm`` is the residual stream's form (models/sift_model.py:58,
x_{i+1} = x_i + mixer_i(norm_i(x_i)) followed by norm_{i+1}): the add folded into the next
norm's launch and, backward, the add's gradient sum and cast folded into the norm's.
"""
import torch

from . import _lib

MAX_DIM = 1024
_DT = {torch.float32: 0, torch.bfloat16: 1}


def supported(x):
    return x.is_cuda and x.dtype in _DT and 0 < x.shape[-1] <= MAX_DIM


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, out_dtype=None):
        if not supported(x):
            raise ValueError(f"rms_norm: CUDA fp32/bf16 input with last dim <= {MAX_DIM} expected, "
                             f"got {x.device} {x.dtype} {tuple(x.shape)}")
        d = x.shape[-1]
        xf = x.contiguous().view(-1, d)
        w = weight.detach().float().contiguous()
        if w.numel() != d:
            raise ValueError(f"rms_norm: weight has {w.numel()} values, x has {d} channels")
        out_dtype = out_dtype or x.dtype
        if out_dtype not in _DT:
            raise ValueError(f"rms_norm: output dtype {out_dtype} not supported")
        y = torch.empty(xf.shape, device=x.device, dtype=out_dtype)
        rstd = torch.empty(xf.shape[0], device=x.device, dtype=torch.float32)
        a = _lib.RMSNormArgs()
        a.rows, a.dim, a.eps, a.dtype, a.out_dtype = xf.shape[0], d, float(eps), _DT[x.dtype], _DT[out_dtype]
        a.x, a.weight, a.y, a.rstd = xf.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr()
        _lib.check(_lib.load().swx_rmsnorm_fwd(a, _lib.stream_ptr(x.device)), "swx_rmsnorm_fwd")
        ctx.save_for_backward(xf, w, rstd)
        ctx.shape, ctx.wdtype, ctx.out_dtype = x.shape, weight.dtype, out_dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        xf, w, rstd = ctx.saved_tensors
        d = xf.shape[-1]
        lib = _lib.load()
        dyf = dy.to(ctx.out_dtype).contiguous().view(-1, d)
        dx = torch.empty_like(xf)
        dw = torch.empty(d, device=xf.device, dtype=torch.float32)
        wsb = lib.swx_rmsnorm_bwd_workspace_bytes(d)
        ws = torch.empty(wsb, device=xf.device, dtype=torch.uint8)
        a = _lib.RMSNormArgs()
        a.rows, a.dim, a.dtype, a.out_dtype = xf.shape[0], d, _DT[xf.dtype], _DT[ctx.out_dtype]
        a.x, a.weight, a.rstd = xf.data_ptr(), w.data_ptr(), rstd.data_ptr()
        a.dy, a.dx, a.dweight = dyf.data_ptr(), dx.data_ptr(), dw.data_ptr()
        a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
        _lib.check(lib.swx_rmsnorm_bwd(a, _lib.stream_ptr(xf.device)), "swx_rmsnorm_bwd")
        return dx.view(ctx.shape), dw.to(ctx.wdtype), None, None


def rms_norm(x, weight, eps=1e-5, out_dtype=None):
    """(x * rsqrt(mean(x^2, -1) + eps)) * weight on the fused kernels (CUDA only), computed
    in fp32.  out_dtype (fp32 or bf16; default x's dtype) is the dtype of the result: a
    bf16 result is the fp32 one rounded once, what a cast right after the norm gives."""
    return RMSNormFn.apply(x, weight, eps, out_dtype)


class AddRMSNormFn(torch.autograd.Function):
    """(s, y) = (x + res, rms_norm(x + res)) with the add folded into the norm's launches.

    Backward: ds (the sum's gradient from its other consumers, possibly None) and dy (the
    norm's) give dx = ds + norm-backward(dy), returned for x and, cast to res's dtype,
    for res -- the add's backward and the cast inside the norm's backward launch."""

    @staticmethod
    def forward(ctx, x, res, weight, eps, out_dtype=None):
        if not supported(x) or res.shape != x.shape or res.dtype not in _DT or not res.is_cuda:
            raise ValueError(f"add_rms_norm: CUDA fp32/bf16 x and a residual of its shape expected, got "
                             f"{x.dtype} {tuple(x.shape)} and {res.dtype} {tuple(res.shape)}")
        d = x.shape[-1]
        xf = x.contiguous().view(-1, d)
        rf = res.contiguous().view(-1, d)
        w = weight.detach().float().contiguous()
        if w.numel() != d:
            raise ValueError(f"rms_norm: weight has {w.numel()} values, x has {d} channels")
        out_dtype = out_dtype or x.dtype
        if out_dtype not in _DT:
            raise ValueError(f"add_rms_norm: output dtype {out_dtype} not supported")
        s = torch.empty_like(xf)
        y = torch.empty(xf.shape, device=x.device, dtype=out_dtype)
        rstd = torch.empty(xf.shape[0], device=x.device, dtype=torch.float32)
        a = _lib.RMSNormArgs()
        a.rows, a.dim, a.eps, a.dtype, a.out_dtype = xf.shape[0], d, float(eps), _DT[x.dtype], _DT[out_dtype]
        a.res_dtype = _DT[res.dtype]
        a.x, a.weight, a.y, a.rstd = xf.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr()
        a.residual, a.sum = rf.data_ptr(), s.data_ptr()
        _lib.check(_lib.load().swx_rmsnorm_fwd(a, _lib.stream_ptr(x.device)), "swx_rmsnorm_fwd")
        ctx.save_for_backward(s, w, rstd)
        ctx.shape, ctx.wdtype, ctx.out_dtype, ctx.res_dtype = x.shape, weight.dtype, out_dtype, res.dtype
        return s.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, ds, dy):
        s, w, rstd = ctx.saved_tensors
        d = s.shape[-1]
        lib = _lib.load()
        if dy is None:
            dy = torch.zeros(s.shape, device=s.device, dtype=ctx.out_dtype)
        dyf = dy.to(ctx.out_dtype).contiguous().view(-1, d)
        dsf = ds.float().contiguous().view(-1, d) if ds is not None else None
        dx = torch.empty_like(s)
        own = ctx.res_dtype != s.dtype          # the residual's gradient needs its own copy
        dres = torch.empty(s.shape, device=s.device, dtype=ctx.res_dtype) if own else dx
        dw = torch.empty(d, device=s.device, dtype=torch.float32)
        wsb = lib.swx_rmsnorm_bwd_workspace_bytes(d)
        ws = torch.empty(wsb, device=s.device, dtype=torch.uint8)
        a = _lib.RMSNormArgs()
        a.rows, a.dim, a.dtype, a.out_dtype = s.shape[0], d, _DT[s.dtype], _DT[ctx.out_dtype]
        a.res_dtype = _DT[ctx.res_dtype]
        a.x, a.weight, a.rstd = s.data_ptr(), w.data_ptr(), rstd.data_ptr()
        a.dy, a.dx, a.dweight = dyf.data_ptr(), dx.data_ptr(), dw.data_ptr()
        a.dsum = dsf.data_ptr() if dsf is not None else None
        a.dres = dres.data_ptr() if own else None
        a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
        _lib.check(lib.swx_rmsnorm_bwd(a, _lib.stream_ptr(s.device)), "swx_rmsnorm_bwd")
        return dx.view(ctx.shape), dres.view(ctx.shape), dw.to(ctx.wdtype), None, None


def add_rms_norm(x, res, weight, eps=1e-5, out_dtype=None):
    """(x + res, rms_norm(x + res, weight)) on the fused kernels (CUDA only): the residual
    stream's add and the next norm in one launch each way.  The sum is in x's dtype
    (computed in fp32); res may be fp32 or bf16."""
    return AddRMSNormFn.apply(x, res, weight, eps, out_dtype)
