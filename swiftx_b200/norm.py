"""RMSNorm of the language model on one fused kernel each way.

The reference's RMSNorm (models/sift_model.py:17-26) is
``x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight``: six launches forward
and about ten backward.  ``rms_norm`` computes the same expression, in fp32 and in the
same order ((x * r) * w), with one launch forward and one (plus a fixed-order weight
gradient sum) backward.  x: (..., d) fp32 or bf16 with d <= 1024; weight (d,) fp32.
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
