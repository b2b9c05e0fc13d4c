"""Selective scan on B200: the reference's Python entry points over the CUDA kernels.

Mirrors models/selective_scan.py of the reference:

* ``selective_scan_fast(u, delta, A, B, C, D=None, mode="auto", chunk=16)``
  (models/selective_scan.py:246-265) -- every mode runs the sm_100a kernel;
* ``selective_scan_ref(u, delta, A, B, C, D=None)`` (:34-60) -- same kernel;
* ``selective_scan_fn(...)`` -- the extended entry point with the SiLU(z) gate and
  softplus(delta + delta_bias) folded in (the block glue of models/sift_block.py:108,134);
* ``parallel_scan(a, x)`` / ``sequential_scan(a, x)`` (:66-99) -- the plain linear
  recurrence h_t = a_t h_{t-1} + x_t along dim 1, on its own kernel.

Shapes: u, delta, z (b, L, D); A (D, N); B, C (b, L, N); D, delta_bias (D,).
Autograd follows the reference's custom Functions: the forward saves only its inputs
plus state checkpoints every 16 steps, the backward recomputes
(models/selective_scan.py:124, models/triton_scan.py:133), and gradients come back
in the input dtype with dA / dD in fp32 (models/triton_scan.py:153-155).  float64
inputs are computed in float64 and return float64 (as the reference's scan keeps the
input dtype, models/selective_scan.py:52), so its float64 gradchecks hold.

There is no CPU path: CPU tensors raise.  The kernel library must be built.
"""
import torch

from . import _lib

_FLOAT_IN = (torch.float32, torch.bfloat16, torch.float64)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("swiftx_b200 selective scan runs on CUDA tensors only "
                               "(no CPU path); move the inputs to the GPU")


def _rows(t):
    """(b, L, W) tensor with unit innermost stride (copies only if that is not so)."""
    return t if t.stride(-1) == 1 else t.contiguous()


def _in_dtype(*ts):
    dt = ts[0].dtype
    return dt if dt in _FLOAT_IN else torch.float32


def _param_dtype(in_dt):
    """dtype of A, D, delta_bias, h0 and their gradients: float64 with float64 inputs
    (computed in float64 throughout), else fp32."""
    return torch.float64 if in_dt == torch.float64 else torch.float32


def _fill_inputs(a, u, delta, A, B, C, D, z, delta_bias, h0, softplus, in_dt, A_is_log=False):
    b, L, Dm = u.shape
    a.batch, a.seqlen, a.dim, a.dstate = b, L, Dm, A.shape[1]
    a.in_dtype = _lib.DTYPE_CODES[in_dt]
    a.delta_softplus = 1 if softplus else 0
    a.flags = _lib.SWX_SCAN_A_LOG if A_is_log else 0
    a.u, a.u_sb, a.u_sl = u.data_ptr(), u.stride(0), u.stride(1)
    a.delta, a.delta_sb, a.delta_sl = delta.data_ptr(), delta.stride(0), delta.stride(1)
    if z is not None:
        a.z, a.z_sb, a.z_sl = z.data_ptr(), z.stride(0), z.stride(1)
    a.B, a.B_sb, a.B_sl = B.data_ptr(), B.stride(0), B.stride(1)
    a.C, a.C_sb, a.C_sl = C.data_ptr(), C.stride(0), C.stride(1)
    a.A = A.data_ptr()
    a.Dskip = D.data_ptr() if D is not None else None
    a.delta_bias = delta_bias.data_ptr() if delta_bias is not None else None
    a.h0 = h0.data_ptr() if h0 is not None else None


def _prep_groups(group_w, group_of, u, z):
    """The SiftX pathway mix fused into the gate: group_w (b, L, G) per-token group weights
    (fp32, made contiguous) and group_of (D,) channel -> group (int32, values in [0, G):
    the kernels index group_w with them unchecked, and checking device values here would
    cost a synchronisation per call).  Returns the pair as the kernels take it, or
    (None, None)."""
    if group_w is None:
        return None, None
    if z is None:
        raise ValueError("group_w (the pathway mix) needs the gate z")
    b, L, Dm = u.shape
    if group_of is None or group_w.dim() != 3 or group_w.shape[:2] != (b, L) or group_of.shape != (Dm,):
        raise ValueError("expected group_w (b, L, G) and group_of (D,)")
    if not 1 <= group_w.shape[2] <= _lib.SWX_MAX_GROUPS:
        raise ValueError(f"at most {_lib.SWX_MAX_GROUPS} pathway groups are supported")
    _require_cuda(group_w, group_of)
    return group_w.detach().float().contiguous(), group_of.to(torch.int32).contiguous()


def _fill_groups(a, gw, gof):
    if gw is not None:
        a.group_w, a.group_w_sb, a.group_w_sl = gw.data_ptr(), gw.stride(0), gw.stride(1)
        a.group_of, a.ngroups = gof.data_ptr(), gw.shape[2]


def _prep(u, delta, A, B, C, D, z, delta_bias, h0):
    _require_cuda(u, delta, A, B, C, D, z, delta_bias, h0)
    in_dt = _in_dtype(u)
    cast = lambda t: None if t is None else _rows(t.to(in_dt))  # noqa: E731
    u, delta, B, C, z = cast(u), cast(delta), cast(B), cast(C), cast(z)
    pdt = _param_dtype(in_dt)
    par = lambda t: None if t is None else t.detach().to(pdt).contiguous()  # noqa: E731
    A, D, delta_bias, h0 = par(A), par(D), par(delta_bias), par(h0)
    if u.dim() != 3 or delta.shape != u.shape or B.dim() != 3 or C.shape != B.shape:
        raise ValueError("expected u, delta (b, L, D) and B, C (b, L, N)")
    b, L, Dm = u.shape
    N = A.shape[1]
    if A.shape != (Dm, N) or B.shape != (b, L, N) or (z is not None and z.shape != u.shape):
        raise ValueError(f"shape mismatch: u {tuple(u.shape)}, A {tuple(A.shape)}, B {tuple(B.shape)}")
    if N > 16:
        raise ValueError(f"d_state {N} > 16 is not supported")
    for name, t in (("D", D), ("delta_bias", delta_bias)):
        if t is not None and t.numel() != Dm:
            raise ValueError(f"{name}: expected {Dm} values, got {t.numel()}")
    if h0 is not None and h0.shape != (b, Dm, N):
        raise ValueError(f"h0: expected shape {(b, Dm, N)}, got {tuple(h0.shape)}")
    return u, delta, A, B, C, D, z, delta_bias, h0, in_dt


def scan_forward(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                 h0=None, out_dtype=None, checkpoints=False, return_last_state=False,
                 return_delta_sum=False, write_out=True, pre_out=None, A_is_log=False,
                 group_w=None, group_of=None, split=True):
    """One kernel launch of the forward scan (no autograd).

    Returns (out, checkpoints or None, last_state or None), plus delta_sum (b, D) -- the
    sum over t of delta_eff -- when return_delta_sum.  write_out=False skips the output
    (out is None), for callers that only need the final state / delta_sum.  pre_out, a
    dense fp32 (b, L, D) tensor, receives the pre-gate output when z is given (the
    backward can then skip recomputing it).  A_is_log: A holds log(-A) (see
    selective_scan_fn).  group_w, group_of: the SiftX pathway mix fused into the gate
    (see selective_scan_fn).  split: let the library cut long sequences of a small batch
    into segments scanned in parallel (SWX_SCAN_SPLIT_FWD; same results to fp32 rounding)."""
    lib = _lib.load()
    u, delta, A, B, C, D, z, delta_bias, h0, in_dt = _prep(u, delta, A, B, C, D, z, delta_bias, h0)
    gw, gof = _prep_groups(group_w, group_of, u, z)
    b, L, Dm = u.shape
    N = A.shape[1]
    pdt = _param_dtype(in_dt)
    out_dt = torch.float64 if in_dt == torch.float64 else (out_dtype or in_dt)
    out = torch.empty((b, L, Dm), device=u.device, dtype=out_dt) if write_out else None
    ck = (torch.empty(lib.swx_scan_checkpoint_floats(b, L, Dm), device=u.device, dtype=pdt)
          if checkpoints else None)
    hl = torch.empty((b, Dm, N), device=u.device, dtype=pdt) if return_last_state else None
    ds = torch.empty((b, Dm), device=u.device, dtype=pdt) if return_delta_sum else None
    a = _lib.ScanArgs()
    _fill_inputs(a, u, delta, A, B, C, D, z, delta_bias, h0, delta_softplus, in_dt, A_is_log)
    a.out_dtype = _lib.DTYPE_CODES[out_dt]
    a.out = out.data_ptr() if out is not None else None
    a.h_last = hl.data_ptr() if hl is not None else None
    a.checkpoints = ck.data_ptr() if ck is not None else None
    a.delta_sum = ds.data_ptr() if ds is not None else None
    if pre_out is not None and z is not None:
        if pre_out.dtype != pdt or not pre_out.is_contiguous() or pre_out.shape != (b, L, Dm) \
                or pre_out.device != u.device:
            raise ValueError(f"pre_out must be a dense {pdt} (b, L, D) tensor on {u.device}")
        a.out_pre = pre_out.data_ptr()
    _fill_groups(a, gw, gof)
    ws = None
    if split:
        a.flags |= _lib.SWX_SCAN_SPLIT_FWD
        wsb = lib.swx_scan_fwd_workspace_bytes(a)
        if wsb > 0:
            ws = torch.empty(wsb, device=u.device, dtype=torch.uint8)
            a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
    _lib.check(lib.swx_scan_fwd(a, _lib.stream_ptr(u.device)), "swx_scan_fwd")
    if return_delta_sum:
        return out, ck, hl, ds
    return out, ck, hl


def scan_backward(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0, ck, dout, y_pre=None,
                  A_is_log=False, group_w=None, group_of=None, group_w_grad=False, dz_out=None):
    """One call of the backward kernels (no autograd).  Returns a dict of gradients.
    y_pre: the pre-gate output the forward wrote to pre_out (optional, with z).
    dz_out: optional (b, L, D) tensor of the input dtype with unit channel stride (e.g. the
    z half of a (b, L, 2D) gradient) that receives dz in place of a new tensor.
    A_is_log: A holds log(-A), and "dA" is the gradient with respect to it.
    group_w, group_of: the pathway mix of the forward; with group_w_grad (needs y_pre)
    "d_group_w" (b, L, G) is the gradient with respect to group_w."""
    lib = _lib.load()
    u, delta, A, B, C, D, z, delta_bias, h0, in_dt = _prep(u, delta, A, B, C, D, z, delta_bias, h0)
    gw, gof = _prep_groups(group_w, group_of, u, z)
    b, L, Dm = u.shape
    N = A.shape[1]
    if dout.shape != (b, L, Dm):
        raise ValueError(f"dout: expected shape {(b, L, Dm)}, got {tuple(dout.shape)}")
    dout = _rows(dout.to(in_dt))
    dev = u.device
    pdt = _param_dtype(in_dt)
    # the kernels read these two through bare pointers: check what they will index
    need = lib.swx_scan_checkpoint_floats(b, L, Dm)
    if ck is None or ck.dtype != pdt or ck.device != dev or not ck.is_contiguous() or ck.numel() < need:
        raise ValueError(f"ck must be the forward's checkpoints: a contiguous {pdt} tensor of at least "
                         f"{need} values on {dev}")
    if y_pre is not None and z is not None and (y_pre.dtype != pdt or not y_pre.is_contiguous()
                                                or y_pre.shape != (b, L, Dm) or y_pre.device != dev):
        raise ValueError(f"y_pre must be the forward's pre_out: a dense {pdt} (b, L, D) tensor on {dev}")
    e = lambda *s, dt=in_dt: torch.empty(s, device=dev, dtype=dt)  # noqa: E731
    g = {"du": e(b, L, Dm), "ddelta": e(b, L, Dm), "dB": e(b, L, N), "dC": e(b, L, N),
         "dA": e(Dm, N, dt=pdt)}
    if dz_out is not None:
        if z is None or dz_out.shape != (b, L, Dm) or dz_out.dtype != in_dt or dz_out.stride(-1) != 1 \
                or dz_out.device != dev:
            raise ValueError("dz_out must be a (b, L, D) tensor of the input dtype with unit channel stride")
        g["dz"] = dz_out
    else:
        g["dz"] = e(b, L, Dm) if z is not None else None
    g["dD"] = e(Dm, dt=pdt) if D is not None else None
    g["ddelta_bias"] = e(Dm, dt=pdt) if delta_bias is not None else None
    g["dh0"] = e(b, Dm, N, dt=pdt) if h0 is not None else None
    wsb = (lib.swx_scan_bwd_workspace_bytes_f64 if in_dt == torch.float64
           else lib.swx_scan_bwd_workspace_bytes)(b, L, Dm)
    ws = torch.empty(max(wsb, 1), device=dev, dtype=torch.uint8)
    a = _lib.ScanArgs()
    _fill_inputs(a, u, delta, A, B, C, D, z, delta_bias, h0, delta_softplus, in_dt, A_is_log)
    a.out_dtype = a.in_dtype
    a.checkpoints = ck.data_ptr()
    a.dout, a.dout_sb, a.dout_sl = dout.data_ptr(), dout.stride(0), dout.stride(1)
    for k in ("du", "ddelta", "dz", "dB", "dC", "dA", "dD", "ddelta_bias", "dh0"):
        setattr(a, k, g[k].data_ptr() if g[k] is not None else None)
    a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
    if dz_out is not None:
        a.dz_sb, a.dz_sl = dz_out.stride(0), dz_out.stride(1)
    if y_pre is not None and z is not None:
        a.out_pre = y_pre.data_ptr()
    _fill_groups(a, gw, gof)
    g["d_group_w"] = None
    if gw is not None and group_w_grad:
        if y_pre is None:
            raise ValueError("the gradient of group_w needs the pre-gate output y_pre")
        g["d_group_w"] = torch.empty(gw.shape, device=dev, dtype=torch.float32)
        a.d_group_w = g["d_group_w"].data_ptr()
    _lib.check(lib.swx_scan_bwd(a, _lib.stream_ptr(dev)), "swx_scan_bwd")
    return g


def scan_correct(out, h_in, u, delta, A, B, C, z=None, delta_bias=None, delta_softplus=False,
                 A_is_log=False):
    """In place: turn ``out``, the forward of a chunk scanned from a zero state, into the
    forward of the same chunk scanned from ``h_in`` (b, D, N):
    out_t += silu(z_t) * sum_n C_t[n] exp(A[:, n] S_t) h_in[n], S_t the running sum of
    delta_eff (swx_scan_correct).  u and B are only shape-checked.  Returns out."""
    lib = _lib.load()
    u, delta, A, B, C, _, z, delta_bias, h_in, in_dt = _prep(u, delta, A, B, C, None, z, delta_bias, h_in)
    if in_dt == torch.float64:
        raise ValueError("scan_correct: float64 is not supported")
    b, L, Dm = u.shape
    if out.shape != (b, L, Dm) or not out.is_contiguous() or out.dtype not in _lib.DTYPE_CODES:
        raise ValueError("out must be a dense (b, L, D) fp32 or bf16 tensor")
    wsb = lib.swx_scan_correct_workspace_bytes(b, L, Dm)
    ws = torch.empty(max(wsb, 1), device=u.device, dtype=torch.uint8)
    a = _lib.ScanArgs()
    _fill_inputs(a, u, delta, A, B, C, None, z, delta_bias, h_in, delta_softplus, in_dt, A_is_log)
    a.out_dtype = _lib.DTYPE_CODES[out.dtype]
    a.out = out.data_ptr()
    a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
    _lib.check(lib.swx_scan_correct(a, _lib.stream_ptr(u.device)), "swx_scan_correct")
    return out


class SelectiveScanFn(torch.autograd.Function):
    """Custom autograd Function over the fused kernels (same save/recompute trade as
    _FusedScanFn / TritonScanFn in the reference)."""

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0, out_dtype,
                return_last_state, A_is_log, group_w=None, group_of=None):
        need_grad = any(ctx.needs_input_grad[i] for i in (0, 1, 2, 3, 4, 5, 6, 7, 9, 13))
        pre = (torch.empty(u.shape, device=u.device, dtype=_param_dtype(_in_dtype(u)))
               if need_grad and z is not None else None)
        out, ck, hl = scan_forward(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0,
                                   out_dtype, checkpoints=need_grad,
                                   return_last_state=return_last_state, pre_out=pre, A_is_log=A_is_log,
                                   group_w=group_w, group_of=group_of)
        ctx.delta_softplus = delta_softplus
        ctx.A_is_log = A_is_log
        ctx.dtypes = [t.dtype if t is not None else None
                      for t in (u, delta, A, B, C, D, z, delta_bias, h0, group_w)]
        if need_grad:
            ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, h0, ck, pre, group_w, group_of)
        if return_last_state:
            ctx.mark_non_differentiable(hl)
            return out, hl
        return out

    @staticmethod
    def backward(ctx, dout, *unused):
        u, delta, A, B, C, D, z, delta_bias, h0, ck, pre, group_w, group_of = ctx.saved_tensors
        g = scan_backward(u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus, h0, ck, dout, y_pre=pre,
                          A_is_log=ctx.A_is_log, group_w=group_w, group_of=group_of,
                          group_w_grad=group_w is not None and ctx.needs_input_grad[13])
        dts = ctx.dtypes
        cast = lambda t, dt: None if t is None or dt is None else t.to(dt)  # noqa: E731
        return (cast(g["du"], dts[0]), cast(g["ddelta"], dts[1]), cast(g["dA"], dts[2]),
                cast(g["dB"], dts[3]), cast(g["dC"], dts[4]), cast(g["dD"], dts[5]),
                cast(g["dz"], dts[6]), cast(g["ddelta_bias"], dts[7]), None,
                cast(g["dh0"], dts[8]), None, None, None, cast(g["d_group_w"], dts[9]), None)


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                      h0=None, out_dtype=None, return_last_state=False, A_is_log=False,
                      group_w=None, group_of=None):
    """Fused selective scan with optional SiLU(z) gate and softplus(delta + delta_bias).

    out = (scan(u, delta_eff, A, B, C) + D*u) * silu(z),  delta_eff = softplus(delta + delta_bias).
    Returns out (and the final state (b, D, N) when return_last_state).

    A_is_log=True: the tensor passed as A holds log(-A) -- the block's A_log parameter --
    and the kernels form A = -exp(A_log) themselves (models/sift_block.py:121 does it in
    two elementwise ops before each call, plus two more in the backward); its gradient
    is returned with respect to A_log.

    group_w (b, L, G), group_of (D,): the SiftX pathway mix (models/sift_block.py:137-142)
    fused into the gate, out = y * group_w[..., group_of] * silu(z) with y the D-skipped
    scan output; group_w receives its gradient (fp32 or bf16 inputs, G <= 8, with z)."""
    return SelectiveScanFn.apply(u, delta, A, B, C, D, z, delta_bias, bool(delta_softplus), h0,
                                 out_dtype, bool(return_last_state), bool(A_is_log), group_w, group_of)


_MODES = ("auto", "parallel", "sequential", "fused", "triton")


def selective_scan_fast(u, delta, A, B, C, D=None, mode="auto", chunk=16):
    """Drop-in for the reference dispatcher (models/selective_scan.py:246-265).

    Every mode computes the same function; on B200 they all run the fused sm_100a
    kernel (the checkpoint interval is fixed at 16 steps, so ``chunk`` has no effect)."""
    if mode not in _MODES:
        raise ValueError(f"unknown mode {mode!r}; expected one of {_MODES}")
    return selective_scan_fn(u, delta, A, B, C, D)


def selective_scan_ref(u, delta, A, B, C, D=None):
    """Reference-named entry (models/selective_scan.py:34): the exact sequential
    recurrence, computed by the same CUDA kernel."""
    return selective_scan_fn(u, delta, A, B, C, D)


# ----------------------------------------------------------------- linear recurrence
_LS_DTYPES = {torch.float32: 0, torch.float64: _lib.SWX_DTYPE_F64}


def _flat3(t):
    """(b, L, ...) -> (b, L, W) view with unit element stride (copies only if needed)."""
    b, L = t.shape[:2]
    v = t.reshape(b, L, -1)
    return v if v.stride(-1) == 1 else v.contiguous()


def _ls_dtype(a, x):
    dt = torch.promote_types(a.dtype, x.dtype)
    return dt if dt in _LS_DTYPES else torch.float32


class LinearScanFn(torch.autograd.Function):
    """h_t = a_t * h_{t-1} + x_t along dim 1 on the sm_100a kernel, with its adjoint as the
    backward (g_t = dh_t + a_{t+1} g_{t+1}; dx = g, da_t = g_t h_{t-1})."""

    @staticmethod
    def forward(ctx, a, x):
        _require_cuda(a, x)
        if a.dim() < 2 or a.shape != x.shape:
            raise ValueError(f"expected a and x of the same shape (b, L, ...), got {tuple(a.shape)} "
                             f"and {tuple(x.shape)}")
        dt = _ls_dtype(a, x)
        af, xf = _flat3(a.detach().to(dt)), _flat3(x.detach().to(dt))
        b, L, W = af.shape
        h = torch.empty((b, L, W), device=a.device, dtype=dt)
        s = _lib.LinearScanArgs()
        s.batch, s.seqlen, s.width, s.dtype = b, L, W, _LS_DTYPES[dt]
        s.a, s.a_sb, s.a_sl = af.data_ptr(), af.stride(0), af.stride(1)
        s.x, s.x_sb, s.x_sl = xf.data_ptr(), xf.stride(0), xf.stride(1)
        s.h = h.data_ptr()
        _lib.check(_lib.load().swx_linear_scan_fwd(s, _lib.stream_ptr(a.device)), "swx_linear_scan_fwd")
        ctx.save_for_backward(af, h)
        ctx.shape, ctx.dtypes = a.shape, (a.dtype, x.dtype)
        return h.view(a.shape).to(x.dtype)

    @staticmethod
    def backward(ctx, dh):
        af, h = ctx.saved_tensors
        b, L, W = h.shape
        dhf = _flat3(dh.to(h.dtype))
        da, dx = torch.empty_like(h), torch.empty_like(h)
        s = _lib.LinearScanArgs()
        s.batch, s.seqlen, s.width, s.dtype = b, L, W, _LS_DTYPES[h.dtype]
        s.a, s.a_sb, s.a_sl = af.data_ptr(), af.stride(0), af.stride(1)
        s.h = h.data_ptr()
        s.dh, s.dh_sb, s.dh_sl = dhf.data_ptr(), dhf.stride(0), dhf.stride(1)
        s.da, s.dx = da.data_ptr(), dx.data_ptr()
        _lib.check(_lib.load().swx_linear_scan_bwd(s, _lib.stream_ptr(h.device)), "swx_linear_scan_bwd")
        return da.view(ctx.shape).to(ctx.dtypes[0]), dx.view(ctx.shape).to(ctx.dtypes[1])


def parallel_scan(a, x):
    """Solve h_t = a_t * h_{t-1} + x_t (h before the first step = 0) along dim 1.

    Drop-in for models/selective_scan.py:66-88: a, x of shape (b, L, ...) -> h like x.
    The reference composes affine maps with a Hillis-Steele scan (log2 L rounds over the
    whole tensor); on B200 the recurrence is one HBM stream (read a, x; write h) with a
    thread per (row, element) chain, so the result matches sequential_scan to rounding.
    Differentiable (the reference's version is not: its in-place updates break autograd).
    fp32 and fp64 compute natively; other float dtypes compute in fp32."""
    return LinearScanFn.apply(a, x)


def sequential_scan(a, x):
    """Same recurrence as parallel_scan (models/selective_scan.py:91-99), same kernel."""
    return LinearScanFn.apply(a, x)
