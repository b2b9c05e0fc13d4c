"""Recurrent decode step on B200 (SiftBlock.step, models/sift_block.py:153-175).

``decode_conv_step``  -- roll the conv window, append x, xc = silu(conv + bias) (in place);
``decode_ssm_step``   -- h = exp(delta*A)*h + delta*B*xc; out = (<h,C> + D*xc)*silu(z) (in place);
``decode_step``       -- both in one launch when delta/B/C are already known.
All tensors fp32 on CUDA; row strides may differ from dense (e.g. the x/z halves of
the in_proj output), the channel / state stride must be 1.
"""
import torch

from . import _lib


def _row(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("swiftx_b200 decode runs on CUDA tensors only (no CPU path)")
    if t.dtype != torch.float32:
        raise ValueError("decode step expects fp32 tensors")
    return t if t.stride(-1) == 1 else t.contiguous()


def _expect(name, t, shape):
    """Raise unless t (when given) has exactly this shape: the kernels index it through a
    bare pointer with the sizes of x, the weights and the states."""
    if t is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")


def _expect_vec(name, t, n):
    """Raise unless t (when given) holds exactly n values (a per-channel vector)."""
    if t is not None and t.numel() != n:
        raise ValueError(f"{name}: expected {n} values, got {t.numel()}")


def _call(mode, x, conv_state=None, conv_weight=None, conv_bias=None, z=None, delta=None, B=None,
          C=None, A=None, Dskip=None, delta_bias=None, ssm_state=None, delta_softplus=True,
          want_xc=False, A_is_log=False, group_w=None, group_of=None, dt_in=None, dt_weight=None):
    lib = _lib.load()
    x, z, delta, B, C = map(_row, (x, z, delta, B, C))
    if x.dim() != 2:
        raise ValueError(f"x: expected (b, D), got {tuple(x.shape)}")
    b, D = x.shape
    _expect("z", z, (b, D))
    a = _lib.DecodeArgs()
    a.batch, a.dim, a.mode = b, D, mode
    a.delta_softplus = 1 if delta_softplus else 0
    a.flags = _lib.SWX_DECODE_A_LOG if A_is_log else 0
    a.x, a.x_sb = x.data_ptr(), x.stride(0)
    keep = []
    if mode & _lib.SWX_DECODE_CONV:
        if not conv_state.is_contiguous() or conv_state.dtype != torch.float32:
            raise ValueError("conv_state must be a dense fp32 (b, D, K) tensor")
        if conv_weight.shape[0] != D or conv_weight.numel() % D:
            raise ValueError(f"conv_weight: expected (D, K) or (D, 1, K) with D={D}, got {tuple(conv_weight.shape)}")
        w = conv_weight.detach().reshape(D, -1).float().contiguous()
        _expect("conv_state", conv_state, (b, D, w.shape[1]))
        _expect_vec("conv_bias", conv_bias, D)
        keep.append(w)
        a.width = w.shape[1]
        a.conv_weight, a.conv_state = w.data_ptr(), conv_state.data_ptr()
        if conv_bias is not None:
            cb = conv_bias.detach().float().contiguous()
            keep.append(cb)
            a.conv_bias = cb.data_ptr()
    xc = None
    if want_xc or not (mode & _lib.SWX_DECODE_SSM):
        xc = torch.empty((b, D), device=x.device, dtype=torch.float32)
        a.xc_out = xc.data_ptr()
    out = None
    if mode & _lib.SWX_DECODE_SSM:
        if not ssm_state.is_contiguous() or ssm_state.dtype != torch.float32:
            raise ValueError("ssm_state must be a dense fp32 (b, D, N) tensor")
        if A.dim() != 2 or A.shape[0] != D:
            raise ValueError(f"A: expected (D, N) with D={D}, got {tuple(A.shape)}")
        Af = A.detach().float().contiguous()
        N = Af.shape[1]
        _expect("ssm_state", ssm_state, (b, D, N))
        _expect("delta", delta, (b, D))
        _expect("B", B, (b, N))
        _expect("C", C, (b, N))
        _expect_vec("Dskip", Dskip, D)
        _expect_vec("delta_bias", delta_bias, D)
        keep.append(Af)
        a.dstate = N
        out = torch.empty((b, D), device=x.device, dtype=torch.float32)
        if dt_in is not None:                     # dt_proj folded into the kernel
            dti = _row(dt_in)
            if dti.stride(0) % 4 or dti.data_ptr() % 16:
                dti = dti.contiguous()
            dtw = dt_weight.detach().float().contiguous()
            _expect("dt_weight", dtw, (D, dtw.shape[1] if dtw.dim() == 2 else -1))
            _expect("dt_in", dti, (b, dtw.shape[1]))
            keep += [dti, dtw]
            a.dt_in, a.dt_in_sb, a.dt_weight, a.dt_rank = dti.data_ptr(), dti.stride(0), dtw.data_ptr(), dtw.shape[1]
        else:
            a.delta, a.delta_sb = delta.data_ptr(), delta.stride(0)
        a.B, a.B_sb, a.C, a.C_sb = B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0)
        a.A, a.ssm_state, a.out = Af.data_ptr(), ssm_state.data_ptr(), out.data_ptr()
        if z is not None:
            a.z, a.z_sb = z.data_ptr(), z.stride(0)
        if group_w is not None:                   # the SiftX pathway mix, before the gate
            gw = group_w.detach().float().contiguous()
            gof = group_of.to(torch.int32).contiguous()
            _expect("group_w", gw, (b, gw.shape[1] if gw.dim() == 2 else -1))
            _expect_vec("group_of", gof, D)
            keep += [gw, gof]
            a.group_w, a.group_w_sb, a.group_of, a.ngroups = gw.data_ptr(), gw.stride(0), gof.data_ptr(), gw.shape[1]
        for name, t in (("Dskip", Dskip), ("delta_bias", delta_bias)):
            if t is not None:
                tf = t.detach().float().contiguous()
                keep.append(tf)
                setattr(a, name, tf.data_ptr())
    _lib.check(lib.swx_decode_step(a, _lib.stream_ptr(x.device)), "swx_decode_step")
    return out, xc


def decode_conv_step(x, conv_state, conv_weight, conv_bias=None):
    """Returns xc (b, D); conv_state (b, D, K) is updated in place."""
    return _call(_lib.SWX_DECODE_CONV, x, conv_state, conv_weight, conv_bias)[1]


def decode_ssm_step(xc, delta, B, C, A, ssm_state, Dskip=None, z=None, delta_bias=None,
                    delta_softplus=True, A_is_log=False, group_w=None, group_of=None, dt_in=None,
                    dt_weight=None):
    """Returns out (b, D); ssm_state (b, D, N) is updated in place.  A_is_log: A holds
    log(-A) (the block's A_log parameter) and the kernel forms A = -exp(A_log) itself.
    group_w (b, G), group_of (D,): the SiftX pathway mix applied before the gate (with z),
    out = y * group_w[:, group_of] * silu(z).  dt_in (b, R), dt_weight (D, R): dt_proj
    folded into the kernel, delta = dt_in @ dt_weight.T (pass delta=None); R a multiple of
    4, at most 256."""
    if dt_in is not None and (delta is not None or dt_weight is None):
        raise ValueError("dt_in replaces delta and needs dt_weight")
    return _call(_lib.SWX_DECODE_SSM, xc, z=z, delta=delta, B=B, C=C, A=A, Dskip=Dskip,
                 delta_bias=delta_bias, ssm_state=ssm_state, delta_softplus=delta_softplus,
                 A_is_log=A_is_log, group_w=group_w, group_of=group_of, dt_in=dt_in, dt_weight=dt_weight)[0]


def decode_step(x, conv_state, conv_weight, conv_bias, delta, B, C, A, ssm_state, Dskip=None,
                z=None, delta_bias=None, delta_softplus=True, return_xc=False, A_is_log=False):
    """Fused conv-window shift + conv + SiLU + state update + readout + gate.
    Returns out (b, D) (and xc when asked); both states are updated in place.
    A_is_log: A holds log(-A), as in decode_ssm_step."""
    out, xc = _call(_lib.SWX_DECODE_CONV | _lib.SWX_DECODE_SSM, x, conv_state, conv_weight, conv_bias,
                    z, delta, B, C, A, Dskip, delta_bias, ssm_state, delta_softplus, want_xc=return_xc,
                    A_is_log=A_is_log)
    return (out, xc) if return_xc else out


def decode_layer_step(x, conv_state, conv_weight, conv_bias, xproj_weight, dt_weight, A, ssm_state, Dskip=None,
                      z=None, delta_bias=None, delta_softplus=True, A_is_log=False):
    """One block's recurrent step between in_proj and out_proj with x_proj and dt_proj
    folded into the kernels (models/sift_block.py:160-175): two launches, no GEMM.
    x, z (b, D) fp32 rows (unit element stride); conv_state (b, D, 4), ssm_state (b, D, 16)
    updated in place; xproj_weight (R + 32, D), dt_weight (D, R).  Returns out (b, D), or
    None when the shape is not one the fused path takes (d_state 16, width 4, D a
    multiple of 64, R a multiple of 4 up to 256, 16-byte aligned rows)."""
    lib = _lib.load()
    x, z = _row(x), _row(z)
    b, D = x.shape
    Af = A.detach().float().contiguous()
    N = Af.shape[1]
    w = conv_weight.detach().reshape(D, -1).float().contiguous()
    xw = xproj_weight.detach().float().contiguous()
    dtw = dt_weight.detach().float().contiguous()
    R = dtw.shape[1]
    if (N != 16 or w.shape[1] != 4 or D % 64 or R % 4 or R > _lib.SWX_DECODE_MAX_DT_RANK
            or xw.shape != (R + 2 * N, D) or not conv_state.is_contiguous() or not ssm_state.is_contiguous()):
        return None
    if x.stride(0) % 4 or x.data_ptr() % 16 or (z is not None and (z.stride(0) % 4 or z.data_ptr() % 16)):
        return None
    # a shape the path takes: the remaining operands must match it (bare pointers below)
    _expect("z", z, (b, D))
    _expect("A", Af, (D, N))
    _expect("dt_weight", dtw, (D, R))
    _expect("conv_state", conv_state, (b, D, 4))
    _expect("ssm_state", ssm_state, (b, D, N))
    for name, t in (("conv_bias", conv_bias), ("Dskip", Dskip), ("delta_bias", delta_bias)):
        _expect_vec(name, t, D)
    keep = [w, Af, xw, dtw]
    a = _lib.DecodeArgs()
    a.batch, a.dim, a.dstate, a.width = b, D, N, 4
    a.mode = _lib.SWX_DECODE_CONV | _lib.SWX_DECODE_SSM
    a.delta_softplus = 1 if delta_softplus else 0
    a.flags = _lib.SWX_DECODE_A_LOG if A_is_log else 0
    a.x, a.x_sb = x.data_ptr(), x.stride(0)
    if z is not None:
        a.z, a.z_sb = z.data_ptr(), z.stride(0)
    a.conv_weight, a.conv_state = w.data_ptr(), conv_state.data_ptr()
    for name, t in (("conv_bias", conv_bias), ("Dskip", Dskip), ("delta_bias", delta_bias)):
        if t is not None:
            tf = t.detach().float().contiguous()
            keep.append(tf)
            setattr(a, name, tf.data_ptr())
    out = torch.empty((b, D), device=x.device, dtype=torch.float32)
    a.A, a.ssm_state, a.out = Af.data_ptr(), ssm_state.data_ptr(), out.data_ptr()
    a.dt_weight, a.dt_rank = dtw.data_ptr(), R
    a.xproj_weight, a.xproj_rows = xw.data_ptr(), R + 2 * N
    wsb = lib.swx_decode_layer_workspace_bytes(b, D, R + 2 * N)
    ws = torch.empty(max(wsb, 16), device=x.device, dtype=torch.uint8)
    a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
    _lib.check(lib.swx_decode_layer_step(a, _lib.stream_ptr(x.device)), "swx_decode_layer_step")
    return out
