"""Sift (Mamba-1) block and language model on the B200 hot path.

A caller-side mirror of the reference's models/sift_block.py and models/sift_model.py:
same constructor arguments, same parameter names and shapes (so reference state_dicts
load unchanged: in_proj, conv1d (D,1,K)+bias, x_proj, dt_proj, A_log, D, out_proj, norm,
norm_f, embedding, tied lm_head), same forward / step / generate behaviour.  The mixer
runs on the sm_100a kernels:

  in_proj (cuBLAS) -> causal conv1d + SiLU (kernel, reads the strided x half in place)
  -> x_proj (cuBLAS) -> dt_proj without bias (cuBLAS)
  -> fused selective scan with A = -exp(A_log), softplus(delta + dt_proj.bias), D skip
     and the SiLU(z) gate (kernel) -> out_proj (cuBLAS)

and decode runs the conv-window kernel, the x_proj GEMV and the state-update kernel (which,
for small batches, forms delta from the low-rank dt itself: dt_proj folded in).
RMSNorm runs on its fused kernels, each residual add folded into the next norm, and,
in training, the token embedding's weight gradient on the sort-free swx_embedding_bwd.
Fusing the gate is exactly the reference's y * silu(z) when no SiftX pathway mixing is
configured (models/sift_block.py:132-142).  With pathway_gate (SiftX), the per-token
group weights softmax(pathway(x)) x G are computed in torch (a (b, L, G) tensor) and the
scan kernels apply them between the scan and the gate, out = y * w[group] * silu(z),
returning their gradient from the backward (the decode kernel applies them too); with
more than 8 groups the mix and gate stay in torch.  The block runs fp32 or bf16
activations: the conv kernels have no float64 form (the scan's float64 kernels serve the
reference's own float64 callers).
"""
import math
from dataclasses import dataclass
from fractions import Fraction

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import embedding as embedding_kernels
from . import norm as norm_kernels
from .conv import causal_conv1d_fn, conv1d_backward, conv1d_forward
from .decode import decode_conv_step, decode_layer_step, decode_ssm_step
from .selective_scan import scan_backward, scan_forward, selective_scan_fn


# bf16 copies of the projection weights for the current SiftLM forward under bf16 autocast
# (id(fp32 weight) -> bf16 view), or None: see _Bf16Linear and SiftLM.forward.  Set only
# for the duration of one SiftLM.forward or GraphedStep build and restored afterwards.  A
# projection whose weight has no entry (another model's, or the table already restored
# by a concurrent forward in another thread) takes the plain F.linear path, which
# computes the same bf16 GEMM under autocast.
_W16 = None


class _Bf16Linear(torch.autograd.Function):
    """y = x @ W^T on a bf16 copy of the fp32 weight made beforehand -- the GEMM bf16
    autocast runs -- without autocast's per-call weight cast, and with the weight gradient
    returned in fp32 straight from the GEMM (mm with an fp32 output) instead of a bf16
    gradient cast back to the parameter's dtype: two elementwise launches fewer per
    projection and step, and dW is not rounded to bf16 on its way to the fp32 parameter."""

    @staticmethod
    def forward(ctx, x, weight, w16):
        ctx.save_for_backward(x, w16)
        return F.linear(x, w16)

    @staticmethod
    def backward(ctx, dy):
        x, w16 = ctx.saved_tensors
        dx = dy.matmul(w16) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = torch.mm(dy.reshape(-1, dy.shape[-1]).t(), x.reshape(-1, x.shape[-1]), out_dtype=torch.float32)
        return dx, dw, None


def _linear(x, weight, bias=None):
    """F.linear(x, weight, bias), through _Bf16Linear when the running SiftLM forward (or a
    GraphedStep) made a bf16 copy of ``weight`` (bias-free projections under bf16
    autocast).  An fp32 input is cast to bf16 first, as autocast casts it."""
    w16 = _W16.get(id(weight)) if _W16 is not None and bias is None else None
    if w16 is not None and x.dtype == torch.float32 and torch.is_autocast_enabled("cuda") \
            and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        x = x.to(torch.bfloat16)
    if w16 is None or x.dtype != torch.bfloat16:
        return F.linear(x, weight, bias)
    return _Bf16Linear.apply(x, weight, w16)


def _bf16_copies(weights, flat=None):
    """bf16 copies of fp32 weights in two launches (one concatenation, one cast) instead
    of one cast per weight: {id(weight): bf16 view}.  ``flat``: an existing bf16 buffer of
    the right size to refresh in place (its views stay valid)."""
    with torch.no_grad():
        if flat is None:
            flat = torch.cat([w.reshape(-1) for w in weights]).to(torch.bfloat16)
        else:
            flat.copy_(torch.cat([w.reshape(-1) for w in weights]))
    out, off = {}, 0
    for w in weights:
        out[id(w)] = flat[off:off + w.numel()].view_as(w)
        off += w.numel()
    return out


# Largest batch whose decode step folds the projections into the kernels (see
# SiftBlock.step).
_FOLD_DT_MAX_BATCH = 32

# Training forwards of pathway-free blocks under bf16 autocast (with the bf16 weight
# copies) run the mixer between in_proj and out_proj as one autograd Function
# (_MixerCore); False keeps the per-op autograd graph.
_FUSED_CORE = True


class _MixerCore(torch.autograd.Function):
    """The mixer between in_proj and out_proj as one autograd node: conv1d + SiLU on the x
    half of xz, x_proj, dt_proj, and the gated selective scan with softplus(delta + bias),
    A = -exp(A_log) and the D skip (models/sift_block.py:111-135).  The forward runs the
    same kernels and GEMMs as the per-op graph, so its output has the same bits.  The
    backward writes the scan's dz and the conv's dx straight into the two halves of one
    d(xz) buffer (no concatenation), and adds the scan's du to x_proj's input gradient
    inside that GEMM (addmm; no separate add of the conv output's two gradients).
    Weights: the fp32 parameters receive the gradients (fp32 straight from the GEMMs, as
    _Bf16Linear); the GEMMs use the forward's bf16 copies."""

    @staticmethod
    def forward(ctx, xz, conv_w, conv_b, xw, xw16, dtw, dtw16, A_log, Dp, dt_bias):
        Dm = xz.shape[-1] // 2
        R = dtw.shape[1]
        with torch.autocast(device_type="cuda", enabled=False):
            x, z = xz[..., :Dm], xz[..., Dm:]
            xc = conv1d_forward(x, conv_w, conv_b, True)
            x_dbl = F.linear(xc, xw16)
            N = (x_dbl.shape[-1] - R) // 2
            delta = F.linear(x_dbl[..., :R], dtw16)
            pre = torch.empty(xc.shape, device=xc.device, dtype=torch.float32)
            y, ck, _ = scan_forward(xc, delta, A_log, x_dbl[..., R:R + N], x_dbl[..., R + N:], Dp, z, dt_bias, True,
                                    checkpoints=True, pre_out=pre, A_is_log=True)
        ctx.save_for_backward(xz, conv_w, conv_b, xc, x_dbl, delta, ck, pre, xw16, dtw16, A_log, Dp, dt_bias)
        ctx.dims = (Dm, R, N)
        return y

    @staticmethod
    def backward(ctx, dy):
        xz, conv_w, conv_b, xc, x_dbl, delta, ck, pre, xw16, dtw16, A_log, Dp, dt_bias = ctx.saved_tensors
        Dm, R, N = ctx.dims
        b, L = xz.shape[0], xz.shape[1]
        with torch.autocast(device_type="cuda", enabled=False):
            dxz = torch.empty_like(xz)
            x, z = xz[..., :Dm], xz[..., Dm:]
            g = scan_backward(xc, delta, A_log, x_dbl[..., R:R + N], x_dbl[..., R + N:], Dp, z, dt_bias, True, None,
                              ck, dy.to(xz.dtype), y_pre=pre, A_is_log=True, dz_out=dxz[..., Dm:])
            dd = g["ddelta"].reshape(-1, Dm)
            x_dbl2 = x_dbl.reshape(-1, R + 2 * N)
            dwdt = torch.mm(dd.t(), x_dbl2[:, :R], out_dtype=torch.float32)                    # dt_proj
            dx_dbl = torch.cat([torch.mm(dd, dtw16), g["dB"].reshape(-1, N), g["dC"].reshape(-1, N)], dim=1)
            dwx = torch.mm(dx_dbl.t(), xc.reshape(-1, Dm), out_dtype=torch.float32)            # x_proj
            dxc = torch.addmm(g["du"].reshape(-1, Dm), dx_dbl, xw16)      # du + d(x_proj input)
            _, dcw, dcb = conv1d_backward(x, conv_w, conv_b, dxc.view(b, L, Dm), True, dx_out=dxz[..., :Dm])
        dcb = dcb.to(conv_b.dtype) if dcb is not None else None
        return (dxz, dcw.reshape(conv_w.shape).to(conv_w.dtype), dcb, dwx, None, dwdt, None,
                g["dA"], g["dD"], g["ddelta_bias"])


# ----------------------------------------------------------------- parameter table
# The block's parameters as data: state_dict key, shape (from the block's dimensions),
# initial distribution, and whether it is excluded from weight decay.  The keys and
# shapes are the reference's (models/sift_block.py:30-101) so its checkpoints load; the
# distributions are the ones its initialisers produce:
#   "fan_in"      U(-s/sqrt(fan_in), +s/sqrt(fan_in)), fan_in = every dim but the first
#                 (torch's default for Linear / Conv1d weights, and dt_proj.weight's
#                 U(+-dt_rank^-1/2)); s = 1/sqrt(n_layers) for out_proj inside a backbone
#   "fan_in_of:K" the same bound as parameter K's (a Conv1d bias)
#   "dt_bias"     inverse softplus of dt, log-uniform over each timescale group's range,
#                 floored at 1e-4 (models/ssm.py:54-71)
#   "s4d_log"     log(n + 1) for state n in every channel: A = -(n + 1) (models/ssm.py:43-51)
#   "ones" / "zeros"
_BLOCK_TABLE = (
    # key              shape                                        init             no decay  when
    ("A_log",          lambda m: (m.d_inner, m.d_state),             "s4d_log",       True,  None),
    ("D",              lambda m: (m.d_inner,),                       "ones",          True,  None),
    ("in_proj.weight", lambda m: (2 * m.d_inner, m.d_model),         "fan_in",        False, None),
    ("in_proj.bias",   lambda m: (2 * m.d_inner,),                   "zeros",         False, "bias"),
    ("conv1d.weight",  lambda m: (m.d_inner, 1, m.d_conv),           "fan_in",        False, None),
    ("conv1d.bias",    lambda m: (m.d_inner,),                       "fan_in_of:conv1d.weight", False, "conv_bias"),
    ("x_proj.weight",  lambda m: (m.dt_rank + 2 * m.d_state, m.d_inner), "fan_in",    False, None),
    ("dt_proj.weight", lambda m: (m.d_inner, m.dt_rank),             "fan_in",        False, None),
    ("dt_proj.bias",   lambda m: (m.d_inner,),                       "dt_bias",       False, None),
    ("pathway.weight", lambda m: (m.n_groups, m.d_inner),            "zeros",         False, "pathway"),
    ("pathway.bias",   lambda m: (m.n_groups,),                      "zeros",         False, "pathway"),
    ("out_proj.weight", lambda m: (m.d_model, m.d_inner),            "fan_in",        False, None),
    ("out_proj.bias",  lambda m: (m.d_model,),                       "zeros",         False, "bias"),
)


class _Slot(nn.Module):
    """The tensors of one named projection (``weight`` and, when it has one, ``bias``),
    so that state_dict keys read ``<name>.weight`` / ``<name>.bias``."""

    def __init__(self):
        super().__init__()
        self.register_parameter("bias", None)       # replaced when the table gives one


def _fan_in(t):
    return math.prod(t.shape[1:])


def _log_uniform(n, lo, hi):
    return torch.exp(torch.empty(n).uniform_(math.log(lo), math.log(hi)))


def _inverse_softplus(y):
    """x with softplus(x) = y: y + log(1 - exp(-y))."""
    return y + torch.log(-torch.expm1(-y))


class SiftBlock(nn.Module):
    """The Sift mixer (models/sift_block.py:30) on the B200 kernels.  Same constructor
    arguments, parameter names and shapes as the reference; built from _BLOCK_TABLE."""

    def __init__(self, d_model, d_state=16, d_conv=4, expand=2, dt_rank="auto", dt_min=1e-3,
                 dt_max=1e-1, conv_bias=True, bias=False, scan_impl="fast", scan_mode="auto",
                 timescales=None, pathway_gate=False, out_scale=1.0):
        super().__init__()
        self.d_model, self.d_state, self.d_conv = d_model, d_state, d_conv
        self.d_inner = expand * d_model
        self.dt_rank = -(-d_model // 16) if dt_rank == "auto" else dt_rank
        self.scan_impl, self.scan_mode = scan_impl, scan_mode    # every impl / mode runs the same kernels
        # SiftX multi-timescale groups (models/sift_block.py:74-93): contiguous channel groups
        # of nearly equal size, each with its own dt range; pathway_gate adds a per-token
        # softmax over the groups
        self.timescales = [tuple(t) for t in timescales] if timescales else None
        ranges = self.timescales or [(dt_min, dt_max)]
        self.n_groups = len(ranges)
        G, Dn = self.n_groups, self.d_inner
        edges = [round(Fraction(i * Dn, G)) for i in range(G + 1)]     # ties to even, as torch.round
        group_of = torch.zeros(Dn, dtype=torch.long)
        for i in range(G):
            group_of[edges[i]:edges[i + 1]] = i
        self.register_buffer("group_of", group_of, persistent=False)
        # the same map as the kernels take it (int32), so no conversion runs per call
        self.register_buffer("group_of_i32", group_of.to(torch.int32), persistent=False)
        present = {"bias": bias, "conv_bias": conv_bias, "pathway": bool(pathway_gate and G > 1)}
        for key, shape, rule, no_decay, when in _BLOCK_TABLE:
            if when is not None and not present[when]:
                continue
            slot_name, _, leaf = key.rpartition(".")
            owner = self
            if slot_name:
                if not hasattr(self, slot_name) or getattr(self, slot_name) is None:
                    self.add_module(slot_name, _Slot())
                owner = getattr(self, slot_name)
            prm = nn.Parameter(torch.empty(shape(self)))
            if no_decay:
                prm._no_weight_decay = True
            if leaf in owner._parameters:
                del owner._parameters[leaf]
            owner.register_parameter(leaf, prm)
        if not present["pathway"]:
            self.pathway = None
        self._initialise(ranges, out_scale)

    @torch.no_grad()
    def _initialise(self, ranges, out_scale=1.0):
        """Draw every parameter from its distribution in _BLOCK_TABLE."""
        params = dict(self.named_parameters())
        for key, _, rule, _, _ in _BLOCK_TABLE:
            t = params.get(key)
            if t is None:
                continue
            if rule == "ones":
                t.fill_(1.0)
            elif rule == "zeros":
                t.zero_()
            elif rule == "s4d_log":
                t.copy_(torch.log(torch.arange(1, self.d_state + 1, dtype=torch.float32)).expand_as(t))
            elif rule.startswith("fan_in"):
                ref = params[rule.split(":", 1)[1]] if ":" in rule else t
                bound = 1.0 / math.sqrt(_fan_in(ref))
                if key == "out_proj.weight":
                    bound *= out_scale
                t.uniform_(-bound, bound)
            elif rule == "dt_bias":
                edges = [round(Fraction(i * self.d_inner, len(ranges))) for i in range(len(ranges) + 1)]
                for (lo, hi), a, b in zip(ranges, edges[:-1], edges[1:]):
                    t[a:b] = _inverse_softplus(_log_uniform(b - a, lo, hi).clamp(min=1e-4))
            else:
                raise ValueError(f"unknown init rule {rule!r} for {key}")

    def _split(self, x):
        x_dbl = _linear(x, self.x_proj.weight)
        dt, B, C = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        return _linear(dt, self.dt_proj.weight), B, C       # dt_proj bias fused into the scan

    def projection_weights(self):
        """The fp32 weights of the bias-free projections (in_proj, x_proj, dt_proj, out_proj)."""
        return [m.weight for m in (self.in_proj, self.x_proj, self.dt_proj, self.out_proj)
                if m is self.dt_proj or m.bias is None]

    def _core_weights(self, xz):
        """The bf16 copies of x_proj's and dt_proj's weights when this forward can run the
        mixer as one _MixerCore node (training, bf16, no pathway mix), else None."""
        if not (_FUSED_CORE and _W16 is not None and self.pathway is None and torch.is_grad_enabled()
                and xz.is_cuda and xz.dtype == torch.bfloat16 and self.x_proj.bias is None
                and self.conv1d.bias is not None and self.d_inner % 2 == 0):
            return None
        w = (_W16.get(id(self.x_proj.weight)), _W16.get(id(self.dt_proj.weight)))
        return w if w[0] is not None and w[1] is not None else None

    def forward(self, hidden):
        """hidden: (b, L, d_model) -> (b, L, d_model)"""
        xz = _linear(hidden, self.in_proj.weight, self.in_proj.bias)
        w16 = self._core_weights(xz)
        if w16 is not None:
            y = _MixerCore.apply(xz, self.conv1d.weight, self.conv1d.bias, self.x_proj.weight, w16[0],
                                 self.dt_proj.weight, w16[1], self.A_log, self.D, self.dt_proj.bias)
            return _linear(y, self.out_proj.weight, self.out_proj.bias)
        x, z = xz.chunk(2, dim=-1)                        # strided views, row stride 2D
        x = causal_conv1d_fn(x, self.conv1d.weight, self.conv1d.bias, "silu")
        delta, B, C = self._split(x)
        fuse_mix = self.pathway is not None and self._mix_fusable(x)
        gate = z if self.pathway is None or fuse_mix else None
        # SiftX: the per-token group weights (models/sift_block.py:140), computed under the
        # caller's autocast like the reference; the kernels apply them before the gate
        gw = self._pathway_weights(x) if fuse_mix else None
        with torch.autocast(device_type=x.device.type, enabled=False):
            # A = -exp(A_log) is formed inside the scan kernels (A_is_log)
            y = selective_scan_fn(x, delta, self.A_log.float(), B, C, self.D.float(), z=gate,
                                  delta_bias=self.dt_proj.bias.float(), delta_softplus=True, A_is_log=True,
                                  group_w=gw, group_of=self.group_of_i32 if fuse_mix else None)
        y = y.to(xz.dtype)
        if self.pathway is not None and not fuse_mix:
            y = self._mix_pathways(y, x) * F.silu(z)
        return _linear(y, self.out_proj.weight, self.out_proj.bias)

    def _pathway_weights(self, x):
        """softmax(pathway(x)) x G: (b, L, G) per-token group weights (models/sift_block.py:140)."""
        return torch.softmax(F.linear(x, self.pathway.weight, self.pathway.bias), dim=-1) * self.n_groups

    def _mix_fusable(self, x):
        """The scan kernels apply the group mix themselves for fp32 / bf16 inputs and at
        most SWX_MAX_GROUPS groups; more groups keep the mix in torch."""
        return x.dtype in (torch.float32, torch.bfloat16) and self.n_groups <= 8

    def _mix_pathways(self, y, x):
        """SiftX: reweight the channel groups per token, softmax x G (1 at init)
        (models/sift_block.py:137-142); the unfused form, for more than 8 groups."""
        return y * self._pathway_weights(x)[..., self.group_of]

    def allocate_state(self, batch, device=None, dtype=torch.float32):
        """(conv window (b, D, d_conv), SSM state (b, D, d_state)), zeroed: the recurrent
        state that step() updates in place (models/sift_block.py:148-151 layout)."""
        shapes = ((batch, self.d_inner, self.d_conv), (batch, self.d_inner, self.d_state))
        return tuple(torch.zeros(sh, device=device, dtype=dtype) for sh in shapes)

    def step(self, hidden, state):
        """hidden: (b, d_model) one token; state (conv_state, ssm_state) updated in place."""
        conv_state, ssm_state = state
        xz = _linear(hidden, self.in_proj.weight, self.in_proj.bias).float()
        x, z = xz.chunk(2, dim=-1)
        if self.pathway is None and hidden.shape[0] <= _FOLD_DT_MAX_BATCH:
            # small batches: conv, x_proj, dt_proj, state update and gate in two launches
            # with both projections inside the kernels (None: a shape the path does not
            # take).  Measured on the graphed 24-layer d_model 1024 step, ms per token
            # fp32 / bf16 projections: batch 1, 0.97 / 1.19 against 1.12 / 1.45 with the
            # GEMMs; batch 16, 1.98 / 1.29 against 2.21 / 1.50; batch 64, 3.19 / 1.69
            # against 3.23 / 1.58; batch 256, 5.44 / 3.64 against 3.97 / 2.03
            y = decode_layer_step(x, conv_state, self.conv1d.weight, self.conv1d.bias, self.x_proj.weight,
                                  self.dt_proj.weight, self.A_log, ssm_state, Dskip=self.D, z=z,
                                  delta_bias=self.dt_proj.bias, A_is_log=True)
            if y is not None:
                return _linear(y.to(self.out_proj.weight.dtype), self.out_proj.weight, self.out_proj.bias)
        xc = decode_conv_step(x, conv_state, self.conv1d.weight, self.conv1d.bias)
        fuse_mix = self.pathway is not None and self.n_groups <= 8
        gate = z if self.pathway is None or fuse_mix else None
        gw = self._pathway_weights(xc).float() if fuse_mix else None
        # A = -exp(A_log) is formed inside the kernel (A_is_log) and the pathway mix applied
        # there.  For small batches dt_proj is folded in too (the kernel forms
        # delta = dt_proj.weight @ dt itself, models/sift_block.py:167,106-108), which saves
        # the GEMM's launch; from a few dozen rows on, the GEMM plus the plain kernel is
        # faster (2.14 against 2.21 ms per token at batch 16, 4.08 against 3.97 at batch
        # 256, fp32, on the step above)
        x_dbl = _linear(xc, self.x_proj.weight)
        dt, B, C = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        fold = self.dt_rank % 4 == 0 and self.dt_rank <= 256 and hidden.shape[0] <= _FOLD_DT_MAX_BATCH
        y = decode_ssm_step(xc, None if fold else _linear(dt, self.dt_proj.weight).float(), B.float(), C.float(),
                            self.A_log, ssm_state, Dskip=self.D, z=gate, delta_bias=self.dt_proj.bias,
                            A_is_log=True, group_w=gw, group_of=self.group_of_i32 if fuse_mix else None,
                            dt_in=dt.float() if fold else None, dt_weight=self.dt_proj.weight if fold else None)
        if self.pathway is not None and not fuse_mix:
            y = self._mix_pathways(y, xc) * F.silu(z)
        return _linear(y.to(self.out_proj.weight.dtype), self.out_proj.weight, self.out_proj.bias)


class RMSNorm(nn.Module):
    def __init__(self, d, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        """models/sift_model.py:25-26; on CUDA (fp32 / bf16, d <= 1024) one fused kernel
        each way, otherwise the reference expression itself.  Under bf16 autocast the
        result comes out in bf16: its consumers here (in_proj, the head) are Linear layers
        that autocast would cast it to bf16 anyway, and the kernel rounds the same fp32
        value once, so the cast (and its backward) is folded into the kernel."""
        if norm_kernels.supported(x):
            return norm_kernels.rms_norm(x, self.weight, self.eps, _norm_out_dtype())
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight

    def forward_residual(self, x, res):
        """(x + res, self(x + res)): the residual stream's add and this norm, on one fused
        kernel each way when the sum keeps x's dtype (fp32 residual stream), else the
        plain add and forward."""
        if norm_kernels.supported(x) and res.dtype in (torch.float32, torch.bfloat16) \
                and torch.promote_types(x.dtype, res.dtype) == x.dtype and res.shape == x.shape:
            return norm_kernels.add_rms_norm(x, res, self.weight, self.eps, _norm_out_dtype())
        s = x + res
        return s, self(s)


def _norm_out_dtype():
    """bf16 under bf16 autocast (the norm's consumers are Linear layers that would cast to
    bf16 anyway), else the input's dtype."""
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        return torch.bfloat16
    return None


@dataclass
class SiftConfig:
    """Model hyper-parameters; field names and defaults are the reference's
    (models/sift_model.py:30), so its YAML configs and call sites construct it unchanged."""
    vocab_size: int = 65
    d_model: int = 128
    n_layers: int = 4
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    dt_rank: object = "auto"
    scan_impl: str = "fast"
    scan_mode: str = "auto"
    tie_embeddings: bool = True
    timescales: object = None
    pathway_gate: bool = False


class _Layer(nn.Module):
    """One pre-norm residual layer, x + mixer(norm(x)); the attribute names ``norm`` and
    ``mixer`` give the reference's state_dict keys (backbone.layers.<i>.norm / .mixer)."""

    def __init__(self, cfg, out_scale):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model)
        self.mixer = SiftBlock(cfg.d_model, d_state=cfg.d_state, d_conv=cfg.d_conv, expand=cfg.expand,
                               dt_rank=cfg.dt_rank, scan_impl=cfg.scan_impl, scan_mode=cfg.scan_mode,
                               timescales=cfg.timescales, pathway_gate=cfg.pathway_gate, out_scale=out_scale)

    def forward(self, x):
        return x + self.mixer(self.norm(x))

    def step(self, x, state):
        return x + self.mixer.step(self.norm(x), state)


class SiftBackbone(nn.Module):
    """n_layers residual layers and the final norm.  Inside a backbone each layer's
    out_proj is drawn with its bound scaled by 1/sqrt(n_layers)."""

    def __init__(self, cfg):
        super().__init__()
        scale = 1.0 / math.sqrt(max(1, cfg.n_layers))
        self.layers = nn.ModuleList(_Layer(cfg, scale) for _ in range(cfg.n_layers))
        self.norm_f = RMSNorm(cfg.d_model)
        self.fuse_residual_norm = True

    def forward(self, x):
        if not self.fuse_residual_norm or not self.layers:
            for layer in self.layers:
                x = layer(x)
            return self.norm_f(x)
        # x_{i+1} = x_i + mixer_i(norm_i(x_i)), with each add folded into the next norm
        # (RMSNorm.forward_residual): the same values as the per-layer form above
        h = self.layers[0].mixer(self.layers[0].norm(x))
        for layer in self.layers[1:]:
            x, n = layer.norm.forward_residual(x, h)
            h = layer.mixer(n)
        return self.norm_f.forward_residual(x, h)[1]


class SiftLM(nn.Module):
    """Byte-level language model: token embedding (N(0, 0.02)), backbone, head tied to the
    embedding when cfg.tie_embeddings (state_dict keys embedding.weight, backbone.*,
    lm_head.weight, as models/sift_model.py:92-101)."""

    def __init__(self, cfg: SiftConfig):
        super().__init__()
        self.cfg = cfg
        self.embedding = _Slot()
        self.embedding.weight = nn.Parameter(torch.empty(cfg.vocab_size, cfg.d_model).normal_(0.0, 0.02))
        self.backbone = SiftBackbone(cfg)
        self.lm_head = _Slot()
        if cfg.tie_embeddings:
            self.lm_head.weight = self.embedding.weight
        else:
            bound = 1.0 / math.sqrt(cfg.d_model)
            self.lm_head.weight = nn.Parameter(torch.empty(cfg.vocab_size, cfg.d_model).uniform_(-bound, bound))
        self.bf16_weight_copies = True      # under bf16 autocast: see forward

    def forward(self, idx, targets=None):
        """Under bf16 autocast on CUDA (and bf16_weight_copies) the projection weights and
        the head's are cast to bf16 once per forward, in two launches, and the projections
        run through _Bf16Linear: the same bf16 GEMMs as autocast, without its per-call
        weight casts, and with fp32 weight gradients from the GEMM itself."""
        global _W16
        w = self.embedding.weight
        if embedding_kernels.supported(idx, w) and torch.is_grad_enabled():
            x = embedding_kernels.embedding(idx, w)
        else:
            x = F.embedding(idx, w)
        prev = _W16
        if self.bf16_weight_copies and w.is_cuda and torch.is_autocast_enabled("cuda") \
                and torch.get_autocast_dtype("cuda") == torch.bfloat16:
            ws = self.projection_weights()
            if ws is not None:
                _W16 = _bf16_copies(ws)
        try:
            logits = _linear(self.backbone(x), self.lm_head.weight, self.lm_head.bias)
        finally:
            _W16 = prev
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), targets.reshape(-1))
        return logits, loss

    def projection_weights(self):
        """The fp32 weights that have bf16 copies under bf16 autocast: every block's
        bias-free projections and the head's (None when one is not fp32)."""
        ws = [p for layer in self.backbone.layers for p in layer.mixer.projection_weights()]
        if self.lm_head.bias is None:
            ws.append(self.lm_head.weight)
        return ws if all(p.dtype == torch.float32 for p in ws) else None

    def allocate_state(self, batch, device=None):
        """One (conv window, SSM state) pair per layer, zeroed."""
        return [layer.mixer.allocate_state(batch, device) for layer in self.backbone.layers]

    def step(self, token, state):
        """Logits for one token per row, advancing ``state`` (from allocate_state) in place:
        the recurrent form of forward (models/sift_model.py:115)."""
        h = F.embedding(token, self.embedding.weight)
        for layer, st in zip(self.backbone.layers, state):
            h = layer.step(h, st)
        return _linear(self.backbone.norm_f(h), self.lm_head.weight, self.lm_head.bias)

    @torch.no_grad()
    def generate(self, idx, max_new_tokens, temperature=1.0, top_k=None, graphed=False):
        """The prompt ``idx`` (b, T) followed by ``max_new_tokens`` sampled tokens, produced
        through the recurrent step (the prompt is consumed token by token, then each new
        token is sampled from the last logits and fed back).  graphed=True replays each
        step from one CUDA graph (GraphedStep)."""
        if graphed:
            stepper = GraphedStep(self, idx.shape[0], idx.device)
            advance = lambda tok: stepper(tok).clone()  # noqa: E731
        else:
            state = self.allocate_state(idx.shape[0], idx.device)
            advance = lambda tok: self.step(tok, state)  # noqa: E731
        logits = None
        for tok in idx.unbind(1):
            logits = advance(tok)
        out = [idx]
        for i in range(max_new_tokens):
            tok = sample(logits, temperature, top_k)
            out.append(tok.unsqueeze(1))
            if i + 1 < max_new_tokens:          # the last token's logits are not needed
                logits = advance(tok)
        return torch.cat(out, dim=1)


class GraphedStep:
    """SiftLM.step for a fixed batch, replayed as one CUDA graph: the embedding, every
    layer's in_proj, conv-window kernel, x_proj / dt_proj, state-update kernel and
    out_proj, the norms and the head -- about fifteen launches per layer -- in one graph
    launch per token.  The recurrent state lives in buffers owned by this object and is
    updated in place by every call, as SiftLM.step updates its state.

    Calling returns the graph's static logits tensor (overwritten by the next call).
    autocast_dtype (e.g. torch.bfloat16) runs the projections under autocast, as the
    reference trainer does; the state and the decode kernels stay fp32.  Under bf16
    autocast (and model.bf16_weight_copies) the projection and head weights are cast to
    bf16 once, here, into a buffer the graph reads, instead of at every token as autocast
    does (the same bf16 values, without re-reading every fp32 weight per step); after
    changing the model's weights, call refresh_weights()."""

    def __init__(self, model, batch, device=None, autocast_dtype=None):
        global _W16
        dev = torch.device(device) if device is not None else next(model.parameters()).device
        self.model = model
        self.state = model.allocate_state(batch, dev)
        self.token = torch.zeros(batch, dtype=torch.long, device=dev)
        amp = lambda: torch.autocast("cuda", dtype=autocast_dtype, enabled=autocast_dtype is not None)  # noqa: E731
        self._weights, self._w16_flat, w16 = None, None, None
        if autocast_dtype == torch.bfloat16 and model.bf16_weight_copies and dev.type == "cuda":
            self._weights = model.projection_weights()
            if self._weights is not None:
                w16 = self.refresh_weights()
        prev = _W16
        _W16 = w16
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side), torch.no_grad(), amp():
                for _ in range(2):                    # one-time library and kernel setup
                    model.step(self.token, self.state)
            torch.cuda.current_stream(dev).wait_stream(side)
            self.reset()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph), torch.no_grad(), amp():
                self.logits = model.step(self.token, self.state)
        finally:
            _W16 = prev

    def refresh_weights(self):
        """Re-take the bf16 copies of the projection weights (after the model's weights
        changed), in place; a no-op without them.  Returns {id(weight): bf16 view}."""
        if self._weights is None:
            return None
        if self._w16_flat is None:
            n = sum(w.numel() for w in self._weights)
            self._w16_flat = torch.empty(n, dtype=torch.bfloat16, device=self._weights[0].device)
        return _bf16_copies(self._weights, flat=self._w16_flat)

    def reset(self):
        """Zero the recurrent state (a fresh sequence)."""
        for conv_state, ssm_state in self.state:
            conv_state.zero_()
            ssm_state.zero_()

    @torch.no_grad()
    def __call__(self, token):
        self.token.copy_(token)
        self.graph.replay()
        return self.logits


def sample(logits, temperature=1.0, top_k=None):
    """One token id per row from (b, vocab) logits: greedy at temperature 0, otherwise
    drawn from softmax(logits / temperature), restricted to the top_k largest when top_k
    is given (exactly k candidates; the reference keeps every logit tied with the k-th)."""
    if temperature == 0:
        return logits.argmax(-1)
    scaled = logits.float() / temperature
    if top_k is None:
        return torch.multinomial(torch.softmax(scaled, -1), 1).squeeze(-1)
    vals, ids = scaled.topk(min(top_k, scaled.shape[-1]), dim=-1)
    pick = torch.multinomial(torch.softmax(vals, -1), 1)
    return ids.gather(-1, pick).squeeze(-1)


def count_params(model):
    """Number of parameter values (a tied head counted once)."""
    return sum(t.numel() for t in {id(p): p for p in model.parameters()}.values())
