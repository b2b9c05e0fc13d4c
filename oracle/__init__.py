"""CPU oracle for the selective-scan hot path -- TEST INFRASTRUCTURE ONLY.

A float64 C restatement (``scan_oracle.c``) of the reference's algorithms:

* ``scan_fwd``   -- models/selective_scan.py:34-60 (selective_scan_ref) plus the
  block's softplus (models/sift_block.py:108) and SiLU(z) gate (:134);
* ``scan_bwd``   -- models/selective_scan.py:211-243 (_FusedScanFn.backward) chained
  through the gate and softplus;
* ``conv1d_fwd`` / ``conv1d_bwd`` -- models/sift_block.py:62-65,117-118;
* ``decode_step`` -- models/sift_block.py:153-175.

It is pinned against golden vectors produced by the reference itself
(``tests/golden``).  Only the tests, ``__graft_entry__.smoke`` and the CPU
baseline of ``bench.py`` use it; the product package never imports it.
All functions take numpy arrays in the reference layouts and return float64.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_dp = ctypes.POINTER(ctypes.c_double)


def build():
    """Compile scan_oracle.c into oracle/_build/liboracle.so."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
                os.path.join(_HERE, "scan_oracle.c")):
            build()
        _lib = ctypes.CDLL(_SO)
    return _lib


def _arr(x):
    if x is None:
        return None
    if hasattr(x, "detach"):                      # torch tensor
        x = x.detach().cpu().double().numpy()
    return np.ascontiguousarray(x, dtype=np.float64)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_dp)


def num_threads():
    return _load().orc_num_threads()


def set_num_threads(n):
    _load().orc_set_num_threads(ctypes.c_int(int(n)))


def scan_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
             h0=None, return_ypre=False, return_last_state=False):
    """Forward scan.  u, delta, z: (b,L,D); A: (D,N); B, C: (b,L,N); D, delta_bias: (D,).

    Returns out, plus ypre (pre-gate y) and/or h_last (b,D,N) when asked.
    """
    lib = _load()
    u, delta, A, B, C, D, z, delta_bias, h0 = map(_arr, (u, delta, A, B, C, D, z, delta_bias, h0))
    b, L, Dm = u.shape
    N = A.shape[1]
    out = np.empty((b, L, Dm))
    ypre = np.empty((b, L, Dm)) if return_ypre else None
    hl = np.empty((b, Dm, N)) if return_last_state else None
    lib.orc_scan_fwd(b, L, Dm, N, _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D),
                     _ptr(z), _ptr(delta_bias), int(bool(delta_softplus)), _ptr(h0),
                     _ptr(out), _ptr(ypre), _ptr(hl))
    res = [out]
    if return_ypre:
        res.append(ypre)
    if return_last_state:
        res.append(hl)
    return res[0] if len(res) == 1 else tuple(res)


def scan_bwd(u, delta, A, B, C, dout, D=None, z=None, delta_bias=None, delta_softplus=False,
             h0=None):
    """Backward scan.  Returns a dict with du, ddelta, dA, dB, dC and, when the matching
    input was given, dD, dz, ddelta_bias, dh0."""
    lib = _load()
    u, delta, A, B, C, D, z, delta_bias, h0, dout = map(
        _arr, (u, delta, A, B, C, D, z, delta_bias, h0, dout))
    b, L, Dm = u.shape
    N = A.shape[1]
    g = {"du": np.empty((b, L, Dm)), "ddelta": np.empty((b, L, Dm)), "dA": np.empty((Dm, N)),
         "dB": np.empty((b, L, N)), "dC": np.empty((b, L, N))}
    g["dD"] = np.empty(Dm) if D is not None else None
    g["dz"] = np.empty((b, L, Dm)) if z is not None else None
    g["ddelta_bias"] = np.empty(Dm) if delta_bias is not None else None
    g["dh0"] = np.empty((b, Dm, N)) if h0 is not None else None
    lib.orc_scan_bwd(b, L, Dm, N, _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D),
                     _ptr(z), _ptr(delta_bias), int(bool(delta_softplus)), _ptr(h0), _ptr(dout),
                     _ptr(g["du"]), _ptr(g["ddelta"]), _ptr(g["dA"]), _ptr(g["dB"]), _ptr(g["dC"]),
                     _ptr(g["dD"]), _ptr(g["dz"]), _ptr(g["ddelta_bias"]), _ptr(g["dh0"]))
    return {k: v for k, v in g.items() if v is not None}


def linear_scan(a, x):
    """h_t = a_t * h_{t-1} + x_t along dim 1 (h starts at 0), the reference's
    sequential_scan (models/selective_scan.py:91-99).  a, x: (b, L, ...)."""
    lib = _load()
    a, x = _arr(a), _arr(x)
    b, L = a.shape[:2]
    W = int(np.prod(a.shape[2:])) if a.ndim > 2 else 1
    h = np.empty(a.shape)
    lib.orc_linear_scan(b, L, ctypes.c_long(W), _ptr(a), _ptr(x), _ptr(h))
    return h


def linear_scan_bwd(a, h, dh):
    """Gradients (da, dx) of linear_scan for the upstream gradient dh, given its output h:
    the reverse recurrence g_t = dh_t + a_{t+1} g_{t+1}, dx = g, da_t = g_t h_{t-1}."""
    lib = _load()
    a, h, dh = _arr(a), _arr(h), _arr(dh)
    b, L = a.shape[:2]
    W = int(np.prod(a.shape[2:])) if a.ndim > 2 else 1
    da, dx = np.empty(a.shape), np.empty(a.shape)
    lib.orc_linear_scan_bwd(b, L, ctypes.c_long(W), _ptr(a), _ptr(h), _ptr(dh), _ptr(da), _ptr(dx))
    return da, dx


def conv1d_fwd(x, weight, bias=None, silu=True):
    """Causal depthwise conv1d (+SiLU).  x: (b,L,D); weight: (D,K) or (D,1,K); bias: (D,)."""
    lib = _load()
    x, weight, bias = _arr(x), _arr(weight), _arr(bias)
    weight = weight.reshape(weight.shape[0], -1)
    b, L, Dm = x.shape
    K = weight.shape[1]
    out = np.empty((b, L, Dm))
    lib.orc_conv1d_fwd(b, L, Dm, K, _ptr(x), ctypes.c_long(L * Dm), ctypes.c_long(Dm),
                       _ptr(weight), _ptr(bias), int(bool(silu)), _ptr(out))
    return out


def conv1d_bwd(x, weight, bias, dout, silu=True):
    """Returns (dx, dweight (D,K), dbias or None)."""
    lib = _load()
    x, weight, bias, dout = _arr(x), _arr(weight), _arr(bias), _arr(dout)
    weight = weight.reshape(weight.shape[0], -1)
    b, L, Dm = x.shape
    K = weight.shape[1]
    dx = np.empty((b, L, Dm))
    dw = np.empty((Dm, K))
    db = np.empty(Dm) if bias is not None else None
    lib.orc_conv1d_bwd(b, L, Dm, K, _ptr(x), ctypes.c_long(L * Dm), ctypes.c_long(Dm),
                       _ptr(weight), _ptr(bias), int(bool(silu)), _ptr(dout),
                       _ptr(dx), _ptr(dw), _ptr(db))
    return dx, dw, db


def decode_step(x, z, delta_raw, B, C, conv_w, conv_b, A, D, dt_bias, conv_state, ssm_state,
                delta_softplus=True):
    """One decode step.  Returns (out (b,D), new_conv_state, new_ssm_state, xc (b,D))."""
    lib = _load()
    x, z, delta_raw, B, C, conv_w, conv_b, A, D, dt_bias = map(
        _arr, (x, z, delta_raw, B, C, conv_w, conv_b, A, D, dt_bias))
    conv_state = _arr(conv_state).copy()
    ssm_state = _arr(ssm_state).copy()
    conv_w = conv_w.reshape(conv_w.shape[0], -1)
    b, Dm = x.shape
    N = A.shape[1]
    K = conv_w.shape[1]
    out = np.empty((b, Dm))
    xc = np.empty((b, Dm))
    lib.orc_decode_step(b, Dm, N, K, _ptr(x), _ptr(z), _ptr(delta_raw), _ptr(B), _ptr(C),
                        _ptr(conv_w), _ptr(conv_b), _ptr(A), _ptr(D), _ptr(dt_bias),
                        int(bool(delta_softplus)), _ptr(conv_state), _ptr(ssm_state),
                        _ptr(out), _ptr(xc))
    return out, conv_state, ssm_state, xc
