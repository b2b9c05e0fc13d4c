"""ctypes binding of the C ABI declared in include/swiftx_b200.h.

The shared library is built in-tree (swiftx_b200/libswiftx_b200.so).  Loading
fails loudly if it is missing: there is no CPU or eager fallback behind it.
"""
import ctypes
import os

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libswiftx_b200.so")

SWX_OK = 0
SWX_ERR_INVALID_ARG = 1
SWX_ERR_UNSUPPORTED = 2
SWX_ERR_CUDA = 3
SWX_ERR_TIMEOUT = 4
SWX_MAX_GROUPS = 8
SWX_SCAN_SPLIT_FWD = 2
SWX_DECODE_MAX_DT_RANK = 256
# capacity of the static scratch of swx_scan_bwd_static_scratch (SWX_STATIC_SCRATCH_BYTES)
SWX_STATIC_SCRATCH_BYTES = 8 << 20

# swx_scan_args.flags: A holds log(-A) (SWX_SCAN_A_LOG)
SWX_SCAN_A_LOG = 1

SWX_DTYPE_F64 = 2
DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float64: SWX_DTYPE_F64}

i64 = ctypes.c_int64
i32 = ctypes.c_int32
vp = ctypes.c_void_p


class ScanArgs(ctypes.Structure):
    """Mirror of ``swx_scan_args``."""
    _fields_ = [
        ("batch", i64), ("seqlen", i64), ("dim", i64), ("dstate", i64),
        ("in_dtype", i32), ("out_dtype", i32), ("delta_softplus", i32), ("flags", i32),
        ("u", vp), ("u_sb", i64), ("u_sl", i64),
        ("delta", vp), ("delta_sb", i64), ("delta_sl", i64),
        ("z", vp), ("z_sb", i64), ("z_sl", i64),
        ("B", vp), ("B_sb", i64), ("B_sl", i64),
        ("C", vp), ("C_sb", i64), ("C_sl", i64),
        ("A", vp), ("Dskip", vp), ("delta_bias", vp), ("h0", vp),
        ("out", vp), ("h_last", vp), ("checkpoints", vp),
        ("dout", vp), ("dout_sb", i64), ("dout_sl", i64),
        ("du", vp), ("ddelta", vp), ("dz", vp), ("dB", vp), ("dC", vp),
        ("dA", vp), ("dD", vp), ("ddelta_bias", vp), ("dh0", vp),
        ("workspace", vp), ("workspace_bytes", i64),
        ("delta_sum", vp),
        ("out_pre", vp),
        ("group_w", vp), ("group_w_sb", i64), ("group_w_sl", i64),
        ("group_of", vp), ("ngroups", i32), ("d_group_w", vp),
        ("dz_sb", i64), ("dz_sl", i64),
    ]


class ConvArgs(ctypes.Structure):
    """Mirror of ``swx_conv_args``."""
    _fields_ = [
        ("batch", i64), ("seqlen", i64), ("dim", i64), ("width", i64),
        ("dtype", i32), ("silu", i32),
        ("x", vp), ("x_sb", i64), ("x_sl", i64),
        ("weight", vp), ("bias", vp), ("out", vp),
        ("dout", vp), ("dout_sb", i64), ("dout_sl", i64),
        ("dx", vp), ("dweight", vp), ("dbias", vp),
        ("workspace", vp), ("workspace_bytes", i64),
        ("dx_sb", i64), ("dx_sl", i64),
    ]


SWX_DECODE_CONV = 1
SWX_DECODE_SSM = 2
SWX_DECODE_A_LOG = 1      # swx_decode_args.flags: A holds log(-A)


class DecodeArgs(ctypes.Structure):
    """Mirror of ``swx_decode_args``."""
    _fields_ = [
        ("batch", i64), ("dim", i64), ("dstate", i64), ("width", i64),
        ("delta_softplus", i32), ("mode", i32),
        ("x", vp), ("x_sb", i64), ("z", vp), ("z_sb", i64),
        ("delta", vp), ("delta_sb", i64), ("B", vp), ("B_sb", i64), ("C", vp), ("C_sb", i64),
        ("conv_weight", vp), ("conv_bias", vp), ("A", vp), ("Dskip", vp), ("delta_bias", vp),
        ("conv_state", vp), ("ssm_state", vp), ("xc_out", vp), ("out", vp),
        ("flags", i32), ("reserved", i32),
        ("group_w", vp), ("group_w_sb", i64), ("group_of", vp), ("ngroups", i32), ("reserved2", i32),
        ("dt_in", vp), ("dt_in_sb", i64), ("dt_weight", vp), ("dt_rank", i32), ("reserved3", i32),
        ("xproj_weight", vp), ("xproj_rows", i32), ("reserved4", i32), ("workspace", vp), ("workspace_bytes", i64),
    ]


class LinearScanArgs(ctypes.Structure):
    """Mirror of ``swx_linear_scan_args``."""
    _fields_ = [
        ("batch", i64), ("seqlen", i64), ("width", i64), ("dtype", i32), ("reserved", i32),
        ("a", vp), ("a_sb", i64), ("a_sl", i64), ("x", vp), ("x_sb", i64), ("x_sl", i64),
        ("h", vp), ("dh", vp), ("dh_sb", i64), ("dh_sl", i64), ("da", vp), ("dx", vp),
    ]


class RMSNormArgs(ctypes.Structure):
    """Mirror of ``swx_rmsnorm_args``."""
    _fields_ = [
        ("rows", i64), ("dim", i64), ("eps", ctypes.c_float), ("dtype", i32), ("out_dtype", i32),
        ("res_dtype", i32), ("x", vp), ("weight", vp), ("y", vp), ("rstd", vp), ("dy", vp), ("dx", vp), ("dweight", vp),
        ("workspace", vp), ("workspace_bytes", i64), ("residual", vp), ("sum", vp), ("dsum", vp), ("dres", vp),
    ]


class EmbeddingArgs(ctypes.Structure):
    """Mirror of ``swx_embedding_args``."""
    _fields_ = [
        ("ntok", i64), ("vocab", i64), ("dim", i64), ("idx", vp), ("dy", vp), ("dweight", vp),
        ("status", vp), ("workspace", vp), ("workspace_bytes", i64),
    ]


_lib = None


def load():
    """Load the kernel library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"swiftx_b200 kernel library not found at {LIB_PATH}; build it with "
            "`python -m swiftx_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.swx_abi_version.restype = ctypes.c_int
    lib.swx_status_string.restype = ctypes.c_char_p
    lib.swx_status_string.argtypes = [ctypes.c_int]
    for fn, st in (("swx_scan_args_size", ScanArgs), ("swx_conv_args_size", ConvArgs),
                   ("swx_decode_args_size", DecodeArgs), ("swx_linear_scan_args_size", LinearScanArgs),
                   ("swx_rmsnorm_args_size", RMSNormArgs), ("swx_embedding_args_size", EmbeddingArgs)):
        getattr(lib, fn).restype = i64
        if getattr(lib, fn)() != ctypes.sizeof(st):
            raise RuntimeError(f"{st.__name__} layout mismatch between the library and its binding")
    lib.swx_scan_checkpoint_floats.restype = i64
    lib.swx_scan_checkpoint_floats.argtypes = [i64, i64, i64]
    for fn in ("swx_scan_bwd_workspace_bytes", "swx_scan_bwd_workspace_bytes_f64", "swx_scan_correct_workspace_bytes"):
        getattr(lib, fn).restype = i64
        getattr(lib, fn).argtypes = [i64, i64, i64]
    for name, st in (("swx_scan_fwd", ScanArgs), ("swx_scan_bwd", ScanArgs),
                     ("swx_scan_bwd_static_scratch", ScanArgs), ("swx_scan_correct", ScanArgs),
                     ("swx_conv1d_fwd", ConvArgs),
                     ("swx_conv1d_bwd", ConvArgs), ("swx_decode_step", DecodeArgs),
                     ("swx_linear_scan_fwd", LinearScanArgs), ("swx_linear_scan_bwd", LinearScanArgs),
                     ("swx_rmsnorm_fwd", RMSNormArgs), ("swx_rmsnorm_bwd", RMSNormArgs),
                     ("swx_embedding_bwd", EmbeddingArgs)):
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.POINTER(st), vp]
    lib.swx_scan_bwd_ctas_per_sm.restype = ctypes.c_int
    lib.swx_scan_bwd_ctas_per_sm.argtypes = [ctypes.POINTER(ScanArgs)]
    lib.swx_scan_bwd_segments.restype = ctypes.c_int
    lib.swx_scan_bwd_segments.argtypes = [ctypes.POINTER(ScanArgs)]
    lib.swx_exp2_fma_eval.restype = ctypes.c_int
    lib.swx_exp2_fma_eval.argtypes = [vp, vp, i64, vp]
    lib.swx_scan_fwd_workspace_bytes.restype = i64
    lib.swx_scan_fwd_workspace_bytes.argtypes = [ctypes.POINTER(ScanArgs)]
    lib.swx_decode_layer_step.restype = ctypes.c_int
    lib.swx_decode_layer_step.argtypes = [ctypes.POINTER(DecodeArgs), vp]
    lib.swx_decode_layer_workspace_bytes.restype = i64
    lib.swx_decode_layer_workspace_bytes.argtypes = [i64, i64, i64]
    lib.swx_device_wait_status.restype = ctypes.c_int
    lib.swx_device_wait_status.argtypes = []
    lib.swx_diag_wait_timeout.restype = ctypes.c_int
    lib.swx_diag_wait_timeout.argtypes = [ctypes.c_uint32, vp]
    lib.swx_rmsnorm_bwd_workspace_bytes.restype = i64
    lib.swx_rmsnorm_bwd_workspace_bytes.argtypes = [i64]
    lib.swx_embedding_bwd_workspace_bytes.restype = i64
    lib.swx_embedding_bwd_workspace_bytes.argtypes = [i64, i64, i64]
    lib.swx_conv1d_bwd_workspace_bytes.restype = i64
    lib.swx_conv1d_bwd_workspace_bytes.argtypes = [i64, i64, i64, i64]
    _lib = lib
    return lib


def check(status, what):
    """Turn a nonzero status into an exception, in the reference's RuntimeError style
    (models/triton_scan.py:160-161); argument errors become ValueError."""
    if status == SWX_OK:
        return
    msg = load().swx_status_string(status).decode()
    if status in (SWX_ERR_INVALID_ARG, SWX_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {status})")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
