"""Drop-in for the reference's models/triton_scan.py on B200.

``selective_scan_triton(u, delta, A, B, C, D=None, chunk=64)`` keeps the reference
signature (models/triton_scan.py:158-162) and runs the hand-written sm_100a kernel
(no Triton).  ``HAS_TRITON`` keeps its meaning for callers -- "the fused GPU scan is
available" -- and is True exactly when the kernel library loads.
"""
from . import _lib
from .selective_scan import selective_scan_fn

try:
    _lib.load()
    HAS_TRITON = True
except RuntimeError:          # library not built
    HAS_TRITON = False


def selective_scan_triton(u, delta, A, B, C, D=None, chunk=64):
    """Same contract as selective_scan_ref: u, delta (b,L,D); A (D,N); B, C (b,L,N); D (D,)."""
    if not HAS_TRITON:
        raise RuntimeError("the swiftx_b200 kernel library is not built")
    return selective_scan_fn(u, delta, A, B, C, D)
