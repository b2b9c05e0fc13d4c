"""swiftx_b200: B200-native selective-scan hot path of the Sift (Mamba-1) model.

Public entry points mirror the reference (BhanuPrakash6640/SwiftX) modules:
models/selective_scan.py -> swiftx_b200.selective_scan,
models/triton_scan.py    -> swiftx_b200.triton_scan.
"""
from .selective_scan import (  # noqa: F401
    LinearScanFn,
    SelectiveScanFn,
    parallel_scan,
    scan_backward,
    scan_forward,
    selective_scan_fast,
    selective_scan_fn,
    selective_scan_ref,
    sequential_scan,
)

__version__ = "0.1.0"
