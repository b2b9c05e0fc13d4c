"""patch_reference_module on CUDA tensors: the patched names run the sm_100a kernels,
float64 included, while CPU tensors reach the original functions untouched.  The
originals here are stand-ins that record their calls (the reference itself does not
travel with the repository)."""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200.integrate import patch_reference_module
from swiftx_b200.workloads import reference_test_inputs

pytestmark = pytest.mark.gpu


def test_patched_names_dispatch_by_device():
    calls = []

    def original(name):
        def fn(*a, **k):
            calls.append(name)
            return "reference"
        return fn

    ns = {n: original(n) for n in ("selective_scan_fast", "selective_scan_ref", "parallel_scan",
                                   "sequential_scan")}
    assert sorted(patch_reference_module(ns)) == sorted(ns)
    patch_reference_module(ns)                        # idempotent
    u, delta, A, B, C, Dsk = reference_test_inputs(2, 9, 3, 4, seed=3)
    assert ns["selective_scan_fast"](u, delta, A, B, C, Dsk, mode="fused") == "reference"
    assert ns["parallel_scan"](torch.rand(2, 5, 3), torch.randn(2, 5, 3)) == "reference"
    assert calls == ["selective_scan_fast", "parallel_scan"]
    for dt in (torch.float32, torch.float64):
        cu = [t.to("cuda", dt) for t in (u, delta, A, B, C, Dsk)]
        y = ns["selective_scan_fast"](*cu, mode="fused")
        assert isinstance(y, torch.Tensor) and y.is_cuda and y.dtype == dt
        y2 = ns["selective_scan_ref"](*cu)
        want = oracle.scan_fwd(*(t.double().numpy() for t in (u, delta, A, B, C)), D=Dsk.double().numpy())
        tol = 1e-9 if dt == torch.float64 else 1e-4
        np.testing.assert_allclose(y.double().cpu().numpy(), want, rtol=tol, atol=tol)
        np.testing.assert_allclose(y2.double().cpu().numpy(), want, rtol=tol, atol=tol)
    a, x = torch.rand(2, 33, 3, 2, device="cuda"), torch.randn(2, 33, 3, 2, device="cuda")
    h = ns["sequential_scan"](a, x)
    np.testing.assert_allclose(h.cpu().numpy(), oracle.linear_scan(a.cpu(), x.cpu()), rtol=1e-5, atol=1e-5)
    assert calls == ["selective_scan_fast", "parallel_scan"]     # CUDA calls never reached them
