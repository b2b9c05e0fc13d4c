"""The reference's own CPU test suite through the device-dispatching patch.

swiftx_b200.integrate.patch_reference_module is what a maintainer appends to the
reference's models/selective_scan.py to switch it over.  This test
copies the reference's models/ and tests/ to a temporary folder, appends those two
lines, and runs the reference's tests for the scan, the block and the model
(tests/test_selective_scan.py, test_sift_block.py, test_model.py) on CPU tensors: they
must pass unchanged, because CPU tensors keep the reference's own code.  Skipped where
the reference checkout is not available (set SWIFTX_REFERENCE to point at one).
"""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("SWIFTX_REFERENCE", "/root/reference")
PATCH = "\nfrom swiftx_b200.integrate import patch_reference_module\npatch_reference_module(globals())\n"


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "models")), reason="reference checkout not available")
def test_reference_cpu_suite_passes_with_patch(tmp_path):
    for d in ("models", "tests"):
        shutil.copytree(os.path.join(REF, d), tmp_path / d, ignore=shutil.ignore_patterns("__pycache__"))
    shutil.copy(os.path.join(REF, "pytest.ini"), tmp_path / "pytest.ini")
    with open(tmp_path / "models" / "selective_scan.py", "a") as f:
        f.write(PATCH)
    env = dict(os.environ, PYTHONPATH=f"{tmp_path}{os.pathsep}{ROOT}", CUDA_VISIBLE_DEVICES="")
    probe = subprocess.run([sys.executable, "-c", "import models.selective_scan as m; "
                            "print(m.selective_scan_fast.__swiftx_original__.__module__)"],
                           cwd=tmp_path, env=env, capture_output=True, text=True)
    assert probe.returncode == 0 and probe.stdout.strip() == "models.selective_scan", probe.stderr
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                        "tests/test_selective_scan.py", "tests/test_sift_block.py", "tests/test_model.py"],
                       cwd=tmp_path, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout
