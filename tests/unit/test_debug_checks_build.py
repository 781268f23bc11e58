"""The debug-checks variant of the kernels compiles for sm_100a (no GPU needed):
every kernel unit builds with -DMT_DEBUG_CHECKS."""

import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
CSRC = os.path.join(ROOT, "meshtrain_b200", "ops", "csrc")


@pytest.mark.parametrize("unit", ["elementwise.cu", "cross_entropy.cu"])
def test_debug_checks_compile(unit):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    import torch

    inc = os.path.join(os.path.dirname(torch.__file__), "include")
    with tempfile.TemporaryDirectory() as tmp:
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
                            "--expt-relaxed-constexpr", "-DMT_DEBUG_CHECKS", "-I", inc, "-I", CSRC, "-c",
                            os.path.join(CSRC, unit), "-o", os.path.join(tmp, "unit.o")],
                           capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
