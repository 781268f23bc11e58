"""The debug-checks build (``ops._C_debug``, setup.py with MT_DEBUG_CHECKS=1).

Its kernels check the indices they read from data and the TMEM / TMA addresses
they form; a failed check records a code and skips the access instead of
faulting.  Correct launches must record nothing (no false positives in the GEMM
and attention kernels), and an out-of-range token id must be recorded, not
read.  Runs in a child process so the package's own extension choice is not
disturbed.
"""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import torch
from meshtrain_b200 import ops
assert ops.debug_checks_built(), "not the debug build"
ops.set_backend("custom")
torch.manual_seed(0)
dev = "cuda"
# GEMM + attention (TMA loads / stores / reduce-adds, TMEM loads / stores): nothing recorded
a = torch.randn(512, 256, device=dev).to(torch.bfloat16)
w = torch.randn(384, 256, device=dev).to(torch.bfloat16)
y = ops.linear(a, w, None)
for hd, hq, hk in ((64, 4, 4), (128, 4, 2)):
    q = torch.randn(2, 256, hq, hd, device=dev).to(torch.bfloat16)
    k, v = (torch.randn(2, 256, hk, hd, device=dev).to(torch.bfloat16) for _ in range(2))
    o, lse = ops.attention(q, k, v, causal=True)
    ops.attention_bwd(torch.randn_like(o), q, k, v, o, lse, causal=True)
torch.cuda.synchronize()
assert ops.read_status(0) == 0
clean = ops.read_checks()
assert clean == 0, f"checks fired on correct launches: {clean:#x}"
# an out-of-range token id: recorded (kErrCheckIndex), not read out of bounds
tok = torch.randn(100, 64, device=dev).to(torch.bfloat16)
ids = torch.tensor([[3, 7, 150, -2]], device=dev)
out = ops.embedding(ids, tok, None, 4)
torch.cuda.synchronize()
flags = ops.read_checks()
assert flags & (1 << 8), f"{flags:#x}"
assert ops.read_checks() == 0  # read clears
print("debug checks ok", hex(flags))
"""


def test_debug_build_records_bad_indices_and_nothing_else():
    import glob

    if not glob.glob(os.path.join(ROOT, "meshtrain_b200", "ops", "_C_debug*.so")):
        pytest.skip("debug-checks extension not built (MT_DEBUG_CHECKS=1 python setup.py build_ext --inplace)")
    env = dict(os.environ, MT_OPS_DEBUG="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "debug checks ok" in r.stdout
