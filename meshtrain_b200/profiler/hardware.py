"""What a worker reports at registration: host, RAM, accelerators, capability tags
(reference profiler/hardware.py:14-83).  B200s report their SM count and NVLink peers.
"""

from __future__ import annotations

import os
import platform
import socket

import psutil
import torch

MIN_USEFUL_ACCELERATOR_BYTES = 1 * 1024 ** 3


def platform_name() -> str:
    s = platform.system().lower()
    return {"darwin": "macos"}.get(s, s)


def detect_accelerators() -> list[dict]:
    accs = []
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            peers = [j for j in range(n) if j != i and torch.cuda.can_device_access_peer(i, j)]
            accs.append({"backend": "cuda", "index": i, "name": p.name, "memory_total": int(p.total_memory),
                         "compute_capability": f"{p.major}.{p.minor}", "sm_count": p.multi_processor_count,
                         "unified_memory": False, "usable": p.total_memory >= MIN_USEFUL_ACCELERATOR_BYTES,
                         "p2p_peers": peers})
    if getattr(torch.backends, "mps", None) is not None and torch.backends.mps.is_available():
        total = psutil.virtual_memory().total
        rec = getattr(torch.mps, "recommended_max_memory", None)
        if rec is not None:
            try:
                total = int(rec())
            except RuntimeError:
                pass
        accs.append({"backend": "mps", "index": 0, "name": f"Apple {platform.machine()}", "memory_total": int(total),
                     "unified_memory": True, "usable": True})
    return accs


def detect_hardware() -> dict:
    accs = detect_accelerators()
    caps = ["cpu", "float32", "float64"] + [a["backend"] for a in accs if a["usable"]]
    if any(a["backend"] == "cuda" and a["usable"] for a in accs):
        caps += ["float16", "bfloat16" if torch.cuda.is_bf16_supported() else "no-bfloat16"]
        if any(a.get("compute_capability") == "10.0" for a in accs):
            caps.append("sm_100")
        if any(a.get("p2p_peers") for a in accs):
            caps.append("nvlink_p2p")
    if any(a["backend"] == "mps" for a in accs):
        caps += ["float16", "unified_memory"]
    vm = psutil.virtual_memory()
    return {"hostname": socket.gethostname(), "platform": platform_name(), "machine": platform.machine(),
            "python": platform.python_version(), "torch": torch.__version__, "cpu_count": os.cpu_count() or 1,
            "ram_total": int(vm.total), "ram_available": int(vm.available), "accelerators": accs,
            "capabilities": sorted(set(caps))}


def primary_backend(hw: dict) -> str:
    for backend in ("cuda", "mps"):
        if any(a["backend"] == backend and a.get("usable", True) for a in hw.get("accelerators", [])):
            return backend
    return "cpu"
