"""The hardware description a worker sends when it registers.

``detect_hardware()`` returns host facts (hostname, platform, CPUs, RAM, torch
version), one record per accelerator, and a sorted list of capability tags the
planner filters on.  Accelerator records come from one probe function per
backend; CUDA devices also report their SM count and which local GPUs they can
reach peer-to-peer (NVLink / NVSwitch on a B200 box), which the coordinator
uses to give stages of one box NCCL links.  Same fields as the reference's
registration record (profiler/hardware.py:14-83).
"""

from __future__ import annotations

import os
import platform
import socket

import psutil
import torch

MIN_USEFUL_ACCELERATOR_BYTES = 1 * 1024 ** 3


def platform_name() -> str:
    system = platform.system().lower()
    return "macos" if system == "darwin" else system


def _cuda_accelerators() -> list[dict]:
    if not torch.cuda.is_available():
        return []
    count = torch.cuda.device_count()
    records = []
    for i in range(count):
        props = torch.cuda.get_device_properties(i)
        records.append({
            "backend": "cuda", "index": i, "name": props.name, "memory_total": int(props.total_memory),
            "compute_capability": f"{props.major}.{props.minor}", "sm_count": props.multi_processor_count,
            "unified_memory": False, "usable": props.total_memory >= MIN_USEFUL_ACCELERATOR_BYTES,
            "p2p_peers": [j for j in range(count) if j != i and torch.cuda.can_device_access_peer(i, j)],
        })
    return records


def _mps_accelerators() -> list[dict]:
    mps = getattr(torch.backends, "mps", None)
    if mps is None or not mps.is_available():
        return []
    budget = psutil.virtual_memory().total
    limit = getattr(torch.mps, "recommended_max_memory", None)
    if limit is not None:
        try:
            budget = int(limit())
        except RuntimeError:
            pass
    return [{"backend": "mps", "index": 0, "name": f"Apple {platform.machine()}", "memory_total": int(budget),
             "unified_memory": True, "usable": True}]


ACCELERATOR_PROBES = (_cuda_accelerators, _mps_accelerators)


def detect_accelerators() -> list[dict]:
    return [record for probe in ACCELERATOR_PROBES for record in probe()]


def capability_tags(accelerators: list[dict]) -> list[str]:
    """Planner-facing tags: backends, dtypes, sm_100, NVLink peer access, unified memory."""
    usable = [a for a in accelerators if a.get("usable", True)]
    tags = {"cpu", "float32", "float64"} | {a["backend"] for a in usable}
    cuda = [a for a in usable if a["backend"] == "cuda"]
    if cuda:
        tags.add("float16")
        tags.add("bfloat16" if torch.cuda.is_bf16_supported() else "no-bfloat16")
        if any(a.get("compute_capability") == "10.0" for a in cuda):
            tags.add("sm_100")
        if any(a.get("p2p_peers") for a in cuda):
            tags.add("nvlink_p2p")
    if any(a["backend"] == "mps" for a in accelerators):
        tags |= {"float16", "unified_memory"}
    return sorted(tags)


def detect_hardware() -> dict:
    accelerators = detect_accelerators()
    vm = psutil.virtual_memory()
    return {"hostname": socket.gethostname(), "platform": platform_name(), "machine": platform.machine(),
            "python": platform.python_version(), "torch": torch.__version__, "cpu_count": os.cpu_count() or 1,
            "ram_total": int(vm.total), "ram_available": int(vm.available), "accelerators": accelerators,
            "capabilities": capability_tags(accelerators)}


def primary_backend(hw: dict) -> str:
    """The backend a worker should run on: CUDA, then MPS, then CPU."""
    present = {a["backend"] for a in hw.get("accelerators", []) if a.get("usable", True)}
    return next((b for b in ("cuda", "mps") if b in present), "cpu")
