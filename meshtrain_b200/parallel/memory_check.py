"""Runtime memory validation of a freshly materialised stage.

Compares the measured parameter bytes and free device memory with the
planner's estimate; raises ``StageMemoryError`` (classified as a startup OOM,
which triggers replanning) when the rest of the estimate cannot fit, and can
probe-allocate the estimated remainder once in 256 MiB blocks (reference
runtime/memory_check.py:29-115).
"""

from __future__ import annotations

import gc

import torch

GB = 1024 ** 3
PROBE_BLOCK = 256 * 1024 ** 2


class StageMemoryError(RuntimeError):
    def __init__(self, message: str, report: dict):
        super().__init__(message)
        self.report = report


def is_oom(exc: BaseException) -> bool:
    if isinstance(exc, StageMemoryError):
        return True
    oom = getattr(torch.cuda, "OutOfMemoryError", None)
    if oom is not None and isinstance(exc, oom):
        return True
    text = str(exc).lower()
    return "out of memory" in text or "mps backend out of memory" in text


def release_device_memory(device) -> None:
    gc.collect()
    if device.backend == "cuda":
        torch.cuda.empty_cache()
    elif device.backend == "mps" and hasattr(torch.mps, "empty_cache"):
        torch.mps.empty_cache()


def validate_stage(stage, device, estimate: dict | None, *, probe: bool = True, safety_factor: float = 0.85) -> dict:
    held = stage.memory_report()
    params = held["parameters"]
    available = device.available_memory(in_use=params)
    stats = device.memory_stats()
    before = int(stats.get("allocated", params)) if device.backend != "cpu" else params
    report = {"backend": device.backend, "actual_parameters": params, "actual_before_training": before,
              "available": int(available), "capacity": int(params + available), "probe": None}
    if not estimate:
        return report
    est_req, est_params = int(estimate["required"]), int(estimate["parameters"])
    remaining = max(0, est_req - est_params)
    report.update(estimated_required=est_req, estimated_parameters=est_params, estimated_remaining=remaining,
                  parameter_estimate_error=(params - est_params) / est_params if est_params else 0.0)
    if device.backend != "cpu" and est_params:
        report["error_before_training"] = (before - est_params) / est_params
    if remaining > available * safety_factor:
        raise StageMemoryError(
            f"stage {stage.stage_index} needs ~{remaining / GB:.2f} GB more after loading its {params / GB:.2f} GB "
            f"of parameters, but the {device.backend} device has only {available / GB:.2f} GB available "
            f"(safety factor {safety_factor})", report)
    if probe and device.backend in ("cuda", "mps") and remaining > 0:
        try:
            blocks = [torch.empty(min(remaining - i, PROBE_BLOCK), dtype=torch.uint8, device=device.device)
                      for i in range(0, remaining, PROBE_BLOCK)]
            device.synchronize()
            report["probe"] = "ok"
            del blocks
        except Exception as exc:  # noqa: BLE001
            if not is_oom(exc):
                raise
            report["probe"] = "oom"
            release_device_memory(device)
            raise StageMemoryError(f"probe allocation of {remaining / GB:.2f} GB failed on {device.backend}: "
                                   f"{str(exc).splitlines()[0][:160]}", report) from exc
        release_device_memory(device)
    return report


def format_validation(report: dict) -> str:
    if "estimated_required" not in report:
        return f"actual parameters {report['actual_parameters'] / GB:.2f} GB, available {report['available'] / GB:.2f} GB"
    parts = [f"estimated = {report['estimated_required'] / GB:.2f} GB",
             f"parameters estimated {report['estimated_parameters'] / GB:.2f} GB vs actual "
             f"{report['actual_parameters'] / GB:.2f} GB ({report['parameter_estimate_error']:+.1%})"]
    if "error_before_training" in report:
        parts.append(f"actual_before_training = {report['actual_before_training'] / GB:.2f} GB "
                     f"(error vs estimated parameters {report['error_before_training']:+.1%})")
    if "actual_peak_step0" in report:
        parts.append(f"actual peak (first step) = {report['actual_peak_step0'] / GB:.2f} GB "
                     f"(error vs estimate {report['peak_estimate_error']:+.1%})")
    return ", ".join(parts)
