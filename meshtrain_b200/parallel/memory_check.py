"""Startup memory validation of a stage that has just been materialised.

After a stage's parameters are on its device, ``validate_stage`` compares what
was actually allocated with the planner's estimate and asks whether the rest
of the estimate (gradients, optimizer state, activations) still fits in what
the device reports free.  If it does not, or if a trial allocation of that
remainder fails, it raises ``StageMemoryError``; the worker reports that as a
startup OOM and the coordinator re-plans with a smaller budget for that
worker (same behaviour as the reference, runtime/memory_check.py:29-115).

The report's keys (``capacity``, ``actual_parameters``, ``estimated_*``,
``error_before_training``, ``actual_peak_step0`` ...) travel in worker events
and run artefacts.
"""

from __future__ import annotations

import gc

import torch

GB = 1024 ** 3
PROBE_BLOCK = 256 * 1024 ** 2   # trial allocation granularity


class StageMemoryError(RuntimeError):
    """The stage cannot fit: carries the validation report for the coordinator."""

    def __init__(self, message: str, report: dict):
        super().__init__(message)
        self.report = report


_OOM_TEXT = ("out of memory", "mps backend out of memory")


def is_oom(exc: BaseException) -> bool:
    """True for allocation failures of any backend (and for StageMemoryError)."""
    oom_type = getattr(torch.cuda, "OutOfMemoryError", ())
    if isinstance(exc, (StageMemoryError,) + ((oom_type,) if oom_type else ())):
        return True
    message = str(exc).lower()
    return any(text in message for text in _OOM_TEXT)


def release_device_memory(device) -> None:
    """Returns cached allocator blocks to the device after a failed or finished stage."""
    gc.collect()
    if device.backend == "cuda":
        torch.cuda.empty_cache()
    elif device.backend == "mps":
        empty = getattr(torch.mps, "empty_cache", None)
        if empty is not None:
            empty()


def _trial_allocation(device, nbytes: int) -> None:
    """Allocates ``nbytes`` in PROBE_BLOCK pieces and frees them; raises on OOM."""
    held = []
    for offset in range(0, nbytes, PROBE_BLOCK):
        held.append(torch.empty(min(PROBE_BLOCK, nbytes - offset), dtype=torch.uint8, device=device.device))
    device.synchronize()
    del held


def validate_stage(stage, device, estimate: dict | None, *, probe: bool = True, safety_factor: float = 0.85) -> dict:
    """Checks a materialised stage against the planner's ``estimate`` (``required`` and ``parameters`` bytes)."""
    params = stage.memory_report()["parameters"]
    free = int(device.available_memory(in_use=params))
    allocated = params if device.backend == "cpu" else int(device.memory_stats().get("allocated", params))
    report = {"backend": device.backend, "actual_parameters": params, "actual_before_training": allocated,
              "available": free, "capacity": int(params + free), "probe": None}
    if not estimate:
        return report
    required, est_params = int(estimate["required"]), int(estimate["parameters"])
    rest = max(0, required - est_params)
    report.update(estimated_required=required, estimated_parameters=est_params, estimated_remaining=rest,
                  parameter_estimate_error=(params - est_params) / est_params if est_params else 0.0)
    if est_params and device.backend != "cpu":
        report["error_before_training"] = (allocated - est_params) / est_params
    budget = free * safety_factor
    if rest > budget:
        raise StageMemoryError(
            f"stage {stage.stage_index} needs ~{rest / GB:.2f} GB more after loading its {params / GB:.2f} GB "
            f"of parameters, but the {device.backend} device has only {free / GB:.2f} GB available "
            f"(safety factor {safety_factor})", report)
    if not (probe and rest and device.backend in ("cuda", "mps")):
        return report
    try:
        _trial_allocation(device, rest)
    except Exception as exc:  # noqa: BLE001 - only allocation failures become a memory error
        if not is_oom(exc):
            raise
        report["probe"] = "oom"
        release_device_memory(device)
        first_line = str(exc).splitlines()[0][:160] if str(exc) else type(exc).__name__
        raise StageMemoryError(f"probe allocation of {rest / GB:.2f} GB failed on {device.backend}: {first_line}",
                               report) from exc
    report["probe"] = "ok"
    release_device_memory(device)
    return report


def validate_engine(engine, device, estimate: dict | None, *, probe: bool = True,
                    safety_factor: float = 0.85) -> dict:
    """Startup check of a device-engine stage, whose flat buffers exist from construction.

    The engine allocates its bf16 weights, fp32 gradients and (unless offloaded) fp32 master
    weights and Adam moments up front, so what remains of the planner's estimate is the
    step's working memory: saved activations, boundary buffers and workspace.  That rest
    must fit in what the device reports free (times ``safety_factor``), or a trial
    allocation of it must succeed on an accelerator; otherwise ``StageMemoryError`` is
    raised and the coordinator re-plans with a smaller budget for this worker.
    """
    slots = engine.offload.device_bytes() if getattr(engine, "offload", None) is not None else 0
    resident = int(engine.flat.device_bytes() + slots)  # flat buffers + the offload slot ring
    free = int(device.available_memory(in_use=resident))
    params = int(engine.flat.bytes_by_role()["parameter"])
    report = {"backend": device.backend, "engine": "device", "actual_parameters": params,
              "actual_before_training": resident, "available": free, "capacity": resident + free, "probe": None}
    if not estimate:
        return report
    required = int(estimate["required"])
    est_resident = sum(int(estimate.get(key) or 0) for key in ("parameters", "gradients", "master_weights",
                                                              "optimizer_state"))
    est_params = int(estimate["parameters"])
    rest = max(0, required - est_resident)
    report.update(estimated_required=required, estimated_parameters=est_params, estimated_resident=est_resident,
                  estimated_remaining=rest,
                  parameter_estimate_error=(params - est_params) / est_params if est_params else 0.0,
                  error_before_training=(resident - est_resident) / est_resident if est_resident else 0.0)
    if free <= 0 or rest > free * safety_factor:
        raise StageMemoryError(
            f"stage {engine.stage} holds {resident / GB:.2f} GB of weights, gradients and optimizer state and "
            f"needs ~{rest / GB:.2f} GB more for a step, but the {device.backend} device has only "
            f"{free / GB:.2f} GB available (safety factor {safety_factor})", report)
    if probe and rest and device.backend in ("cuda", "mps"):
        try:
            _trial_allocation(device, rest)
        except Exception as exc:  # noqa: BLE001 - only allocation failures become a memory error
            if not is_oom(exc):
                raise
            report["probe"] = "oom"
            release_device_memory(device)
            raise StageMemoryError(f"probe allocation of {rest / GB:.2f} GB failed on {device.backend}",
                                   report) from exc
        report["probe"] = "ok"
        release_device_memory(device)
    return report


def format_validation(report: dict) -> str:
    """One line for logs: estimate vs. measured parameters, load and first-step peak."""
    gb = lambda key: report[key] / GB  # noqa: E731
    if "estimated_required" not in report:
        return f"actual parameters {gb('actual_parameters'):.2f} GB, available {gb('available'):.2f} GB"
    pieces = [f"estimated = {gb('estimated_required'):.2f} GB",
              f"parameters estimated {gb('estimated_parameters'):.2f} GB vs actual {gb('actual_parameters'):.2f} GB "
              f"({report['parameter_estimate_error']:+.1%})"]
    optional = (("error_before_training", "actual_before_training", "error vs estimated parameters"),
                ("peak_estimate_error", "actual_peak_step0", "error vs estimate"))
    labels = {"actual_before_training": "actual_before_training", "actual_peak_step0": "actual peak (first step)"}
    for err_key, value_key, what in optional:
        if err_key in report and value_key in report:
            pieces.append(f"{labels[value_key]} = {gb(value_key):.2f} GB ({what} {report[err_key]:+.1%})")
    return ", ".join(pieces)
