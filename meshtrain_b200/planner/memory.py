"""Per-stage device memory estimate (reference planner/memory.py:9-185, extended).

Components for a stage with parameter bytes P on a device of T bytes:

    usable               = T * safety_factor[backend] - framework_reserve[backend]  (capped by live free)
    parameters           = P
    gradients            = P                (autograd engine)  |  2P fp32 (device engine, bf16 params)
    master_weights       = 0                (autograd)         |  2P fp32 copy (device engine)
    optimizer_state      = k * P, k = 2 for Adam (autograd)    |  4P: two fp32 moments (device engine)
    optimizer_step_temp  = P (torch foreach Adam)               |  0 (fused single-launch Adam)
    saved_activations    = in_flight * sum(saved bytes) * activation_safety
    input/output buffers = in_flight * boundary bytes (+ 2 input-gradient buffers)
    transport_buffers    = 2 * boundary (CPU stages share host memory with the pool)
    temporary_workspace  = 2 * max output bytes + max per-layer saved bytes

in_flight = 1 on the last stage, M under GPipe, min(S - s, M, cap) under 1F1B.
With ``offload`` the fp32 masters and Adam moments live in pinned host RAM and
drop out of the device total (``host_offload`` reports them).
B200 defaults: safety 0.92 of 180 GB HBM3e, 2 GB framework reserve (CUDA
context, NCCL buffers, cuBLAS-free kernels need no workspace).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

GB = 1024 ** 3
OPTIMIZER_STATE_FACTOR = {"sgd": 0.0, "adam": 2.0, "adamw": 2.0}
OPTIMIZER_TEMP_FACTOR = {"sgd": 0.0, "adam": 1.0, "adamw": 1.0}
DEFAULT_SAFETY_FACTOR = {"cuda": 0.85, "mps": 0.80, "cpu": 0.85}
DEFAULT_FRAMEWORK_RESERVE = {"cuda": int(0.4 * GB), "mps": 0, "cpu": int(0.25 * GB)}
B200_SAFETY_FACTOR = 0.92
B200_FRAMEWORK_RESERVE = int(2.0 * GB)


@dataclass
class MemoryEstimate:
    total: int
    usable: int
    parameters: int
    gradients: int
    optimizer_state: int
    optimizer_step_temporary: int = 0
    master_weights: int = 0
    saved_activations: int = 0
    input_buffers: int = 0
    output_buffers: int = 0
    transport_buffers: int = 0
    temporary_workspace: int = 0
    framework_reserve: int = 0
    host_staging: int = 0
    host_offload: int = 0
    in_flight: int = 1
    available: int | None = None

    COMPONENTS = ("parameters", "gradients", "optimizer_state", "optimizer_step_temporary", "master_weights",
                  "saved_activations", "input_buffers", "output_buffers", "transport_buffers", "temporary_workspace")

    @property
    def required(self) -> int:
        return sum(getattr(self, k) for k in self.COMPONENTS)

    @property
    def budget(self) -> int:
        return self.usable

    @property
    def reserved(self) -> int:
        return self.total - self.usable

    @property
    def fits(self) -> bool:
        return self.required <= self.usable

    def to_dict(self) -> dict:
        return {**asdict(self), "required": self.required, "budget": self.budget, "reserved": self.reserved,
                "fits": self.fits}

    def format(self, worker: str, unified: bool = False) -> str:
        gb = lambda n: f"{n / GB:8.2f} GB"  # noqa: E731
        rows = [("total accelerator memory" + ("*" if unified else ""), self.total)]
        if self.available is not None:
            rows.append(("available (live, incl. cache)", self.available))
        rows.append(("usable (after safety/framework)", self.usable))
        rows += [(k.replace("_", " "), getattr(self, k)) for k in self.COMPONENTS if getattr(self, k)]
        rows += [("required", self.required), ("free after plan", self.usable - self.required)]
        out = [f"Worker: {worker}"] + [f"    {k:<34}{gb(v)}" for k, v in rows]
        if self.host_staging:
            out.append(f"    {'host staging (pinned RAM)':<34}{gb(self.host_staging)}")
        if self.host_offload:
            out.append(f"    {'offloaded to host (pinned RAM)':<34}{gb(self.host_offload)}")
        if unified:
            out.append("    * unified memory shared with the OS")
        return "\n".join(out)


def reserved_bytes(total: int, headroom_fraction: float, headroom_min_bytes: int) -> int:
    return int(max(total * headroom_fraction, headroom_min_bytes))


def in_flight_microbatches(schedule: str, stage_index: int, num_stages: int, num_microbatches: int,
                           max_inflight: int | None = None) -> int:
    if stage_index >= num_stages - 1:
        return 1
    if schedule == "1f1b":
        cap = num_microbatches if max_inflight is None else max_inflight
        return max(1, min(num_stages - stage_index, num_microbatches, cap))
    return num_microbatches


def estimate_stage_memory(layers, *, total: int, optimizer: str, num_microbatches: int, is_last: bool,
                          stage_index: int | None = None, num_stages: int | None = None, schedule: str = "gpipe",
                          max_inflight: int | None = None, backend: str = "cuda", safety_factor: float | None = None,
                          framework_reserve: int | None = None, headroom_fraction: float | None = None,
                          headroom_min_bytes: int | None = None, activation_safety: float = 1.25,
                          available: int | None = None, engine: str = "autograd",
                          param_dtype_bytes: int = 4, offload: bool = False) -> MemoryEstimate:
    """``engine``: "autograd" (torch optimizers, reference accounting) or "device" (flat fp32
    master/grad/Adam buffers of the GPU engine)."""
    if num_stages is None:
        num_stages, stage_index = (1, 0) if is_last else (2, 0)
    stage_index = stage_index if stage_index is not None else (num_stages - 1 if is_last else 0)
    P = sum(l.param_bytes for l in layers)
    in_flight = 1 if is_last else in_flight_microbatches(schedule, stage_index, num_stages, num_microbatches,
                                                         max_inflight)
    saved = sum(l.saved_bytes for l in layers)
    in_bytes, out_bytes = layers[0].input_bytes, layers[-1].activation_bytes
    boundary = max(in_bytes, out_bytes)
    if headroom_fraction is not None or headroom_min_bytes is not None:
        usable = int(total) - reserved_bytes(total, headroom_fraction or 0.0, headroom_min_bytes or 0)
        fw = 0
    else:
        sf = DEFAULT_SAFETY_FACTOR.get(backend, 0.85) if safety_factor is None else safety_factor
        fw = DEFAULT_FRAMEWORK_RESERVE.get(backend, 0) if framework_reserve is None else framework_reserve
        usable = int(total * sf) - fw
    if available is not None:
        usable = max(0, min(usable, int(available)))
    if engine == "device":
        n = P // max(1, param_dtype_bytes)          # parameter count
        grads = 4 * n
        master = 0 if param_dtype_bytes == 4 else 4 * n
        opt_state = int(n * 4 * OPTIMIZER_STATE_FACTOR[optimizer])
        temp = 0
        host = 0
        if offload:
            host = master + opt_state
            master, opt_state = 0, 0
    else:
        grads = P
        master = 0
        opt_state = int(P * OPTIMIZER_STATE_FACTOR[optimizer])
        temp = int(P * OPTIMIZER_TEMP_FACTOR[optimizer])
        host = 0
    return MemoryEstimate(
        total=int(total), usable=usable, parameters=P, gradients=grads, optimizer_state=opt_state,
        optimizer_step_temporary=temp, master_weights=master,
        saved_activations=int(in_flight * saved * activation_safety),
        input_buffers=in_flight * in_bytes,
        output_buffers=(0 if is_last else in_flight * out_bytes) + 2 * in_bytes,
        transport_buffers=2 * boundary if backend == "cpu" else 0,
        temporary_workspace=2 * max(l.activation_bytes for l in layers) + max(l.saved_bytes for l in layers),
        framework_reserve=fw,
        host_staging=0 if backend == "cpu" or engine == "device" else (in_flight + 2) * boundary,
        host_offload=host, in_flight=in_flight, available=available)
