"""Device memory a stage needs, component by component.

For a stage holding parameters of P bytes (n parameters) on a device of T bytes:

| component                | autograd engine (torch optimizers)  | device engine (flat fp32 buffers)        |
|--------------------------|-------------------------------------|------------------------------------------|
| parameters               | P                                   | P (bf16 compute copies)                  |
| gradients                | P                                   | 4n (fp32)                                |
| master_weights           | 0                                   | 4n when P is not fp32 (0 with offload)   |
| optimizer_state          | 2P for Adam/AdamW                   | 8n, two fp32 moments (0 with offload)    |
| optimizer_step_temporary | P for Adam/AdamW (foreach temps)    | 0 (one fused launch)                     |
| saved_activations        | in_flight x saved bytes x activation_safety                                    |
| input / output buffers   | in_flight x boundary bytes, plus two input-gradient buffers                    |
| transport_buffers        | 2 x boundary on CPU stages (the pool shares host memory)                       |
| temporary_workspace      | 2 x largest layer output + largest per-layer saved (or recomputed) bytes       |
| offload_slots            | 0                                   | the device staging ring of offloaded state |

``in_flight`` is 1 on the last stage, M under GPipe and min(S - s, M, cap)
under 1F1B.  The usable budget is T x safety factor - framework reserve (or
the V1 headroom rule when one is configured), capped by what the device
reports free.  With offload the fp32 masters and Adam moments move to pinned
host RAM (``host_offload``).  The autograd column is the reference's
accounting (planner/memory.py:9-185); the device column is the GPU engine's.
On a B200 the defaults leave 8 % of the 180 GB HBM3e and 2 GB for the CUDA
context and NCCL buffers.
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
    offload_slots: int = 0  # device staging ring that streams offloaded state
    in_flight: int = 1
    available: int | None = None

    COMPONENTS = ("parameters", "gradients", "optimizer_state", "optimizer_step_temporary", "master_weights",
                  "saved_activations", "input_buffers", "output_buffers", "transport_buffers", "temporary_workspace",
                  "offload_slots")

    @property
    def required(self) -> int:
        return sum(getattr(self, name) for name in self.COMPONENTS)

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
        return dict(asdict(self), required=self.required, budget=self.budget, reserved=self.reserved, fits=self.fits)

    def format(self, worker: str, unified: bool = False) -> str:
        rows = [("total accelerator memory" + ("*" if unified else ""), self.total)]
        if self.available is not None:
            rows.append(("available (live, incl. cache)", self.available))
        rows.append(("usable (after safety/framework)", self.usable))
        rows += [(name.replace("_", " "), getattr(self, name)) for name in self.COMPONENTS if getattr(self, name)]
        rows += [("required", self.required), ("free after plan", self.usable - self.required)]
        if self.host_staging:
            rows.append(("host staging (pinned RAM)", self.host_staging))
        if self.host_offload:
            rows.append(("offloaded to host (pinned RAM)", self.host_offload))
        text = [f"Worker: {worker}"] + [f"    {label:<34}{value / GB:8.2f} GB" for label, value in rows]
        if unified:
            text.append("    * unified memory shared with the OS")
        return "\n".join(text)


def reserved_bytes(total: int, headroom_fraction: float, headroom_min_bytes: int) -> int:
    """The V1 headroom rule: keep max(fraction x total, minimum) free."""
    return int(max(total * headroom_fraction, headroom_min_bytes))


def in_flight_microbatches(schedule: str, stage_index: int, num_stages: int, num_microbatches: int,
                           max_inflight: int | None = None) -> int:
    """Microbatch graphs a stage holds at its peak under the schedule."""
    if stage_index >= num_stages - 1:
        return 1
    if schedule != "1f1b":
        return num_microbatches
    cap = num_microbatches if max_inflight is None else max_inflight
    return max(1, min(num_stages - stage_index, num_microbatches, cap))


def usable_bytes(total: int, backend: str, *, safety_factor=None, framework_reserve=None, headroom_fraction=None,
                 headroom_min_bytes=None, available=None) -> tuple[int, int]:
    """(usable budget, framework reserve) of a device of ``total`` bytes."""
    if headroom_fraction is not None or headroom_min_bytes is not None:
        usable, reserve = int(total) - reserved_bytes(total, headroom_fraction or 0.0, headroom_min_bytes or 0), 0
    else:
        factor = DEFAULT_SAFETY_FACTOR.get(backend, 0.85) if safety_factor is None else safety_factor
        reserve = DEFAULT_FRAMEWORK_RESERVE.get(backend, 0) if framework_reserve is None else framework_reserve
        usable = int(total * factor) - reserve
    if available is not None:
        usable = max(0, min(usable, int(available)))
    return usable, reserve


def _state_bytes(P: int, optimizer: str, engine: str, param_dtype_bytes: int, offload: bool) -> dict:
    """Gradients, master weights, optimizer moments and step temporaries (+ what goes to the host)."""
    if engine != "device":
        return {"gradients": P, "master_weights": 0, "optimizer_state": int(P * OPTIMIZER_STATE_FACTOR[optimizer]),
                "optimizer_step_temporary": int(P * OPTIMIZER_TEMP_FACTOR[optimizer]), "host_offload": 0}
    n = P // max(1, param_dtype_bytes)
    master = 0 if param_dtype_bytes == 4 else 4 * n
    moments = int(4 * n * OPTIMIZER_STATE_FACTOR[optimizer])
    host = master + moments if offload else 0
    return {"gradients": 4 * n, "master_weights": 0 if offload else master,
            "optimizer_state": 0 if offload else moments, "optimizer_step_temporary": 0, "host_offload": host}


def estimate_stage_memory(layers, *, total: int, optimizer: str, num_microbatches: int, is_last: bool,
                          stage_index: int | None = None, num_stages: int | None = None, schedule: str = "gpipe",
                          max_inflight: int | None = None, backend: str = "cuda", safety_factor: float | None = None,
                          framework_reserve: int | None = None, headroom_fraction: float | None = None,
                          headroom_min_bytes: int | None = None, activation_safety: float = 1.25,
                          available: int | None = None, engine: str = "autograd",
                          param_dtype_bytes: int = 4, offload: bool = False,
                          offload_ring: dict | None = None) -> MemoryEstimate:
    """Estimate for the contiguous ``layers`` (LayerProfiles) as one stage; see the module table."""
    if num_stages is None:
        num_stages = 1 if is_last else 2
    if stage_index is None:
        stage_index = num_stages - 1 if is_last else 0
    in_flight = 1 if is_last else in_flight_microbatches(schedule, stage_index, num_stages, num_microbatches,
                                                         max_inflight)
    P = sum(layer.param_bytes for layer in layers)
    inp, out = layers[0].input_bytes, layers[-1].activation_bytes
    boundary = max(inp, out)
    usable, reserve = usable_bytes(total, backend, safety_factor=safety_factor, framework_reserve=framework_reserve,
                                   headroom_fraction=headroom_fraction, headroom_min_bytes=headroom_min_bytes,
                                   available=available)
    state = _state_bytes(P, optimizer, engine, param_dtype_bytes, offload)
    slots = 0
    if offload and engine == "device":
        from meshtrain_b200.parallel.offload import slot_ring_bytes

        slots = slot_ring_bytes(P // max(1, param_dtype_bytes), **(offload_ring or {}))
    staged_on_host = backend != "cpu" and engine != "device"
    return MemoryEstimate(
        total=int(total), usable=usable, parameters=P,
        saved_activations=int(in_flight * sum(layer.saved_bytes for layer in layers) * activation_safety),
        input_buffers=in_flight * inp,
        output_buffers=(0 if is_last else in_flight * out) + 2 * inp,
        transport_buffers=2 * boundary if backend == "cpu" else 0,
        temporary_workspace=2 * max(layer.activation_bytes for layer in layers)
        + max(max(layer.saved_bytes, layer.recompute_bytes) for layer in layers),
        framework_reserve=reserve, host_staging=(in_flight + 2) * boundary if staged_on_host else 0,
        in_flight=in_flight, available=available, offload_slots=slots, **state)


def estimate_interleaved_rank(layers, pieces: list[tuple[int, int]], rank: int, world: int, chunks: int,
                              num_microbatches: int, *, total: int, optimizer: str, param_dtype_bytes: int,
                              offload: bool = False, offload_ring: dict | None = None,
                              **usable_kw) -> MemoryEstimate:
    """Estimate for rank ``rank`` of an interleaved 1F1B placement (pieces r, r + world, ...).

    Its program keeps up to ``interleaved_warmup + 1`` chunk-forwards alive, each holding one
    chunk's saved activations, so the estimate counts that many times the largest chunk's
    activations (expressed as an in-flight count over all of the rank's saved bytes).
    ``usable_kw`` are the safety-factor / reserve / headroom arguments of ``usable_bytes``.
    """
    import math

    from meshtrain_b200.parallel.schedule import interleaved_warmup

    mine = [pieces[c * world + rank] for c in range(chunks)]
    rank_layers = [layers[i] for a, b in mine for i in range(a, b)]
    saved = sum(lay.saved_bytes for lay in rank_layers) or 1
    largest = max(sum(layers[i].saved_bytes for i in range(a, b)) for a, b in mine)
    alive = interleaved_warmup(rank, world, num_microbatches, chunks) + 1
    in_flight = max(1, math.ceil(alive * largest / saved))  # in_flight x saved >= alive x largest
    return estimate_stage_memory(rank_layers, total=int(total), optimizer=optimizer,
                                 num_microbatches=max(num_microbatches, in_flight), is_last=False,
                                 stage_index=0, num_stages=in_flight + 1, schedule="1f1b", max_inflight=in_flight,
                                 engine="device", param_dtype_bytes=param_dtype_bytes, offload=offload,
                                 offload_ring=offload_ring, **usable_kw)
