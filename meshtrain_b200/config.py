"""Job configuration: YAML validated by strict pydantic models (unknown keys are errors).

The sections, key names and defaults are the reference's (config.py:16-215), so
every reference YAML validates unchanged; that schema is an interface.  Keys
added for the B200 build are optional: model types ``gpt`` / ``llama`` and
their shape keys (``mlp_ratio``, ``n_kv_heads``, ``ffn_hidden``, ``rope_theta``,
``init_std``, ``split_blocks``), ``data``, ``offload``,
``network.tensor_transport: nccl`` and ``kernels``, plus checkpointing keys
under ``training``.

Field types and ranges are declared on the models; rules that relate several
fields live in ``RULES`` tables next to each model and run after the fields
have been parsed, each returning an error message or None.
"""

from __future__ import annotations

from pathlib import Path
from typing import ClassVar, Literal

import yaml
from pydantic import BaseModel, ConfigDict, Field, ValidationError, model_validator

GB = 1024 ** 3
BACKENDS = ("cuda", "mps", "cpu")


class ConfigError(ValueError):
    pass


class _Section(BaseModel):
    """A config section: no unknown keys; cross-field ``RULES`` checked after parsing."""

    model_config = ConfigDict(extra="forbid")
    RULES: ClassVar[tuple] = ()

    @model_validator(mode="after")
    def _apply_rules(self):
        for rule in self.RULES:
            problem = rule(self)
            if problem:
                raise ValueError(problem)
        return self


class JobConfig(_Section):
    name: str = "meshtrain-job"
    seed: int = 0
    runs_dir: str = "runs"


def _heads_divide_hidden(m):
    if m.type != "mlp" and m.hidden_size % m.heads:
        return "hidden_size must be divisible by heads"


def _kv_heads_divide_heads(m):
    if m.n_kv_heads is not None and m.heads % m.n_kv_heads:
        return "heads must be a multiple of n_kv_heads"


def _mlp_sizes(m):
    if m.sizes is not None and (len(m.sizes) < 2 or min(m.sizes) < 1):
        return "mlp sizes need >= 2 positive entries"


def _split_blocks_needs_blocks(m):
    if m.split_blocks and m.type == "mlp":
        return "split_blocks applies to gpt / tiny_transformer / llama models"


class ModelConfig(_Section):
    type: Literal["mlp", "tiny_transformer", "gpt", "llama"]
    sizes: list[int] | None = None                 # mlp layer widths
    layers: int = Field(6, ge=1)
    hidden_size: int = Field(256, ge=8)
    heads: int = Field(4, ge=1)
    vocab_size: int = Field(256, ge=2)
    seq_len: int = Field(64, ge=2)
    dtype: Literal["float32", "float16", "bfloat16"] = "float32"
    mlp_ratio: int | None = Field(None, ge=1)
    n_kv_heads: int | None = Field(None, ge=1)
    ffn_hidden: int | None = Field(None, ge=16)
    rope_theta: float | None = Field(None, gt=0)
    init_std: float | None = Field(None, gt=0)
    split_blocks: bool = False                     # partition units of half a block (attention / MLP)

    RULES = (_split_blocks_needs_blocks, _heads_divide_hidden, _mlp_sizes, _kv_heads_divide_heads)

    def spec_kwargs(self) -> dict:
        """Keyword arguments of the model registry for this model."""
        fields = self.model_dump(exclude_none=True)
        if self.type == "mlp":
            return {k: fields[k] for k in ("type", "sizes", "dtype") if k in fields}
        fields.pop("sizes", None)
        if not self.split_blocks:
            fields.pop("split_blocks", None)
        return fields


class DataConfig(_Section):
    kind: Literal["default", "uniform", "arithmetic"] = "default"
    seed: int | None = None


def _microbatches_divide_batch(t):
    if t.batch_size % (t.microbatch_size or t.batch_size):
        return "batch_size must be a multiple of microbatch_size"


def _recompute_policy_known(t):
    from meshtrain_b200.parallel.recompute import parse_policy

    try:
        parse_policy(t.activation_recompute)
    except ValueError as exc:
        return str(exc)


class TrainingConfig(_Section):
    batch_size: int = Field(32, ge=1)
    microbatch_size: int | None = Field(None, ge=1)
    learning_rate: float = Field(0.01, gt=0)
    optimizer: Literal["sgd", "adam", "adamw"] = "sgd"
    weight_decay: float = Field(0.0, ge=0)
    steps: int = Field(100, ge=1)
    log_every: int = Field(10, ge=1)
    checkpoint_every: int | None = Field(None, ge=1)
    checkpoint_dir: str | None = None   # default: <runs_dir>/<job>/checkpoints
    resume_from: str | None = None      # a checkpoint directory; training continues at its newest complete step
    # device engine: none | all | every:K | largest:N (parallel/recompute.py)
    activation_recompute: str = "none"

    RULES = (_microbatches_divide_batch, _recompute_policy_known)

    @property
    def num_microbatches(self) -> int:
        return self.batch_size // (self.microbatch_size or self.batch_size)


class StagePlacement(_Section):
    worker: str | None = None
    device: str | None = None
    layers: tuple[int, int]


def _manual_needs_stages(p):
    if p.strategy == "manual" and not p.stages:
        return "manual placement requires placement.stages"


def _stages_contiguous(p):
    edges = [s.layers for s in p.stages or []]
    empty = next((r for r in edges if r[0] >= r[1]), None)
    if empty is not None:
        return f"empty layer range {empty}"
    if any(a[1] != b[0] for a, b in zip(edges, edges[1:])):
        return "manual stages must be contiguous and ordered"


class PlacementConfig(_Section):
    strategy: Literal["topology_aware", "auto", "equal", "compute", "manual"] = "topology_aware"
    num_stages: int | None = Field(None, ge=1)
    stages: list[StagePlacement] | None = None
    enforce_memory_check: bool = True
    memory_headroom_fraction: float | None = Field(None, ge=0, lt=1)  # V1 key, still honoured
    memory_headroom_min_gb: float | None = Field(None, ge=0)          # V1 key, still honoured
    activation_overhead_factor: float = Field(1.25, ge=1)

    RULES = (_manual_needs_stages, _stages_contiguous)


class MemoryConfig(_Section):
    safety_factor: float = Field(0.85, gt=0, le=1)
    backend_safety_factor: dict[str, float] = {"mps": 0.80}
    framework_reserve_gb: dict[str, float] = {"cuda": 0.4, "mps": 0.0, "cpu": 0.25}
    validate_runtime_usage: bool = True
    probe_allocation: bool = True
    max_replans: int = Field(2, ge=0)
    replan_shrink: float = Field(0.85, gt=0, lt=1)

    def safety_factors(self) -> dict[str, float]:
        """Per backend: the backend's own factor where set, else the global one."""
        return {b: self.backend_safety_factor.get(b, self.safety_factor) for b in BACKENDS} | \
            dict(self.backend_safety_factor)

    def framework_reserve_bytes(self) -> dict[str, int]:
        return {backend: int(gb * GB) for backend, gb in self.framework_reserve_gb.items()}


class WorkersConfig(_Section):
    allow: list[Literal["cuda", "mps", "cpu"]] = list(BACKENDS)
    require: list[str] = []


class NetworkConfig(_Section):
    tensor_transport: Literal["tcp", "pipe", "nccl"] = "tcp"
    timeout_s: float = Field(60.0, gt=0)
    connect_timeout_s: float = Field(30.0, gt=0)
    max_tensor_mb: float = Field(1024.0, gt=0)
    # host links only: fp32 boundary tensors cross as 16-bit floats (lossy; networking/compression.py)
    compression: Literal["none", "bf16", "fp16"] = "none"


class PipelineConfig(_Section):
    schedule: Literal["gpipe", "1f1b"] = "1f1b"
    max_inflight_microbatches: int | None = Field(None, ge=1)
    # device engine: model chunks per GPU (interleaved 1F1B when > 1; needs the 1f1b schedule
    # and a microbatch count that is a multiple of the number of stages)
    virtual_stages: int = Field(1, ge=1, le=8)
    # device engine (plain or interleaved): after this many steps, move stage boundaries once if the measured
    # per-stage work is unbalanced (parallel/migration.py); None keeps the planned split
    rebalance_after_steps: int | None = Field(None, ge=2)


class TransportConfig(_Section):
    model_config = ConfigDict(extra="forbid", populate_by_name=True)

    async_: bool = Field(True, alias="async")
    pinned_memory: bool = True
    buffer_pool: bool = True
    max_outbound_queue: int | None = Field(None, ge=1)


class OffloadConfig(_Section):
    """Fp32 master weights / Adam moments in pinned host RAM (device engine)."""

    # "auto": host only if the startup memory estimate says the stage does not fit with its state resident
    params: Literal["device", "host", "auto"] = "device"
    optimizer: Literal["device", "host", "auto"] = "device"
    prefetch_ahead: int = Field(1, ge=0)
    chunk_mb: float = Field(256.0, gt=0)
    device_budget_gb: float | None = Field(None, gt=0)  # device memory for the slot ring


def _manual_stages_cover_model(c):
    stages = c.placement.stages
    if stages:
        n = c.model_num_layers()
        if stages[0].layers[0] != 0 or stages[-1].layers[1] != n:
            return f"manual stages must cover layers [0, {n})"


def _virtual_stages_supported(c):
    if c.pipeline.virtual_stages > 1:
        if c.pipeline.schedule != "1f1b":
            return "pipeline.virtual_stages > 1 runs interleaved 1F1B: set pipeline.schedule to 1f1b"


class MeshTrainConfig(_Section):
    job: JobConfig = JobConfig()
    model: ModelConfig
    data: DataConfig = DataConfig()
    training: TrainingConfig = TrainingConfig()
    placement: PlacementConfig = PlacementConfig()
    workers: WorkersConfig = WorkersConfig()
    network: NetworkConfig = NetworkConfig()
    pipeline: PipelineConfig = PipelineConfig()
    transport: TransportConfig = TransportConfig()
    memory: MemoryConfig = MemoryConfig()
    offload: OffloadConfig = OffloadConfig()
    kernels: Literal["custom", "torch"] = "custom"

    RULES = (_manual_stages_cover_model, _virtual_stages_supported)

    def model_spec_dict(self) -> dict:
        spec = self.model.spec_kwargs()
        if self.data.kind != "default":
            spec["data"] = self.data.kind
        return spec

    def pipeline_settings(self, job_id: str, **overrides):
        """The host runtime's settings for this job (``overrides`` win)."""
        from meshtrain_b200.parallel.pipeline import PipelineSettings

        t, p, x = self.training, self.pipeline, self.transport
        settings = dict(job_id=job_id, steps=t.steps, batch_size=t.batch_size, num_microbatches=t.num_microbatches,
                        timeout_s=self.network.timeout_s, log_every=t.log_every, schedule=p.schedule,
                        max_inflight_microbatches=p.max_inflight_microbatches, async_transport=x.async_,
                        max_outbound_queue=x.max_outbound_queue, pinned_memory=x.pinned_memory,
                        buffer_pool=x.buffer_pool, wire_compression=self.network.compression)
        return PipelineSettings(**{**settings, **overrides})

    def build_model_spec(self):
        from meshtrain_b200.models import build_model_spec

        seed = self.job.seed if self.data.seed is None else self.data.seed
        return build_model_spec(self.model_spec_dict(), seed=seed)

    def model_num_layers(self) -> int:
        return self.build_model_spec().num_layers


def parse_config(data: dict) -> MeshTrainConfig:
    try:
        return MeshTrainConfig.model_validate(data)
    except ValidationError as exc:
        raise ConfigError(f"invalid MeshTrain config:\n{exc}") from exc


def load_config(path: str | Path) -> MeshTrainConfig:
    data = yaml.safe_load(Path(path).read_text())
    if not isinstance(data, dict):
        raise ConfigError(f"{path}: top level must be a mapping")
    return parse_config(data)
