"""Validated job configuration (YAML -> strict pydantic; unknown keys are errors).

The schema and defaults of the reference are kept (reference config.py:16-215),
so every reference YAML validates unchanged.  Optional keys added for the B200
build: model types ``gpt`` / ``llama`` and their shape keys, ``data``,
``offload``, ``network.tensor_transport: nccl`` and ``kernels``.
"""

from __future__ import annotations

from pathlib import Path
from typing import Literal

import yaml
from pydantic import BaseModel, ConfigDict, Field, ValidationError, model_validator


class _Strict(BaseModel):
    model_config = ConfigDict(extra="forbid")


class JobConfig(_Strict):
    name: str = "meshtrain-job"
    seed: int = 0
    runs_dir: str = "runs"


class ModelConfig(_Strict):
    type: Literal["mlp", "tiny_transformer", "gpt", "llama"]
    sizes: list[int] | None = None  # mlp
    layers: int = Field(6, ge=1)
    hidden_size: int = Field(256, ge=8)
    heads: int = Field(4, ge=1)
    vocab_size: int = Field(256, ge=2)
    seq_len: int = Field(64, ge=2)
    dtype: Literal["float32", "float16", "bfloat16"] = "float32"
    # added: GPT / Llama shape
    mlp_ratio: int | None = Field(None, ge=1)
    n_kv_heads: int | None = Field(None, ge=1)
    ffn_hidden: int | None = Field(None, ge=16)
    rope_theta: float | None = Field(None, gt=0)
    init_std: float | None = Field(None, gt=0)
    # added: partition units of half a block (attention / MLP) for gpt and llama
    split_blocks: bool = False

    @model_validator(mode="after")
    def _check(self):
        if self.split_blocks and self.type not in ("gpt", "tiny_transformer", "llama"):
            raise ValueError("split_blocks applies to gpt / tiny_transformer / llama models")
        if self.type != "mlp" and self.hidden_size % self.heads:
            raise ValueError("hidden_size must be divisible by heads")
        if self.sizes is not None and (len(self.sizes) < 2 or min(self.sizes) < 1):
            raise ValueError("mlp sizes need >= 2 positive entries")
        if self.n_kv_heads is not None and self.heads % self.n_kv_heads:
            raise ValueError("heads must be a multiple of n_kv_heads")
        return self

    def spec_kwargs(self) -> dict:
        d = self.model_dump(exclude_none=True)
        if not d.get("split_blocks"):
            d.pop("split_blocks", None)
        if self.type == "mlp":
            return {k: v for k, v in d.items() if k in ("type", "sizes", "dtype")}
        return {k: v for k, v in d.items() if k != "sizes"}


class DataConfig(_Strict):
    kind: Literal["default", "uniform", "arithmetic"] = "default"
    seed: int | None = None


class TrainingConfig(_Strict):
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

    @model_validator(mode="after")
    def _check(self):
        mb = self.microbatch_size or self.batch_size
        if self.batch_size % mb:
            raise ValueError("batch_size must be a multiple of microbatch_size")
        return self

    @property
    def num_microbatches(self) -> int:
        return self.batch_size // (self.microbatch_size or self.batch_size)


class StagePlacement(_Strict):
    worker: str | None = None
    device: str | None = None
    layers: tuple[int, int]


class PlacementConfig(_Strict):
    strategy: Literal["topology_aware", "auto", "equal", "compute", "manual"] = "topology_aware"
    num_stages: int | None = Field(None, ge=1)
    stages: list[StagePlacement] | None = None
    enforce_memory_check: bool = True
    memory_headroom_fraction: float | None = Field(None, ge=0, lt=1)  # deprecated
    memory_headroom_min_gb: float | None = Field(None, ge=0)          # deprecated
    activation_overhead_factor: float = Field(1.25, ge=1)

    @model_validator(mode="after")
    def _check(self):
        if self.strategy == "manual" and not self.stages:
            raise ValueError("manual placement requires placement.stages")
        if self.stages:
            prev = None
            for s in self.stages:
                if s.layers[0] >= s.layers[1]:
                    raise ValueError(f"empty layer range {s.layers}")
                if prev is not None and s.layers[0] != prev:
                    raise ValueError("manual stages must be contiguous and ordered")
                prev = s.layers[1]
        return self


class MemoryConfig(_Strict):
    safety_factor: float = Field(0.85, gt=0, le=1)
    backend_safety_factor: dict[str, float] = {"mps": 0.80}
    framework_reserve_gb: dict[str, float] = {"cuda": 0.4, "mps": 0.0, "cpu": 0.25}
    validate_runtime_usage: bool = True
    probe_allocation: bool = True
    max_replans: int = Field(2, ge=0)
    replan_shrink: float = Field(0.85, gt=0, lt=1)

    def safety_factors(self) -> dict[str, float]:
        out = {b: self.safety_factor for b in ("cuda", "mps", "cpu")}
        out.update(self.backend_safety_factor)
        return out

    def framework_reserve_bytes(self) -> dict[str, int]:
        return {b: int(v * 1024 ** 3) for b, v in self.framework_reserve_gb.items()}


class WorkersConfig(_Strict):
    allow: list[Literal["cuda", "mps", "cpu"]] = ["cuda", "mps", "cpu"]
    require: list[str] = []


class NetworkConfig(_Strict):
    tensor_transport: Literal["tcp", "pipe", "nccl"] = "tcp"
    timeout_s: float = Field(60.0, gt=0)
    connect_timeout_s: float = Field(30.0, gt=0)
    max_tensor_mb: float = Field(1024.0, gt=0)


class PipelineConfig(_Strict):
    schedule: Literal["gpipe", "1f1b"] = "1f1b"
    max_inflight_microbatches: int | None = Field(None, ge=1)


class TransportConfig(_Strict):
    async_: bool = Field(True, alias="async")
    pinned_memory: bool = True
    buffer_pool: bool = True
    max_outbound_queue: int | None = Field(None, ge=1)

    model_config = ConfigDict(extra="forbid", populate_by_name=True)


class OffloadConfig(_Strict):
    """Tier fp32 master weights / Adam moments to pinned host RAM (GPU engine)."""

    params: Literal["device", "host"] = "device"
    optimizer: Literal["device", "host"] = "device"
    prefetch_ahead: int = Field(1, ge=0)
    chunk_mb: float = Field(256.0, gt=0)


class MeshTrainConfig(_Strict):
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

    @model_validator(mode="after")
    def _check(self):
        if self.placement.stages:
            n = self.model_num_layers()
            if self.placement.stages[0].layers[0] != 0 or self.placement.stages[-1].layers[1] != n:
                raise ValueError(f"manual stages must cover layers [0, {n})")
        return self

    def model_spec_dict(self) -> dict:
        d = self.model.spec_kwargs()
        if self.data.kind != "default":
            d["data"] = self.data.kind
        return d

    def pipeline_settings(self, job_id: str, **overrides):
        from meshtrain_b200.parallel.pipeline import PipelineSettings

        kw = dict(job_id=job_id, steps=self.training.steps, batch_size=self.training.batch_size,
                  num_microbatches=self.training.num_microbatches, timeout_s=self.network.timeout_s,
                  log_every=self.training.log_every, schedule=self.pipeline.schedule,
                  max_inflight_microbatches=self.pipeline.max_inflight_microbatches,
                  async_transport=self.transport.async_, max_outbound_queue=self.transport.max_outbound_queue,
                  pinned_memory=self.transport.pinned_memory, buffer_pool=self.transport.buffer_pool)
        kw.update(overrides)
        return PipelineSettings(**kw)

    def build_model_spec(self):
        from meshtrain_b200.models import build_model_spec

        return build_model_spec(self.model_spec_dict(), seed=self.data.seed if self.data.seed is not None
                                else self.job.seed)

    def model_num_layers(self) -> int:
        return self.build_model_spec().num_layers


class ConfigError(ValueError):
    pass


def parse_config(data: dict) -> MeshTrainConfig:
    try:
        return MeshTrainConfig.model_validate(data)
    except ValidationError as exc:
        raise ConfigError(f"invalid MeshTrain config:\n{exc}") from exc


def load_config(path: str | Path) -> MeshTrainConfig:
    with open(path) as f:
        data = yaml.safe_load(f)
    if not isinstance(data, dict):
        raise ConfigError(f"{path}: top level must be a mapping")
    return parse_config(data)
