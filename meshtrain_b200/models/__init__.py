"""Model registry: ``type`` in {mlp, tiny_transformer, gpt, llama}.

``tiny_transformer`` (the reference's name, reference models/__init__.py:14-31)
and ``gpt`` build the same GPT family.
"""

from __future__ import annotations

import torch

from meshtrain_b200.models.base import ModelSpec, PipelineLayer, layer_seed
from meshtrain_b200.models.gpt import GPTSpec
from meshtrain_b200.models.llama import LlamaSpec
from meshtrain_b200.models.mlp import MLPSpec
from meshtrain_b200.models.split import SplitBlockSpec, split_blocks

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def build_model_spec(cfg: dict, seed: int = 0) -> ModelSpec:
    """Build a ModelSpec from the ``model:`` section of a config (plus optional ``data`` kind).

    ``split_blocks: true`` (gpt / llama) makes each block's attention and MLP halves
    separate partition units (models/split.py); parameters and tensor IDs are unchanged.
    """
    cfg = dict(cfg)
    if cfg.pop("split_blocks", False):
        return split_blocks(build_model_spec(cfg, seed))
    kind = cfg.pop("type")
    dtype = DTYPES[cfg.pop("dtype", "float32")]
    data = cfg.pop("data", None)
    if kind == "mlp":
        return MLPSpec(sizes=cfg.get("sizes"), seed=seed, dtype=dtype)
    if kind in ("tiny_transformer", "gpt"):
        return GPTSpec(
            layers=cfg.get("layers", 6),
            hidden_size=cfg.get("hidden_size", 256),
            heads=cfg.get("heads", 4),
            vocab_size=cfg.get("vocab_size", 256),
            seq_len=cfg.get("seq_len", 64),
            seed=seed,
            dtype=dtype,
            mlp_ratio=cfg.get("mlp_ratio", 4),
            init_std=cfg.get("init_std"),
            data=data or ("arithmetic" if kind == "tiny_transformer" else "uniform"),
        )
    if kind == "llama":
        return LlamaSpec(
            layers=cfg.get("layers", 32),
            hidden_size=cfg.get("hidden_size", 4096),
            heads=cfg.get("heads", 32),
            kv_heads=cfg.get("n_kv_heads") or cfg.get("heads", 32),
            ffn_hidden=cfg.get("ffn_hidden", 14336),
            vocab_size=cfg.get("vocab_size", 128256),
            seq_len=cfg.get("seq_len", 4096),
            rope_theta=cfg.get("rope_theta", 500000.0),
            seed=seed,
            dtype=dtype,
            init_std=cfg.get("init_std", 0.02),
            data=data or "uniform",
        )
    raise ValueError(f"unknown model type {kind!r}")


__all__ = ["ModelSpec", "PipelineLayer", "MLPSpec", "GPTSpec", "LlamaSpec", "SplitBlockSpec", "split_blocks",
           "build_model_spec", "layer_seed", "DTYPES"]
