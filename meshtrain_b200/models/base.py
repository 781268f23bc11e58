"""Model specification: an ordered list of layers + loss + synthetic data.

A model is cut into contiguous layer ranges (pipeline stages).  Every layer is
initialised under its own seed, ``layer_seed(seed, i)``, so any rank can build
exactly ``layers[start:end]`` and obtain the parameters the single-process
model has (reference models/base.py:18-61; the seed formula is kept so
per-layer parameters agree with the reference's).

Layers are :class:`PipelineLayer` modules with an explicit ``fwd``/``bwd``
pair.  The GPU pipeline engine calls those directly (no autograd graph, weight
gradients accumulated in place into fp32 buffers); ``forward`` wraps the same
pair in an autograd Function so the layer also works inside ordinary PyTorch
autograd (the reference-compatible ``Stage`` path and the single-process
oracle).
"""

from __future__ import annotations

import abc
from dataclasses import dataclass

import torch
from torch import nn


def layer_seed(seed: int, index: int) -> int:
    return (seed * 1_000_003 + index * 7919) % (2**31 - 1)


class PipelineLayer(nn.Module):
    """A layer with an explicit forward/backward pair.

    ``fwd(x, saved)`` returns the output and stores what backward needs in the
    ``saved`` dict.  ``bwd(dy, saved, grads)`` returns the input gradient (or
    None for integer inputs) and *accumulates* parameter gradients into
    ``grads[name]`` (fp32 tensors shaped like the parameters).
    """

    takes_integer_input = False

    def fwd(self, x: torch.Tensor, saved: dict) -> torch.Tensor:  # pragma: no cover - abstract
        raise NotImplementedError

    def bwd(self, dy: torch.Tensor, saved: dict, grads: dict[str, torch.Tensor]) -> torch.Tensor | None:
        raise NotImplementedError  # pragma: no cover - abstract

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        names = [n for n, _ in self.named_parameters()]
        params = [p for _, p in self.named_parameters()]
        return _LayerFn.apply(self, names, x, *params)


class _LayerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, layer, names, x, *params):
        saved: dict = {}
        with torch.no_grad():
            y = layer.fwd(x, saved)
        ctx.layer, ctx.names, ctx.saved = layer, names, saved
        ctx.param_meta = [(p.shape, p.dtype, p.device) for p in params]
        return y

    @staticmethod
    def backward(ctx, dy):
        grads = {n: torch.zeros(shape, dtype=torch.float32, device=dev)
                 for n, (shape, _dt, dev) in zip(ctx.names, ctx.param_meta)}
        with torch.no_grad():
            dx = ctx.layer.bwd(dy.contiguous(), ctx.saved, grads)
        ctx.saved = None
        pgrads = [grads[n].to(dt) for n, (_s, dt, _d) in zip(ctx.names, ctx.param_meta)]
        return (None, None, dx, *pgrads)


class ModelSpec(abc.ABC):
    name: str = "model"
    # Ops a worker must support to host a stage (see worker/capabilities.py).
    required_ops: tuple[str, ...] = ("linear", "cross_entropy")

    def __init__(self, seed: int = 0, dtype: torch.dtype = torch.float32):
        self.seed = seed
        self.dtype = dtype

    @property
    @abc.abstractmethod
    def num_layers(self) -> int: ...

    @abc.abstractmethod
    def _make_layer(self, index: int) -> nn.Module: ...

    @abc.abstractmethod
    def layer_name(self, index: int) -> str: ...

    @abc.abstractmethod
    def loss_fn(self, output: torch.Tensor, target: torch.Tensor) -> torch.Tensor: ...

    @abc.abstractmethod
    def make_batch(self, step: int, batch_size: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Deterministic synthetic (inputs, targets) on CPU for ``step``."""

    def global_layer(self, index: int) -> int:
        """Layer index used in tensor IDs (``model.layers.<g>.<name>``) for layer ``index``."""
        return index

    # -- shapes used by the GPU engine's p2p buffers ------------------------
    def boundary_shape(self, microbatch_size: int) -> tuple[int, ...]:
        """Shape of the activation crossing a stage boundary for one microbatch."""
        raise NotImplementedError

    def build_layer(self, index: int, device: torch.device | str | None = None) -> nn.Module:
        if not 0 <= index < self.num_layers:
            raise IndexError(index)
        dev = torch.device(device) if device is not None else torch.device("cpu")
        if dev.type == "cuda":
            # Per-layer seeded init straight on the device (large models): same
            # seed schedule, CUDA generator.
            with torch.random.fork_rng(devices=[dev]):
                torch.manual_seed(layer_seed(self.seed, index))
                with torch.device(dev):
                    layer = self._make_layer(index)
        else:
            with torch.random.fork_rng(devices=[]):
                torch.manual_seed(layer_seed(self.seed, index))
                layer = self._make_layer(index)
        return layer.to(self.dtype)

    def build_stage(self, start: int, end: int, device=None) -> nn.Sequential:
        """Contiguous layer range [start, end)."""
        if not 0 <= start < end <= self.num_layers:
            raise ValueError(f"invalid layer range [{start}, {end}) for {self.num_layers} layers")
        return nn.Sequential(*[self.build_layer(i, device) for i in range(start, end)])

    def build_full(self) -> nn.Sequential:
        return self.build_stage(0, self.num_layers)

    def describe(self) -> dict:
        return {"type": self.name, "num_layers": self.num_layers, "seed": self.seed,
                "parameters": self.parameter_count()}

    def parameter_count(self) -> int:
        with torch.device("meta"):
            return sum(p.numel() for i in range(self.num_layers) for p in self._make_layer(i).parameters())

    def layer_parameter_counts(self) -> list[int]:
        with torch.device("meta"):
            return [sum(p.numel() for p in self._make_layer(i).parameters()) for i in range(self.num_layers)]

    def flops_per_token(self) -> float:
        """Training FLOPs per token (forward + backward), for MFU reporting."""
        return 6.0 * self.parameter_count()


@dataclass
class StageRange:
    start: int
    end: int

    @property
    def size(self) -> int:
        return self.end - self.start


def uniform_tokens(seed: int, step: int, batch_size: int, seq_len: int, vocab: int):
    """i.i.d. uniform tokens; targets are the inputs shifted by one."""
    g = torch.Generator().manual_seed(seed * 100_003 + step)
    seq = torch.randint(0, vocab, (batch_size, seq_len + 1), generator=g)
    return seq[:, :-1].contiguous(), seq[:, 1:].contiguous()


def arithmetic_tokens(seed: int, step: int, batch_size: int, seq_len: int, vocab: int):
    """Arithmetic progressions ``(a + b t) mod V`` (reference models/tiny_transformer.py:96-102)."""
    g = torch.Generator().manual_seed(seed * 100_003 + step)
    a = torch.randint(0, vocab, (batch_size, 1), generator=g)
    b = torch.randint(1, 8, (batch_size, 1), generator=g)
    t = torch.arange(seq_len + 1)[None]
    seq = (a + b * t) % vocab
    return seq[:, :-1].contiguous(), seq[:, 1:].contiguous()
