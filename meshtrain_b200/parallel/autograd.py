"""Explicit autograd boundaries between pipeline stages.

Autograd never crosses a process: a received activation becomes a fresh leaf;
the gradient that comes back later continues the chain with
``output.backward(grad)``.  ``ContextStore`` keeps each microbatch's local
graph keyed by (step, microbatch) and rejects duplicates and unknown keys
(reference runtime/distributed_autograd.py:28-108).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


class BoundaryError(RuntimeError):
    """Activation / gradient routing violated the pipeline protocol."""


def make_boundary_input(received: torch.Tensor, requires_grad: bool) -> torch.Tensor:
    leaf = received.detach()
    if requires_grad and leaf.is_floating_point():
        leaf.requires_grad_(True)
    return leaf


def boundary_backward(output: torch.Tensor, grad_output: torch.Tensor) -> None:
    if grad_output.shape != output.shape:
        raise BoundaryError(f"gradient shape {tuple(grad_output.shape)} != activation shape {tuple(output.shape)}")
    if grad_output.device.type != output.device.type:
        raise BoundaryError(f"gradient on {grad_output.device}, activation on {output.device}")
    output.backward(grad_output.to(output.dtype))


def boundary_input_grad(inp: torch.Tensor) -> torch.Tensor | None:
    if not inp.requires_grad:
        return None
    return torch.zeros_like(inp) if inp.grad is None else inp.grad  # an unused input has zero gradient


@dataclass
class MicrobatchContext:
    step_id: int
    microbatch_id: int
    input: torch.Tensor | None = None
    output: torch.Tensor | None = None
    timings: dict[str, float] = field(default_factory=dict)
    autograd_saved_bytes: int = 0
    peak_saved_bytes: int = 0

    @property
    def key(self) -> tuple[int, int]:
        return (self.step_id, self.microbatch_id)

    def saved_bytes(self) -> int:
        n = self.autograd_saved_bytes
        for t in (self.input, self.output):
            if t is not None:
                n += t.numel() * t.element_size()
        return n


class ContextStore:
    def __init__(self) -> None:
        self._ctx: dict[tuple[int, int], MicrobatchContext] = {}

    def put(self, ctx: MicrobatchContext) -> None:
        if ctx.key in self._ctx:
            raise BoundaryError(f"duplicate forward for step={ctx.step_id} microbatch={ctx.microbatch_id}")
        self._ctx[ctx.key] = ctx

    def pop(self, step_id: int, microbatch_id: int) -> MicrobatchContext:
        try:
            return self._ctx.pop((step_id, microbatch_id))
        except KeyError:
            raise BoundaryError(f"gradient for unknown step={step_id} microbatch={microbatch_id}; "
                                f"pending={sorted(self._ctx)}") from None

    def __len__(self) -> int:
        return len(self._ctx)

    def pending(self) -> list[tuple[int, int]]:
        return sorted(self._ctx)

    def saved_bytes(self) -> int:
        return sum(c.saved_bytes() for c in self._ctx.values())

    def clear(self) -> None:
        self._ctx.clear()
