"""Autograd across stage boundaries on the host runtime.

Autograd graphs never span two processes.  The activation a stage receives
becomes a fresh leaf tensor (``detach_as_leaf``); the stage's forward builds a
local graph from that leaf to its output; when the output's gradient comes
back from downstream, ``continue_backward`` resumes the chain from the output
and ``input_gradient`` is what travels upstream.  Between the two, the graph
of each in-flight microbatch is parked in a ``GraphTable`` under its
``(step, microbatch)`` key, which refuses duplicates and unknown keys
(reference runtime/distributed_autograd.py:28-108).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


class BoundaryError(RuntimeError):
    """Activation / gradient routing violated the pipeline protocol."""


def detach_as_leaf(received: torch.Tensor, requires_grad: bool) -> torch.Tensor:
    """A received activation as the root of this stage's graph."""
    leaf = received.detach()
    if requires_grad and leaf.is_floating_point():
        leaf.requires_grad_(True)
    return leaf


def continue_backward(output: torch.Tensor, grad: torch.Tensor) -> None:
    """Backpropagates ``grad`` (dL/d output, from downstream) through the local graph."""
    if tuple(grad.shape) != tuple(output.shape):
        raise BoundaryError(f"gradient shape {tuple(grad.shape)} != activation shape {tuple(output.shape)}")
    if grad.device.type != output.device.type:
        raise BoundaryError(f"gradient on {grad.device}, activation on {output.device}")
    output.backward(grad if grad.dtype == output.dtype else grad.to(output.dtype))


def input_gradient(leaf: torch.Tensor) -> torch.Tensor | None:
    """dL/d input of the stage (zeros when the input did not reach the loss)."""
    if not leaf.requires_grad:
        return None
    return leaf.grad if leaf.grad is not None else torch.zeros_like(leaf)


@dataclass
class MicrobatchGraph:
    """A microbatch's local graph between its forward and its backward."""

    step_id: int
    microbatch_id: int
    leaf: torch.Tensor | None = None
    output: torch.Tensor | None = None
    autograd_saved_bytes: int = 0
    timings: dict[str, float] = field(default_factory=dict)

    @property
    def key(self) -> tuple[int, int]:
        return self.step_id, self.microbatch_id

    def held_bytes(self) -> int:
        """Bytes kept alive for the backward: autograd's saved tensors plus the boundary tensors."""
        ends = sum(t.numel() * t.element_size() for t in (self.leaf, self.output) if t is not None)
        return self.autograd_saved_bytes + ends

    def release(self) -> None:
        self.leaf = self.output = None


class GraphTable:
    """In-flight microbatch graphs of one stage, keyed by (step, microbatch)."""

    def __init__(self) -> None:
        self._graphs: dict[tuple[int, int], MicrobatchGraph] = {}

    def park(self, graph: MicrobatchGraph) -> None:
        if graph.key in self._graphs:
            raise BoundaryError(f"duplicate forward for step={graph.step_id} microbatch={graph.microbatch_id}")
        self._graphs[graph.key] = graph

    def take(self, step_id: int, microbatch_id: int) -> MicrobatchGraph:
        graph = self._graphs.pop((step_id, microbatch_id), None)
        if graph is None:
            raise BoundaryError(f"gradient for unknown step={step_id} microbatch={microbatch_id}; "
                                f"pending={self.pending()}")
        return graph

    def pending(self) -> list[tuple[int, int]]:
        return sorted(self._graphs)

    def held_bytes(self) -> int:
        return sum(g.held_bytes() for g in self._graphs.values())

    def __len__(self) -> int:
        return len(self._graphs)

    def clear(self) -> None:
        self._graphs.clear()
