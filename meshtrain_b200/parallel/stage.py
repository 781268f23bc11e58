"""A pipeline stage on the host runtime: a contiguous slice of the model under
PyTorch autograd, with its optimizer and the graphs of its in-flight microbatches.

This is the portable path (CPU, MPS, heterogeneous or TCP-connected stages,
fp32 parity runs).  GPU stages inside one box use the device engine
(parallel/engine.py) instead.  Same contract as the reference's stage
(runtime/stage.py:28-211): ``forward`` parks the microbatch's graph;
``backward`` / ``loss_backward`` resume it and return the input gradient;
``optimizer_step`` refuses to run while graphs are parked.

A stage's step timings are host wall-clock spans, so each call waits for the
device (``sync_compute``) before it returns; the device engine avoids that
with CUDA events.
"""

from __future__ import annotations

import contextlib
import time
from typing import Callable

import torch
from torch import nn

from meshtrain_b200.parallel.autograd import (BoundaryError, GraphTable, MicrobatchGraph, continue_backward,
                                              detach_as_leaf, input_gradient)
from meshtrain_b200.parallel.tensor_store import LocalTensorStore, TensorRole, activation_id, parameter_id
from meshtrain_b200.worker.device import CPUDeviceAdapter, DeviceAdapter

OPTIMIZERS = {
    "sgd": lambda params, lr, kw: torch.optim.SGD(params, lr=lr, momentum=kw.get("momentum", 0.0)),
    "adam": lambda params, lr, kw: torch.optim.Adam(params, lr=lr),
    "adamw": lambda params, lr, kw: torch.optim.AdamW(params, lr=lr, weight_decay=kw.get("weight_decay", 0.0)),
}


def build_optimizer(name: str, params, lr: float, **kw) -> torch.optim.Optimizer:
    make = OPTIMIZERS.get(name.lower())
    if make is None:
        raise ValueError(f"unknown optimizer {name!r}")
    return make(params, lr, kw)


class SavedTensorMeter:
    """Counts the bytes autograd saves for backward, parameters excluded."""

    def __init__(self, params):
        self.param_ids = {id(p) for p in params}
        self.nbytes = 0
        self._hooks = torch.autograd.graph.saved_tensors_hooks(self._pack, lambda t: t)

    def _pack(self, t: torch.Tensor) -> torch.Tensor:
        owner = t if t._base is None else t._base
        if id(t) not in self.param_ids and id(owner) not in self.param_ids:
            self.nbytes += t.numel() * t.element_size()
        return t

    def __enter__(self):
        self._hooks.__enter__()
        return self

    def __exit__(self, *exc):
        self._hooks.__exit__(*exc)


class Stage:
    def __init__(self, module: nn.Module, *, stage_index: int, num_stages: int, device: DeviceAdapter | None = None,
                 optimizer: str = "sgd", lr: float = 0.01,
                 loss_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None,
                 name: str | None = None, layer_offset: int = 0):
        if stage_index == num_stages - 1 and loss_fn is None:
            raise ValueError("the last stage needs a loss function")
        self.device = device or CPUDeviceAdapter()
        self.module = self.device.move_module(module)
        self.stage_index, self.num_stages = stage_index, num_stages
        self.name = name or f"stage{stage_index}"
        self.layer_offset = layer_offset
        self.loss_fn = loss_fn
        self.params = list(self.module.parameters())
        self.optimizer = build_optimizer(optimizer, self.params, lr) if self.params else None
        self.contexts = GraphTable()
        self.tensor_store = LocalTensorStore(self.name, self.device.backend)
        for local, p in self.module.named_parameters():
            self.tensor_store.put(self.global_name(local), p, TensorRole.PARAMETER)

    @property
    def is_first(self) -> bool:
        return self.stage_index == 0

    @property
    def is_last(self) -> bool:
        return self.stage_index == self.num_stages - 1

    def global_name(self, local_name: str) -> str:
        """'<i>.<param>' inside the slice -> the model-wide tensor ID of layer offset+i."""
        index, rest = local_name.split(".", 1)
        return parameter_id(self.layer_offset + int(index), rest)

    # ---------------------------------------------------------------- compute
    @contextlib.contextmanager
    def _clocked(self, into: dict, phase: str):
        """Host wall time of the block, the device's queued work included, stored as ``into[phase]``."""
        began = time.perf_counter()
        yield
        self.device.sync_compute()
        into[phase] = time.perf_counter() - began

    def forward(self, inp: torch.Tensor, graph: MicrobatchGraph) -> torch.Tensor:
        """Runs the slice on one microbatch and parks its graph; returns the output."""
        with self._clocked(graph.timings, "forward"):
            leaf = detach_as_leaf(self.device.move_tensor(inp), requires_grad=not self.is_first)
            with SavedTensorMeter(self.params) as meter:
                out = self.module(leaf)
            graph.leaf, graph.output, graph.autograd_saved_bytes = leaf, out, meter.nbytes
        self.contexts.park(graph)
        self.tensor_store.put(activation_id(graph.step_id, graph.microbatch_id, self.stage_index), leaf,
                              TensorRole.ACTIVATION)
        return out

    def _resume(self, key: tuple[int, int]) -> MicrobatchGraph:
        graph = self.contexts.take(*key)
        self.tensor_store.discard(activation_id(*key, self.stage_index))
        return graph

    def _input_grad(self, graph: MicrobatchGraph):
        grad = None if self.is_first else input_gradient(graph.leaf)
        graph.release()
        return grad

    def loss_backward(self, target, key: tuple[int, int], loss_scale: float = 1.0):
        """Last stage: loss of a parked microbatch, then its backward -> (loss, input grad, graph)."""
        if not self.is_last:
            raise BoundaryError("loss_backward is only valid on the last stage")
        graph = self._resume(key)
        with self._clocked(graph.timings, "backward"):
            loss = self.loss_fn(graph.output, self.device.move_tensor(target))
            loss.mul(loss_scale).backward()
        return loss.detach(), self._input_grad(graph), graph

    def forward_loss(self, inp, target, graph: MicrobatchGraph, loss_scale: float = 1.0):
        """Last stage, forward and backward in one call -> (loss, input grad)."""
        self.forward(inp, graph)
        loss, grad, _ = self.loss_backward(target, graph.key, loss_scale)
        return loss, grad

    def backward(self, grad_output, key: tuple[int, int]):
        """Resumes a parked microbatch with dL/d output -> (input grad, graph)."""
        graph = self._resume(key)
        with self._clocked(graph.timings, "backward"):
            continue_backward(graph.output, self.device.move_tensor(grad_output))
        return self._input_grad(graph), graph

    def optimizer_step(self) -> float:
        """Applies the accumulated gradients; returns its wall time (refused while graphs are parked)."""
        if len(self.contexts):
            raise BoundaryError(f"optimizer step with pending microbatches {self.contexts.pending()}")
        clock: dict[str, float] = {}
        with self._clocked(clock, "step"):
            if self.optimizer is not None:
                self.optimizer.step()
        return clock["step"]

    def zero_grad(self) -> None:
        if self.optimizer is not None:
            self.optimizer.zero_grad(set_to_none=True)
        else:
            self.module.zero_grad(set_to_none=True)

    # ---------------------------------------------------------------- state
    def refresh_tensor_store(self) -> None:
        """Registers gradients and optimizer moments under their global tensor IDs."""
        for local, p in self.module.named_parameters():
            gid = self.global_name(local)
            if p.grad is not None:
                self.tensor_store.put(f"{gid}.grad", p.grad, TensorRole.GRADIENT)
            state = self.optimizer.state.get(p, {}) if self.optimizer is not None else {}
            for key, value in state.items():
                if torch.is_tensor(value) and value.dim() > 0:
                    self.tensor_store.put(f"{gid}.optim.{key}", value, TensorRole.OPTIMIZER_STATE)

    def named_gradients(self, prefix: str = "") -> dict[str, torch.Tensor]:
        return {prefix + n: p.grad.detach().cpu().clone() for n, p in self.module.named_parameters()
                if p.grad is not None}

    def named_parameters_cpu(self, prefix: str = "") -> dict[str, torch.Tensor]:
        return {prefix + n: p.detach().cpu().clone() for n, p in self.module.named_parameters()}

    def memory_report(self) -> dict[str, int]:
        def nbytes(ts):
            return sum(t.numel() * t.element_size() for t in ts)

        moments = []
        if self.optimizer is not None:
            moments = [v for st in self.optimizer.state.values() for v in st.values() if torch.is_tensor(v)]
        return {"parameters": nbytes(self.params), "gradients": nbytes(p.grad for p in self.params if p.grad is not None),
                "optimizer_state": nbytes(moments), "saved_activations": self.contexts.held_bytes()}
