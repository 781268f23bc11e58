"""A pipeline stage under PyTorch autograd: a contiguous layer slice, its optimizer
and its saved microbatch contexts (reference runtime/stage.py:28-211).

This is the portable path (CPU, MPS, heterogeneous or TCP-connected stages, fp32
parity); GPU stages inside one box run ``parallel/engine.py`` instead.
"""

from __future__ import annotations

import time
from typing import Callable

import torch
from torch import nn

from meshtrain_b200.parallel.autograd import (BoundaryError, ContextStore, MicrobatchContext, boundary_backward,
                                              boundary_input_grad, make_boundary_input)
from meshtrain_b200.parallel.tensor_store import LocalTensorStore, TensorRole, activation_id, parameter_id
from meshtrain_b200.worker.device import CPUDeviceAdapter, DeviceAdapter


def build_optimizer(name: str, params, lr: float, **kw) -> torch.optim.Optimizer:
    name = name.lower()
    if name == "sgd":
        return torch.optim.SGD(params, lr=lr, momentum=kw.get("momentum", 0.0))
    if name == "adam":
        return torch.optim.Adam(params, lr=lr)
    if name == "adamw":
        return torch.optim.AdamW(params, lr=lr, weight_decay=kw.get("weight_decay", 0.0))
    raise ValueError(f"unknown optimizer {name!r}")


class Stage:
    def __init__(self, module: nn.Module, *, stage_index: int, num_stages: int, device: DeviceAdapter | None = None,
                 optimizer: str = "sgd", lr: float = 0.01,
                 loss_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None,
                 name: str | None = None, layer_offset: int = 0):
        self.device = device or CPUDeviceAdapter()
        self.module = self.device.move_module(module)
        self.stage_index, self.num_stages = stage_index, num_stages
        self.name = name or f"stage{stage_index}"
        params = list(self.module.parameters())
        self.optimizer = build_optimizer(optimizer, params, lr) if params else None
        self.loss_fn = loss_fn
        self.contexts = ContextStore()
        self._param_ids = {id(p) for p in params}
        if self.is_last and loss_fn is None:
            raise ValueError("the last stage needs a loss function")
        self.layer_offset = layer_offset
        self.tensor_store = LocalTensorStore(self.name, self.device.backend)
        for n, p in self.module.named_parameters():
            self.tensor_store.put(self.global_name(n), p, TensorRole.PARAMETER)

    @property
    def is_first(self) -> bool:
        return self.stage_index == 0

    @property
    def is_last(self) -> bool:
        return self.stage_index == self.num_stages - 1

    def global_name(self, local_name: str) -> str:
        idx, rest = local_name.split(".", 1)
        return parameter_id(int(idx) + self.layer_offset, rest)

    def refresh_tensor_store(self) -> None:
        for n, p in self.module.named_parameters():
            gid = self.global_name(n)
            if p.grad is not None:
                self.tensor_store.put(gid + ".grad", p.grad, TensorRole.GRADIENT)
            if self.optimizer is not None:
                for key, v in self.optimizer.state.get(p, {}).items():
                    if torch.is_tensor(v) and v.dim() > 0:
                        self.tensor_store.put(f"{gid}.optim.{key}", v, TensorRole.OPTIMIZER_STATE)

    def forward(self, inp: torch.Tensor, ctx: MicrobatchContext) -> torch.Tensor:
        """Local forward; keeps the graph in ``ctx``; returns the attached output."""
        t0 = time.perf_counter()
        x = make_boundary_input(self.device.move_tensor(inp), requires_grad=not self.is_first)
        pids = self._param_ids
        saved = 0

        def pack(t):
            nonlocal saved
            base = t._base if t._base is not None else t
            if id(t) not in pids and id(base) not in pids:
                saved += t.numel() * t.element_size()
            return t

        with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
            out = self.module(x)
        ctx.autograd_saved_bytes = saved
        self.device.sync_compute()
        ctx.input, ctx.output = x, out
        ctx.timings["forward"] = time.perf_counter() - t0
        self.contexts.put(ctx)
        self.tensor_store.put(activation_id(ctx.step_id, ctx.microbatch_id, self.stage_index), x,
                              TensorRole.ACTIVATION)
        return out

    def _finish_backward(self, ctx: MicrobatchContext):
        grad = boundary_input_grad(ctx.input) if not self.is_first else None
        ctx.input = ctx.output = None
        return grad

    def forward_loss(self, inp, target, ctx: MicrobatchContext, loss_scale: float = 1.0):
        if not self.is_last:
            raise BoundaryError("forward_loss is only valid on the last stage")
        out = self.forward(inp, ctx)
        ctx.peak_saved_bytes = self.contexts.saved_bytes()
        t0 = time.perf_counter()
        loss = self.loss_fn(out, self.device.move_tensor(target))
        self.contexts.pop(ctx.step_id, ctx.microbatch_id)
        self.tensor_store.discard(activation_id(ctx.step_id, ctx.microbatch_id, self.stage_index))
        (loss * loss_scale).backward()
        self.device.sync_compute()
        ctx.timings["backward"] = time.perf_counter() - t0
        return loss.detach(), self._finish_backward(ctx)

    def loss_backward(self, target, key: tuple[int, int], loss_scale: float = 1.0):
        if not self.is_last:
            raise BoundaryError("loss_backward is only valid on the last stage")
        ctx = self.contexts.pop(*key)
        self.tensor_store.discard(activation_id(*key, self.stage_index))
        t0 = time.perf_counter()
        loss = self.loss_fn(ctx.output, self.device.move_tensor(target))
        (loss * loss_scale).backward()
        self.device.sync_compute()
        ctx.timings["backward"] = time.perf_counter() - t0
        return loss.detach(), self._finish_backward(ctx), ctx

    def backward(self, grad_output, key: tuple[int, int]):
        ctx = self.contexts.pop(*key)
        self.tensor_store.discard(activation_id(*key, self.stage_index))
        t0 = time.perf_counter()
        boundary_backward(ctx.output, self.device.move_tensor(grad_output))
        self.device.sync_compute()
        ctx.timings["backward"] = time.perf_counter() - t0
        return self._finish_backward(ctx), ctx

    def optimizer_step(self) -> float:
        if len(self.contexts):
            raise BoundaryError(f"optimizer step with pending microbatches {self.contexts.pending()}")
        t0 = time.perf_counter()
        if self.optimizer is not None:
            self.optimizer.step()
        self.device.sync_compute()
        return time.perf_counter() - t0

    def zero_grad(self) -> None:
        (self.optimizer or self.module).zero_grad(set_to_none=True)

    def named_gradients(self, prefix: str = "") -> dict[str, torch.Tensor]:
        return {f"{prefix}{n}": p.grad.detach().cpu().clone()
                for n, p in self.module.named_parameters() if p.grad is not None}

    def named_parameters_cpu(self, prefix: str = "") -> dict[str, torch.Tensor]:
        return {f"{prefix}{n}": p.detach().cpu().clone() for n, p in self.module.named_parameters()}

    def memory_report(self) -> dict[str, int]:
        params = sum(p.numel() * p.element_size() for p in self.module.parameters())
        grads = sum(p.grad.numel() * p.grad.element_size() for p in self.module.parameters() if p.grad is not None)
        opt = 0
        if self.optimizer is not None:
            for state in self.optimizer.state.values():
                opt += sum(v.numel() * v.element_size() for v in state.values() if torch.is_tensor(v))
        return {"parameters": params, "gradients": grads, "optimizer_state": opt,
                "saved_activations": self.contexts.saved_bytes()}
