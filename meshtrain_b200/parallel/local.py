"""Single-host multi-process pipeline harness and the single-process oracle.

``run_local_pipeline`` starts one spawned process per stage, links them with
multiprocessing pipes or loopback TCP (optionally behind an emulated
bandwidth/latency link) and runs ``run_stage`` in each; results come back as
bytes.  ``reference_step`` is the correctness oracle: the whole model in one
process with the same per-layer seeds, batches, microbatch split and ``loss/M``
accumulation (reference runtime/local.py:28-228).
"""

from __future__ import annotations

import multiprocessing as mp
import os
import queue
import time
import traceback
from dataclasses import dataclass

import torch

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.networking.serialization import bytes_to_tensor, tensor_to_bytes
from meshtrain_b200.networking.packet import DTYPE_NAMES
from meshtrain_b200.parallel.pipeline import PipelineSettings, StageResult, run_stage
from meshtrain_b200.parallel.stage import Stage, build_optimizer


@dataclass
class LocalStage:
    layers: tuple[int, int]
    device: str | None = "cpu"
    threads: int | None = None  # emulate a slower worker with fewer torch threads


_TENSOR_FIELDS = ("gradients", "initial_params", "final_params")


def _pack(res: StageResult) -> StageResult:
    for f in _TENSOR_FIELDS:
        d = getattr(res, f)
        if d is not None:
            setattr(res, f, {k: (tensor_to_bytes(v), DTYPE_NAMES[v.dtype], tuple(v.shape)) for k, v in d.items()})
    return res


def _unpack(res: StageResult) -> StageResult:
    for f in _TENSOR_FIELDS:
        d = getattr(res, f)
        if d is not None:
            setattr(res, f, {k: bytes_to_tensor(*v) for k, v in d.items()})
    return res


class _PortBoard:
    """Lets the TCP child of stage i learn the listening port of stage i+1."""

    def __init__(self, shared):
        self.d = shared

    def get_port(self, index: int, timeout: float = 30.0) -> int:
        t0 = time.time()
        while index not in self.d:
            if time.time() - t0 > timeout:
                raise TimeoutError(f"stage {index} never published its port")
            time.sleep(0.01)
        return self.d[index]


def _stage_process(index, stages, model_cfg, seed, settings, optimizer, lr, transport, links, results,
                   capture_params, torch_threads, link_emulation=None):
    os.environ.setdefault("MESHTRAIN_QUIET", "1")
    threads = stages[index].threads or torch_threads
    if threads:
        torch.set_num_threads(threads)
    from meshtrain_b200.telemetry import EventLogger
    from meshtrain_b200.worker.device import select_device

    up = down = None
    worker = f"local{index}"
    try:
        spec = build_model_spec(model_cfg, seed=seed)
        st = stages[index]
        if transport == "pipe":
            from meshtrain_b200.networking.transport import PipeTransport

            up = PipeTransport(links[index - 1][1]) if index > 0 else None
            down = PipeTransport(links[index][0]) if index < len(stages) - 1 else None
        else:
            from meshtrain_b200.networking.tcp import TCPListener, connect

            listener = None
            if index > 0:
                listener = TCPListener("127.0.0.1", 0)
                results.put(("port", index, listener.port))
            if index < len(stages) - 1:
                down = connect("127.0.0.1", links.get_port(index + 1), timeout=settings.timeout_s,
                               hello={"job_id": settings.job_id, "stage": index})
            if listener is not None:
                up, _ = listener.accept(timeout=settings.timeout_s)
                listener.close()
        if link_emulation is not None:
            from meshtrain_b200.networking.emulation import EmulatedLink

            bw, lat = link_emulation
            up = EmulatedLink(up, bw, lat) if up is not None else None
            down = EmulatedLink(down, bw, lat) if down is not None else None
        stage = Stage(spec.build_stage(*st.layers), stage_index=index, num_stages=len(stages),
                      device=select_device(st.device), optimizer=optimizer, lr=lr, loss_fn=spec.loss_fn, name=worker,
                      layer_offset=st.layers[0])
        res = run_stage(stage, spec, settings, upstream=up, downstream=down, worker=worker,
                        logger=EventLogger(worker, settings.job_id), capture_params=capture_params)
        results.put(("result", index, _pack(res)))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        results.put(("error", index, f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))
    finally:
        for link in (up, down):
            if link is not None:
                link.close()


def run_local_pipeline(model_cfg: dict, stages: list[LocalStage], settings: PipelineSettings, *, seed: int = 0,
                       optimizer: str = "sgd", lr: float = 0.01, transport: str = "pipe", capture_params: bool = False,
                       torch_threads: int | None = 1, timeout_s: float = 600.0,
                       link_emulation: tuple[float, float] | None = None) -> list[StageResult]:
    """Run a pipeline as local processes; ``link_emulation=(bytes_per_s, latency_s)`` throttles links."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    manager = None
    if transport == "pipe":
        links = [ctx.Pipe(duplex=True) for _ in range(len(stages) - 1)]
    elif transport == "tcp":
        manager = ctx.Manager()
        links = _PortBoard(manager.dict())
    else:
        raise ValueError(f"unknown local transport {transport!r}")
    procs = [ctx.Process(target=_stage_process, name=f"meshtrain-stage{i}",
                         args=(i, stages, model_cfg, seed, settings, optimizer, lr, transport, links, results,
                               capture_params, torch_threads, link_emulation))
             for i in range(len(stages))]
    for p in procs:
        p.start()
    out: dict[int, StageResult] = {}
    errors: dict[int, str] = {}
    try:
        while len(out) + len(errors) < len(stages):
            try:
                kind, index, payload = results.get(timeout=timeout_s)
            except queue.Empty:
                raise TimeoutError(f"local pipeline produced no result within {timeout_s}s") from None
            if kind == "port":
                links.d[index] = payload
            elif kind == "result":
                out[index] = _unpack(payload)
            else:
                errors[index] = payload  # neighbours fail through ERROR packets / timeouts; keep collecting
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()
        if manager is not None:
            manager.shutdown()
    if errors:
        raise RuntimeError("local pipeline failed:\n" + "\n".join(f"stage {i}: {e}" for i, e in sorted(errors.items())))
    return [out[i] for i in range(len(stages))]


def reference_step(model_cfg: dict, settings: PipelineSettings, *, seed: int = 0, optimizer: str = "sgd",
                   lr: float = 0.01, steps: int = 1, device: str = "cpu"):
    """Single-process oracle -> (losses, last-step grads '<layer>.<param>', final params)."""
    from meshtrain_b200.worker.device import select_device

    spec = build_model_spec(model_cfg, seed=seed)
    dev = select_device(device)
    model = dev.move_module(spec.build_full())
    opt = build_optimizer(optimizer, model.parameters(), lr)
    M = settings.num_microbatches
    losses, grads = [], {}
    for local_step in range(steps):
        step = settings.step_offset + local_step
        x, y = spec.make_batch(step, settings.batch_size)
        total = 0.0
        for xm, ym in zip(x.chunk(M), y.chunk(M)):
            loss = spec.loss_fn(model(dev.move_tensor(xm)), dev.move_tensor(ym))
            (loss / M).backward()
            total += loss.item()
        losses.append(total / M)
        grads = {n: p.grad.detach().cpu().clone() for n, p in model.named_parameters()}
        opt.step()
        opt.zero_grad(set_to_none=True)
    params = {n: p.detach().cpu().clone() for n, p in model.named_parameters()}
    return losses, grads, params


def global_param_names(stages: list[LocalStage], local: dict[str, torch.Tensor], stage_index: int) -> dict:
    """'0.weight' inside stage i -> '<start+0>.weight' in the full model."""
    start = stages[stage_index].layers[0]
    out = {}
    for name, t in local.items():
        idx, rest = name.split(".", 1)
        out[f"{int(idx) + start}.{rest}"] = t
    return out
