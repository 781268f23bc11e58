"""Single-host multi-process harness for the host runtime, and the single-process oracle.

``run_local_pipeline`` spawns one process per stage and links neighbours by
multiprocessing pipes or loopback TCP (optionally behind an emulated
bandwidth / latency link); each process runs ``run_stage`` and sends its
``StageResult`` back (tensors as ``torch.save`` bytes).  For TCP, stage i
publishes its listening port in a shared integer array and stage i-1 polls
for it: no manager process is needed.

``reference_step`` is the correctness oracle: the whole model in one process,
built with the same per-layer seeds, fed the same ``make_batch(step)``, split
into the same microbatches, each loss scaled by 1/M before backward, one
optimizer step per global step (reference runtime/local.py:192-218).
"""

from __future__ import annotations

import io
import multiprocessing as mp
import os
import queue
import time
import traceback
from dataclasses import dataclass

import torch

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.pipeline import PipelineSettings, StageResult, run_stage
from meshtrain_b200.parallel.stage import Stage, build_optimizer


@dataclass
class LocalStage:
    layers: tuple[int, int]
    device: str | None = "cpu"
    threads: int | None = None  # emulate a slower worker with fewer torch threads


_CAPTURES = ("gradients", "initial_params", "final_params")


def _to_bytes(obj) -> bytes:
    buf = io.BytesIO()
    torch.save(obj, buf)
    return buf.getvalue()


def _from_bytes(data: bytes):
    return torch.load(io.BytesIO(data), weights_only=True)


def _wait_port(ports, index: int, timeout: float) -> int:
    give_up = time.monotonic() + timeout
    while ports[index] == 0:
        if time.monotonic() > give_up:
            raise TimeoutError(f"stage {index} never published its port")
        time.sleep(0.01)
    return ports[index]


def _open_links(index: int, count: int, transport: str, wiring, settings: PipelineSettings):
    """(upstream, downstream) links of stage ``index``."""
    last = count - 1
    if transport == "pipe":
        from meshtrain_b200.networking.transport import PipeTransport

        up = PipeTransport(wiring[index - 1][1]) if index > 0 else None
        down = PipeTransport(wiring[index][0]) if index < last else None
        return up, down
    from meshtrain_b200.networking.tcp import TCPListener, connect

    listener = None
    if index > 0:
        listener = TCPListener("127.0.0.1", 0)
        wiring[index] = listener.port
    down = None
    if index < last:
        port = _wait_port(wiring, index + 1, settings.timeout_s)
        down = connect("127.0.0.1", port, timeout=settings.timeout_s,
                       hello={"job_id": settings.job_id, "stage": index})
    up = None
    if listener is not None:
        up, _ = listener.accept(timeout=settings.timeout_s)
        listener.close()
    return up, down


def _stage_main(index, stages, model_cfg, seed, settings, optimizer, lr, transport, wiring, results,
                capture_params, torch_threads, link_emulation=None):
    os.environ.setdefault("MESHTRAIN_QUIET", "1")
    me = stages[index]
    if me.threads or torch_threads:
        torch.set_num_threads(me.threads or torch_threads)
    from meshtrain_b200.telemetry import EventLogger
    from meshtrain_b200.worker.device import select_device

    worker = f"local{index}"
    up = down = None
    try:
        up, down = _open_links(index, len(stages), transport, wiring, settings)
        if link_emulation is not None:
            from meshtrain_b200.networking.emulation import EmulatedLink

            bandwidth, latency = link_emulation
            up = up and EmulatedLink(up, bandwidth, latency)
            down = down and EmulatedLink(down, bandwidth, latency)
        spec = build_model_spec(model_cfg, seed=seed)
        stage = Stage(spec.build_stage(*me.layers), stage_index=index, num_stages=len(stages),
                      device=select_device(me.device), optimizer=optimizer, lr=lr, loss_fn=spec.loss_fn, name=worker,
                      layer_offset=me.layers[0])
        result = run_stage(stage, spec, settings, upstream=up, downstream=down, worker=worker,
                           logger=EventLogger(worker, settings.job_id), capture_params=capture_params)
        tensors = {name: getattr(result, name) for name in _CAPTURES}
        for name in _CAPTURES:
            setattr(result, name, None)
        results.put(("done", index, (result, _to_bytes(tensors))))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        results.put(("failed", index, f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))
    finally:
        for link in (up, down):
            if link is not None:
                link.close()


def run_local_pipeline(model_cfg: dict, stages: list[LocalStage], settings: PipelineSettings, *, seed: int = 0,
                       optimizer: str = "sgd", lr: float = 0.01, transport: str = "pipe", capture_params: bool = False,
                       torch_threads: int | None = 1, timeout_s: float = 600.0,
                       link_emulation: tuple[float, float] | None = None) -> list[StageResult]:
    """Runs a pipeline as local processes; ``link_emulation=(bytes_per_s, latency_s)`` throttles links."""
    ctx = mp.get_context("spawn")
    n = len(stages)
    if transport == "pipe":
        wiring = [ctx.Pipe(duplex=True) for _ in range(n - 1)]
    elif transport == "tcp":
        wiring = ctx.Array("i", n, lock=False)
    else:
        raise ValueError(f"unknown local transport {transport!r}")
    results = ctx.Queue()
    procs = [ctx.Process(target=_stage_main, name=f"meshtrain-stage{i}",
                         args=(i, stages, model_cfg, seed, settings, optimizer, lr, transport, wiring, results,
                               capture_params, torch_threads, link_emulation)) for i in range(n)]
    for p in procs:
        p.start()
    done: dict[int, StageResult] = {}
    failed: dict[int, str] = {}
    give_up = time.monotonic() + timeout_s
    try:
        while len(done) + len(failed) < n:  # a failure does not stop collection: neighbours fail via ERROR packets
            try:
                tag, index, payload = results.get(timeout=1.0)
            except queue.Empty:
                for i, p in enumerate(procs):  # a process that died before reporting (e.g. at import)
                    if p.exitcode not in (None, 0) and i not in done and i not in failed:
                        failed[i] = f"stage process exited with code {p.exitcode} before reporting"
                if time.monotonic() > give_up:
                    raise TimeoutError(f"local pipeline produced no result within {timeout_s}s") from None
                continue
            if tag == "done":
                result, blob = payload
                for name, value in _from_bytes(blob).items():
                    setattr(result, name, value)
                done[index] = result
            else:
                failed[index] = payload
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()
    if failed:
        raise RuntimeError("local pipeline failed:\n" + "\n".join(f"stage {i}: {e}" for i, e in sorted(failed.items())))
    return [done[i] for i in range(n)]


def reference_step(model_cfg: dict, settings: PipelineSettings, *, seed: int = 0, optimizer: str = "sgd",
                   lr: float = 0.01, steps: int = 1, device: str = "cpu", torch_threads: int | None = 1):
    """Single-process oracle -> (per-step mean losses, last step's grads by '<layer>.<param>', final params).

    On the CPU the oracle runs with ``torch_threads`` intra-op threads - by default
    one, like the stage processes of ``run_local_pipeline`` - so both sides reduce
    in the same order and agree to the last bits, not just to float tolerance.
    """
    previous = torch.get_num_threads()
    if torch_threads and device == "cpu":
        torch.set_num_threads(torch_threads)
    try:
        return _reference_step(model_cfg, settings, seed=seed, optimizer=optimizer, lr=lr, steps=steps,
                               device=device)
    finally:
        torch.set_num_threads(previous)


def _reference_step(model_cfg: dict, settings: PipelineSettings, *, seed: int, optimizer: str, lr: float,
                    steps: int, device: str):
    from meshtrain_b200.worker.device import select_device

    spec = build_model_spec(model_cfg, seed=seed)
    dev = select_device(device)
    model = dev.move_module(spec.build_full())
    opt = build_optimizer(optimizer, model.parameters(), lr)
    M = settings.num_microbatches
    losses: list[float] = []
    grads: dict[str, torch.Tensor] = {}
    for step in range(settings.step_offset, settings.step_offset + steps):
        inputs, targets = spec.make_batch(step, settings.batch_size)
        step_loss = 0.0
        for x, y in zip(inputs.chunk(M), targets.chunk(M)):
            loss = spec.loss_fn(model(dev.move_tensor(x)), dev.move_tensor(y))
            (loss / M).backward()
            step_loss += loss.item()
        losses.append(step_loss / M)
        grads = {name: p.grad.detach().cpu().clone() for name, p in model.named_parameters()}
        opt.step()
        opt.zero_grad(set_to_none=True)
    params = {name: p.detach().cpu().clone() for name, p in model.named_parameters()}
    return losses, grads, params


def global_param_names(stages: list[LocalStage], local: dict[str, torch.Tensor], stage_index: int) -> dict:
    """'<i>.<param>' inside stage ``stage_index`` -> '<start+i>.<param>' in the full model."""
    start = stages[stage_index].layers[0]
    renamed = {}
    for name, tensor in local.items():
        index, rest = name.split(".", 1)
        renamed[f"{start + int(index)}.{rest}"] = tensor
    return renamed
