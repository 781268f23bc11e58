"""Worker-side execution: the data-plane listener and the two stage executors.

``DataPlaneServer`` owns the worker's TCP port.  Each incoming connection opens
with a HELLO: ``command_kind == "PROBE"`` is answered by the link profiler, a
HELLO carrying ``job_id`` + ``stage`` is parked until the executor of the next
stage claims it as its upstream link (reference worker/executor.py:35-110).

``run_assignment`` executes one START_STAGE command:

* host path (``network.tensor_transport`` tcp/pipe): the reference's runtime -
  materialise only this stage's layers, validate memory against the planner's
  estimate, connect links, run ``run_stage`` (reference worker/executor.py:113-203);
* device path (``nccl``): the stage joins a NCCL process group at the job's
  rendezvous (rank = stage index) and runs the device engine - flat fp32
  state, hand-written kernels, activations over NVLink - emitting the same
  STEP_COMPLETE records.

Memory failures before the first step surface as ``StageMemoryError`` (with the
measured capacity) after the device memory has been released, so the
coordinator can replan.
"""

from __future__ import annotations

import datetime
import json
import threading
import time
from pathlib import Path
from typing import Callable

from meshtrain_b200.config import parse_config
from meshtrain_b200.networking.tcp import TCPListener, TCPTransport, connect
from meshtrain_b200.networking.transport import TransportTimeout
from meshtrain_b200.parallel.memory_check import (StageMemoryError, format_validation, is_oom,
                                                  release_device_memory, validate_stage)
from meshtrain_b200.parallel.pipeline import StageResult, run_stage
from meshtrain_b200.parallel.stage import Stage
from meshtrain_b200.profiler.network import serve_probe
from meshtrain_b200.telemetry import EventLogger
from meshtrain_b200.utils.timeline import Timeline


class DataPlaneServer:
    def __init__(self, host: str = "0.0.0.0", port: int = 29500, *, token: str | None = None,
                 max_payload_bytes: int = 2 * 1024 ** 3, logger: EventLogger | None = None):
        self.listener = TCPListener(host, port, token=token, max_payload_bytes=max_payload_bytes)
        self.port = self.listener.port
        self.logger = logger
        self._parked: dict[tuple[str, int], TCPTransport] = {}
        self._cv = threading.Condition()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._accept_loop, daemon=True, name="dataplane-accept")

    def start(self) -> "DataPlaneServer":
        self._thread.start()
        return self

    def _accept_loop(self) -> None:
        while not self._stop.is_set():
            try:
                link, hello = self.listener.accept(timeout=0.5)
            except TransportTimeout:
                continue
            except Exception as exc:  # noqa: BLE001 - bad HELLO or token: drop it, keep serving
                if self._stop.is_set():
                    return
                if self.logger is not None:
                    self.logger.log("DATAPLANE_REJECTED", error=str(exc)[:200])
                continue
            if hello.get("command_kind") == "PROBE":
                threading.Thread(target=self._probe, args=(link,), daemon=True, name="probe").start()
            elif "job_id" in hello and "stage" in hello:
                with self._cv:
                    self._parked[(str(hello["job_id"]), int(hello["stage"]))] = link
                    self._cv.notify_all()
            else:
                link.close()

    @staticmethod
    def _probe(link: TCPTransport) -> None:
        try:
            serve_probe(link)
        except Exception:  # noqa: BLE001 - the prober reports its own failure
            pass
        finally:
            link.close()

    def claim(self, job_id: str, from_stage: int, timeout: float, stop_event=None) -> TCPTransport:
        deadline = time.monotonic() + timeout
        key = (job_id, from_stage)
        with self._cv:
            while key not in self._parked:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TransportTimeout(f"stage {from_stage} of job {job_id} never connected "
                                           f"(waited {timeout:.0f}s)")
                if stop_event is not None and stop_event.is_set():
                    raise TransportTimeout("claim cancelled: job stopped")
                self._cv.wait(min(left, 0.5))
            return self._parked.pop(key)

    def close(self) -> None:
        self._stop.set()
        self.listener.close()
        with self._cv:
            for link in self._parked.values():
                link.close()
            self._parked.clear()


def run_assignment(assignment: dict, *, device, dataplane: DataPlaneServer | None, worker_name: str,
                   token: str | None = None, metrics_callback: Callable[[dict], None] | None = None,
                   stop_event: threading.Event | None = None, runs_dir: str = "runs") -> StageResult:
    cfg = parse_config(assignment["config"])
    if cfg.network.tensor_transport == "nccl":
        return run_device_assignment(assignment, device=device, worker_name=worker_name,
                                     metrics_callback=metrics_callback, stop_event=stop_event, runs_dir=runs_dir)
    job_id = assignment["job_id"]
    data_job = assignment.get("data_job_id", job_id)
    idx, n = int(assignment["stage_index"]), int(assignment["num_stages"])
    start, end = assignment["layers"]
    run_dir = Path(runs_dir) / job_id
    logger = EventLogger(worker_name, job_id, jsonl_path=run_dir / f"events-{worker_name}.jsonl")
    spec = cfg.build_model_spec()
    estimate = assignment.get("memory_estimate")
    emit = metrics_callback or (lambda rec: None)
    up = down = None
    stage = None
    try:
        logger.log("STAGE_ASSIGNED", stage=idx, layers=f"{start}-{end - 1}", device=str(device.device),
                   attempt=assignment.get("attempt", 0))
        try:
            stage = Stage(spec.build_stage(start, end), stage_index=idx, num_stages=n, device=device,
                          optimizer=cfg.training.optimizer, lr=cfg.training.learning_rate, loss_fn=spec.loss_fn,
                          name=worker_name, layer_offset=start)
            if cfg.memory.validate_runtime_usage:
                sf = cfg.memory.safety_factors().get(device.backend, cfg.memory.safety_factor)
                report = validate_stage(stage, device, estimate, probe=cfg.memory.probe_allocation, safety_factor=sf)
                logger.log("MEMORY_VALIDATED", stage=idx, summary=format_validation(report))
                emit({"event": "MEMORY_VALIDATION", "job": job_id, "worker": worker_name, "stage": idx,
                      "phase": "startup", **report})
        except Exception as exc:
            if not is_oom(exc):
                raise
            rep = getattr(exc, "report", None) or {"available": device.available_memory()}
            stage = None
            release_device_memory(device)
            logger.log("STAGE_MEMORY_FAILED", stage=idx, error=str(exc)[:300])
            raise StageMemoryError(f"startup: {exc}", rep) from exc
        max_bytes = int(cfg.network.max_tensor_mb * 1024 ** 2)
        if assignment.get("downstream"):
            d = assignment["downstream"]
            hello = {"job_id": data_job, "stage": idx}
            if token is not None:
                hello["token"] = token
            down = connect(d["host"], int(d["port"]), timeout=cfg.network.connect_timeout_s, hello=hello,
                           frame_timeout_s=cfg.network.timeout_s, max_payload_bytes=max_bytes, stop_event=stop_event)
            logger.log("LINK_CONNECTED", direction="downstream", peer=f"{d['host']}:{d['port']}")
        if idx > 0:
            if dataplane is None:
                raise RuntimeError("a non-first host stage needs a data-plane server")
            up = dataplane.claim(data_job, idx - 1, timeout=cfg.network.connect_timeout_s, stop_event=stop_event)
            up.frame_timeout_s = cfg.network.timeout_s
            up.max_payload_bytes = max_bytes
            logger.log("LINK_CONNECTED", direction="upstream", peer=up.peer)
        tc = cfg.training
        ckpt_dir = tc.checkpoint_dir or str(run_dir / "checkpoints")
        offset = 0
        if tc.resume_from:
            from meshtrain_b200.checkpoint import load_host_stage

            offset = load_host_stage(tc.resume_from, stage, (start, end))
            logger.log("RESUMED", stage=idx, step=offset, source=tc.resume_from)
        settings = cfg.pipeline_settings(data_job, log_microbatch_events=bool(assignment.get("trace", False)),
                                         trace=bool(assignment.get("timeline", True)), step_offset=offset)
        first = {"done": False}

        def on_step(rec: dict) -> None:
            if not first["done"] and estimate:
                first["done"] = True
                peak = int(rec["memory"].get("device_peak", 0))
                need = int(estimate["required"])
                rec["memory_validation"] = {"estimated_required": need, "actual_peak_step0": peak,
                                            "peak_estimate_error": (peak - need) / need if need else 0.0,
                                            "note": "process RSS" if device.backend == "cpu" else
                                            "torch allocator peak"}
            rec["job"] = job_id
            done_steps = rec["step"] + 1
            if tc.checkpoint_every and done_steps % tc.checkpoint_every == 0:
                from meshtrain_b200.checkpoint import save_host_stage

                save_host_stage(ckpt_dir, stage, done_steps, (start, end))
                rec["checkpoint"] = {"dir": ckpt_dir, "step": done_steps}
            emit(rec)

        result = run_stage(stage, spec, settings, upstream=up, downstream=down, worker=worker_name, logger=logger,
                           metrics_callback=on_step, stop_event=stop_event)
        if result.timeline is not None:
            run_dir.mkdir(parents=True, exist_ok=True)
            (run_dir / f"timeline-stage{idx}-{worker_name}.json").write_text(json.dumps(result.timeline))
        return result
    finally:
        for link in (up, down):
            if link is not None:
                link.close()
        stage = None
        release_device_memory(device)
        logger.close()


def run_device_assignment(assignment: dict, *, device, worker_name: str,
                          metrics_callback: Callable[[dict], None] | None = None,
                          stop_event: threading.Event | None = None, runs_dir: str = "runs") -> StageResult:
    """One stage of a device-engine job: NCCL p2p between the job's GPUs (gloo when on CPU)."""
    import torch
    import torch.distributed as dist

    from meshtrain_b200.parallel.engine import PipelineEngine
    from meshtrain_b200.parallel.p2p import StageLinks

    cfg = parse_config(assignment["config"])
    job_id = assignment["job_id"]
    idx, n = int(assignment["stage_index"]), int(assignment["num_stages"])
    start, end = assignment["layers"]
    rv = assignment.get("rendezvous")
    if n > 1 and not rv:
        raise ValueError("a multi-stage device job needs a rendezvous address")
    logger = EventLogger(worker_name, job_id, jsonl_path=Path(runs_dir) / job_id / f"events-{worker_name}.jsonl")
    emit = metrics_callback or (lambda rec: None)
    tc = cfg.training
    M = tc.num_microbatches
    mbs = tc.microbatch_size or tc.batch_size
    spec = cfg.build_model_spec()
    result = StageResult(idx, worker_name)
    timeline = Timeline(worker_name, idx)
    dev = device.device
    joined = False
    try:
        if n > 1:
            backend = "nccl" if dev.type == "cuda" else "gloo"
            kw = {"device_id": dev} if backend == "nccl" else {}
            if dev.type == "cuda":
                torch.cuda.set_device(dev)
            dist.init_process_group(backend, init_method=f"tcp://{rv['host']}:{rv['port']}", rank=idx, world_size=n,
                                    timeout=datetime.timedelta(seconds=cfg.network.timeout_s), **kw)
            joined = True
        links = StageLinks(idx, n) if n > 1 else None
        if links is not None and dev.type == "cuda":
            links.warmup(dev)
        offload = None
        if cfg.offload.params == "host" or cfg.offload.optimizer == "host":
            from meshtrain_b200.parallel.offload import HostOffload

            offload = HostOffload(prefetch_ahead=cfg.offload.prefetch_ahead, chunk_mb=cfg.offload.chunk_mb)
        try:
            eng = PipelineEngine(spec, layer_range=(start, end), stage=idx, num_stages=n, device=dev,
                                 num_microbatches=M, schedule=cfg.pipeline.schedule,
                                 max_inflight=cfg.pipeline.max_inflight_microbatches, optimizer=tc.optimizer,
                                 lr=tc.learning_rate, weight_decay=tc.weight_decay, links=links,
                                 init_on_device=dev.type == "cuda", offload=offload, microbatch_size=mbs)
        except Exception as exc:
            if not is_oom(exc):
                raise
            release_device_memory(device)
            raise StageMemoryError(f"startup: {exc}", {"available": device.available_memory()}) from exc
        logger.log("STAGE_ASSIGNED", stage=idx, layers=f"{start}-{end - 1}", device=str(dev), engine="device")
        seq = getattr(spec, "seq_len", 1)
        offset = 0
        if tc.resume_from:
            from meshtrain_b200.checkpoint import load_stage_checkpoint

            offset = load_stage_checkpoint(tc.resume_from, eng)
            logger.log("RESUMED", stage=idx, step=offset, source=tc.resume_from)
        ckpt_dir = tc.checkpoint_dir or str(Path(runs_dir) / job_id / "checkpoints")
        for local_step in range(tc.steps):
            if stop_event is not None and stop_event.is_set():
                raise RuntimeError("stopped")
            step = offset + local_step
            x, y = spec.make_batch(step, tc.batch_size) if (eng.is_first or eng.is_last) else (None, None)
            wall0 = timeline.now()
            t0 = time.perf_counter()
            st = eng.train_step(step, x if eng.is_first else None, y if eng.is_last else None, timed=True)
            step_s = time.perf_counter() - t0
            dm = device.memory_stats()
            rec = {"event": "STEP_COMPLETE", "job": job_id, "worker": worker_name, "stage": idx,
                   "backend": device.backend, "engine": "device", "step": step, "schedule": cfg.pipeline.schedule,
                   "step_s": step_s, "device_step_ms": st.step_ms, "forward_s": st.forward_ms / 1e3,
                   "backward_s": st.backward_ms / 1e3, "optimizer_s": st.optimizer_ms / 1e3,
                   "compute_s": st.compute_ms / 1e3, "comm_s": st.wait_ms / 1e3,
                   "exposed_communication_s": st.exposed_p2p_ms / 1e3, "bubble_fraction": st.bubble_fraction,
                   "exposed_p2p_ms": st.exposed_p2p_ms, "idle_s": max(0.0, step_s - st.step_ms / 1e3),
                   "bytes_sent": st.bytes_sent, "bytes_received": st.bytes_received,
                   "memory": {"device_allocated": dm.get("allocated", 0), "device_peak": dm.get("peak_allocated", 0),
                              "device_total": dm.get("total", 0), **eng.flat.bytes_by_role()}}
            if eng.is_last:
                loss = float(st.loss) / M
                rec["loss"] = loss
                rec["samples_per_s"] = tc.batch_size / step_s
                rec["tokens_per_s"] = tc.batch_size * seq / step_s
                result.losses.append(loss)
            timeline.add_device_spans(st.spans, step, wall0)
            if tc.checkpoint_every and (step + 1) % tc.checkpoint_every == 0:
                from meshtrain_b200.checkpoint import save_stage_checkpoint

                save_stage_checkpoint(ckpt_dir, eng, step + 1)
                rec["checkpoint"] = {"dir": ckpt_dir, "step": step + 1}
            result.step_metrics.append(rec)
            emit(rec)
            if local_step % tc.log_every == 0 or local_step == tc.steps - 1:
                logger.log("STEP_COMPLETE", step, None, step_s=step_s, device_ms=st.step_ms,
                           bubble=st.bubble_fraction, **({"loss": rec["loss"]} if "loss" in rec else {}))
        result.timeline = timeline.export()
        if links is not None:
            dist.barrier()
        return result
    finally:
        if joined and dist.is_initialized():
            dist.destroy_process_group()
        release_device_memory(device)
        logger.close()
