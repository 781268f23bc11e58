"""What a worker runs: its data-plane port and the executors of one stage assignment.

``DataPlaneServer`` owns the worker's TCP data port.  Every connection opens
with a HELLO: a ``command_kind == "PROBE"`` connection is answered by the link
profiler on a thread of its own; a HELLO that names a job and a stage is an
upstream link waiting for the stage executor that will claim it.  Links and
claims meet in a switchboard of futures keyed by (job, stage), so whichever
side comes first waits for the other (reference worker/executor.py:35-110).

``run_assignment`` executes one START_STAGE command:

* host runtime (``network.tensor_transport`` tcp/pipe): materialise only this
  stage's layers, check them against the planner's memory estimate, dial the
  downstream stage and claim the upstream link, then run ``run_stage``
  (reference worker/executor.py:113-203);
* device engine (``nccl``): join the job's NCCL process group (rank = stage
  index) at its rendezvous and run the GPU engine: flat fp32 state,
  hand-written kernels, activations over NVLink; it emits the same
  STEP_COMPLETE records, and a host watchdog turns a silent or failed peer
  into an error within ``network.timeout_s``.

A memory failure before the first step is raised as ``StageMemoryError``
(carrying what the device really offered) after the stage's memory has been
released, so the coordinator can re-plan.
"""

from __future__ import annotations

import datetime
import json
import threading
import time
from concurrent.futures import Future, TimeoutError as FutureTimeout
from pathlib import Path
from typing import Callable

from meshtrain_b200.config import parse_config
from meshtrain_b200.networking.tcp import TCPListener, TCPTransport, connect
from meshtrain_b200.networking.transport import TransportTimeout
from meshtrain_b200.parallel.memory_check import (StageMemoryError, format_validation, is_oom,
                                                  release_device_memory, validate_engine, validate_stage)
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
        self._board: dict[tuple[str, int], Future] = {}
        self._lock = threading.Lock()
        self._closed = threading.Event()
        self._acceptor = threading.Thread(target=self._accept_forever, daemon=True, name="dataplane-accept")

    def start(self) -> "DataPlaneServer":
        self._acceptor.start()
        return self

    def _slot(self, key: tuple[str, int]) -> Future:
        with self._lock:
            return self._board.setdefault(key, Future())

    def _accept_forever(self) -> None:
        while not self._closed.is_set():
            try:
                link, hello = self.listener.accept(timeout=0.5)
            except TransportTimeout:
                continue
            except Exception as exc:  # noqa: BLE001 - a bad HELLO or token: drop it, keep serving
                if self._closed.is_set():
                    return
                if self.logger is not None:
                    self.logger.log("DATAPLANE_REJECTED", error=str(exc)[:200])
                continue
            if hello.get("command_kind") == "PROBE":
                threading.Thread(target=self._answer_probe, args=(link,), daemon=True, name="probe").start()
            elif "job_id" in hello and "stage" in hello:
                slot = self._slot((str(hello["job_id"]), int(hello["stage"])))
                if slot.done():  # a stale link of the same key: the newest connection wins
                    with self._lock:
                        slot = self._board[(str(hello["job_id"]), int(hello["stage"]))] = Future()
                slot.set_result(link)
            else:
                link.close()

    @staticmethod
    def _answer_probe(link: TCPTransport) -> None:
        try:
            serve_probe(link)
        except Exception:  # noqa: BLE001 - the prober reports its own failure
            pass
        finally:
            link.close()

    def claim(self, job_id: str, from_stage: int, timeout: float, stop_event=None) -> TCPTransport:
        """Waits for the link that stage ``from_stage`` of ``job_id`` opened to this worker."""
        key = (job_id, from_stage)
        slot = self._slot(key)
        give_up = time.monotonic() + timeout
        while True:
            if stop_event is not None and stop_event.is_set():
                raise TransportTimeout("claim cancelled: job stopped")
            left = give_up - time.monotonic()
            if left <= 0:
                raise TransportTimeout(f"stage {from_stage} of job {job_id} never connected "
                                       f"(waited {timeout:.0f}s)")
            try:
                link = slot.result(timeout=min(left, 0.5))
            except FutureTimeout:
                continue
            with self._lock:
                self._board.pop(key, None)
            return link

    def close(self) -> None:
        self._closed.set()
        self.listener.close()
        with self._lock:
            slots, self._board = list(self._board.values()), {}
        for slot in slots:
            if slot.done():
                slot.result().close()


class HostAssignment:
    """One stage of a host-runtime job on this worker."""

    def __init__(self, assignment: dict, cfg, *, device, dataplane, worker_name: str, token: str | None,
                 emit: Callable[[dict], None], stop_event, runs_dir: str):
        self.a, self.cfg, self.device, self.dataplane = assignment, cfg, device, dataplane
        self.worker, self.token, self.emit, self.stop_event = worker_name, token, emit, stop_event
        self.job_id = assignment["job_id"]
        self.data_job = assignment.get("data_job_id", self.job_id)
        self.index, self.count = int(assignment["stage_index"]), int(assignment["num_stages"])
        self.layers = tuple(assignment["layers"])
        self.estimate = assignment.get("memory_estimate")
        self.run_dir = Path(runs_dir) / self.job_id
        self.log = EventLogger(worker_name, self.job_id, jsonl_path=self.run_dir / f"events-{worker_name}.jsonl")
        self.spec = cfg.build_model_spec()
        self.stage = None
        self.links: list = []

    def materialise(self) -> None:
        """Builds this stage's layers on the device and validates its memory (startup OOM -> StageMemoryError)."""
        cfg, device, (start, end) = self.cfg, self.device, self.layers
        try:
            self.stage = Stage(self.spec.build_stage(start, end), stage_index=self.index, num_stages=self.count,
                               device=device, optimizer=cfg.training.optimizer, lr=cfg.training.learning_rate,
                               loss_fn=self.spec.loss_fn, name=self.worker, layer_offset=start)
            if cfg.memory.validate_runtime_usage:
                safety = cfg.memory.safety_factors().get(device.backend, cfg.memory.safety_factor)
                report = validate_stage(self.stage, device, self.estimate, probe=cfg.memory.probe_allocation,
                                        safety_factor=safety)
                self.log.log("MEMORY_VALIDATED", stage=self.index, summary=format_validation(report))
                self.emit({"event": "MEMORY_VALIDATION", "job": self.job_id, "worker": self.worker,
                           "stage": self.index, "phase": "startup", **report})
        except Exception as exc:
            if not is_oom(exc):
                raise
            report = getattr(exc, "report", None) or {"available": device.available_memory()}
            self.stage = None
            release_device_memory(device)
            self.log.log("STAGE_MEMORY_FAILED", stage=self.index, error=str(exc)[:300])
            raise StageMemoryError(f"startup: {exc}", report) from exc

    def connect(self):
        """(upstream, downstream) links: dial the next stage, claim the one the previous stage opened."""
        net = self.cfg.network
        limit = int(net.max_tensor_mb * 1024 ** 2)
        down = up = None
        nxt = self.a.get("downstream")
        if nxt:
            hello = {"job_id": self.data_job, "stage": self.index, **({"token": self.token} if self.token else {})}
            down = connect(nxt["host"], int(nxt["port"]), timeout=net.connect_timeout_s, hello=hello,
                           frame_timeout_s=net.timeout_s, max_payload_bytes=limit, stop_event=self.stop_event)
            self.links.append(down)
            self.log.log("LINK_CONNECTED", direction="downstream", peer=f"{nxt['host']}:{nxt['port']}")
        if self.index > 0:
            if self.dataplane is None:
                raise RuntimeError("a non-first host stage needs a data-plane server")
            up = self.dataplane.claim(self.data_job, self.index - 1, timeout=net.connect_timeout_s,
                                      stop_event=self.stop_event)
            self.links.append(up)
            up.endpoint.sock.settimeout(net.timeout_s)
            up.frame_timeout_s, up.max_payload_bytes = net.timeout_s, limit
            self.log.log("LINK_CONNECTED", direction="upstream", peer=up.peer)
        return up, down

    def _step_hook(self, ckpt_dir: str):
        first = [True]
        training, device, estimate = self.cfg.training, self.device, self.estimate

        def on_step(record: dict) -> None:
            if first[0] and estimate:
                first[0] = False
                peak, need = int(record["memory"].get("device_peak", 0)), int(estimate["required"])
                record["memory_validation"] = {
                    "estimated_required": need, "actual_peak_step0": peak,
                    "peak_estimate_error": (peak - need) / need if need else 0.0,
                    "note": "process RSS" if device.backend == "cpu" else "torch allocator peak"}
            record["job"] = self.job_id
            done = record["step"] + 1
            if training.checkpoint_every and done % training.checkpoint_every == 0:
                from meshtrain_b200.checkpoint import save_host_stage

                save_host_stage(ckpt_dir, self.stage, done, self.layers)
                record["checkpoint"] = {"dir": ckpt_dir, "step": done}
            self.emit(record)
        return on_step

    def run(self) -> StageResult:
        try:
            self.log.log("STAGE_ASSIGNED", stage=self.index, layers=f"{self.layers[0]}-{self.layers[1] - 1}",
                         device=str(self.device.device), attempt=self.a.get("attempt", 0))
            self.materialise()
            up, down = self.connect()
            training = self.cfg.training
            offset = 0
            if training.resume_from:
                from meshtrain_b200.checkpoint import load_host_stage

                offset = load_host_stage(training.resume_from, self.stage, self.layers)
                self.log.log("RESUMED", stage=self.index, step=offset, source=training.resume_from)
            settings = self.cfg.pipeline_settings(self.data_job, step_offset=offset,
                                                  log_microbatch_events=bool(self.a.get("trace", False)),
                                                  trace=bool(self.a.get("timeline", True)))
            ckpt_dir = training.checkpoint_dir or str(self.run_dir / "checkpoints")
            result = run_stage(self.stage, self.spec, settings, upstream=up, downstream=down, worker=self.worker,
                               logger=self.log, metrics_callback=self._step_hook(ckpt_dir),
                               stop_event=self.stop_event)
            if result.timeline is not None:
                self.run_dir.mkdir(parents=True, exist_ok=True)
                (self.run_dir / f"timeline-stage{self.index}-{self.worker}.json").write_text(
                    json.dumps(result.timeline))
            return result
        finally:
            for link in self.links:
                link.close()
            self.stage = None
            release_device_memory(self.device)
            self.log.close()


def run_assignment(assignment: dict, *, device, dataplane: DataPlaneServer | None, worker_name: str,
                   token: str | None = None, metrics_callback: Callable[[dict], None] | None = None,
                   stop_event: threading.Event | None = None, runs_dir: str = "runs") -> StageResult:
    """Executes one START_STAGE command on this worker."""
    cfg = parse_config(assignment["config"])
    if cfg.network.tensor_transport == "nccl":
        return run_device_assignment(assignment, device=device, worker_name=worker_name,
                                     metrics_callback=metrics_callback, stop_event=stop_event, runs_dir=runs_dir)
    return HostAssignment(assignment, cfg, device=device, dataplane=dataplane, worker_name=worker_name, token=token,
                          emit=metrics_callback or (lambda record: None), stop_event=stop_event,
                          runs_dir=runs_dir).run()


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
    launched = False
    watch = None
    from meshtrain_b200.parallel.watchdog import PeerFailure, groups_abandoned

    try:
        chunk_ranges = [tuple(r) for r in assignment.get("chunk_ranges") or []] or None
        if n > 1:
            backend = "nccl" if dev.type == "cuda" else "gloo"
            kw = {"device_id": dev} if backend == "nccl" else {}
            if dev.type == "cuda":
                torch.cuda.set_device(dev)
            dist.init_process_group(backend, init_method=f"tcp://{rv['host']}:{rv['port']}", rank=idx, world_size=n,
                                    timeout=datetime.timedelta(seconds=cfg.network.timeout_s), **kw)
            joined = True
        links = StageLinks(idx, n, ring=chunk_ranges is not None) if n > 1 else None
        if links is not None and dev.type == "cuda":
            links.warmup(dev)
        if links is not None:
            from meshtrain_b200.parallel.watchdog import PeerWatch

            watch = PeerWatch(idx, n, groups=links.groups(), timeout_s=cfg.network.timeout_s,
                              prefix=f"meshtrain/{assignment.get('data_job_id', job_id)}")
        offload = None
        from meshtrain_b200.parallel.placement import config_mode

        state_offload = assignment.get("state_offload")  # the coordinator's tier decision (offload "auto")
        if state_offload is None:
            state_offload = config_mode(cfg.offload) == "host"
        if state_offload:
            from meshtrain_b200.parallel.offload import HostOffload

            offload = HostOffload(prefetch_ahead=cfg.offload.prefetch_ahead, chunk_mb=cfg.offload.chunk_mb,
                                  device_budget_gb=cfg.offload.device_budget_gb)
        from meshtrain_b200.coordinator.scheduler import recompute_units

        recompute = recompute_units(cfg) or None
        try:
            eng = PipelineEngine(spec, layer_range=None if chunk_ranges else (start, end), chunk_ranges=chunk_ranges,
                                 stage=idx, num_stages=n, device=dev,
                                 num_microbatches=M, schedule=cfg.pipeline.schedule,
                                 max_inflight=cfg.pipeline.max_inflight_microbatches, optimizer=tc.optimizer,
                                 lr=tc.learning_rate, weight_decay=tc.weight_decay, links=links,
                                 init_on_device=dev.type == "cuda", offload=offload, microbatch_size=mbs,
                                 recompute=recompute)
            if cfg.memory.validate_runtime_usage:
                safety = cfg.memory.safety_factors().get(device.backend, cfg.memory.safety_factor)
                report = validate_engine(eng, device, assignment.get("memory_estimate"),
                                         probe=cfg.memory.probe_allocation, safety_factor=safety)
                logger.log("MEMORY_VALIDATED", stage=idx, summary=format_validation(report))
                emit({"event": "MEMORY_VALIDATION", "job": job_id, "worker": worker_name, "stage": idx,
                      "phase": "startup", **report})
        except Exception as exc:
            if watch is not None:
                watch.startup_gate(f"{type(exc).__name__}: {exc}", cfg.network.timeout_s)
            if not is_oom(exc):
                raise
            report = getattr(exc, "report", None) or {"available": device.available_memory()}
            eng = None
            release_device_memory(device)
            logger.log("STAGE_MEMORY_FAILED", stage=idx, error=str(exc)[:300])
            raise StageMemoryError(f"startup: {exc}", report) from exc
        if watch is not None:
            watch.startup_gate(None, cfg.network.timeout_s)  # every rank built and validated its stage
        logger.log("STAGE_ASSIGNED", stage=idx, layers=f"{start}-{end - 1}", device=str(dev), engine="device")
        seq = getattr(spec, "seq_len", 1)
        offset = 0
        if tc.resume_from:
            from meshtrain_b200.checkpoint import load_stage_checkpoint

            offset = load_stage_checkpoint(tc.resume_from, eng)
            logger.log("RESUMED", stage=idx, step=offset, source=tc.resume_from)
        ckpt_dir = tc.checkpoint_dir or str(Path(runs_dir) / job_id / "checkpoints")
        launched = True  # from here on NCCL work toward a peer may be in flight
        for local_step in range(tc.steps):
            if stop_event is not None and stop_event.is_set():
                raise RuntimeError("stopped")
            if watch is not None:
                watch.check()  # a failed peer stops this stage before it launches anything
            step = offset + local_step
            x, y = spec.make_batch(step, tc.batch_size) if (eng.is_first or eng.is_last) else (None, None)
            wall0 = timeline.now()
            t0 = time.perf_counter()
            try:
                st = eng.train_step(step, x if eng.is_first else None, y if eng.is_last else None, timed=True)
            except Exception as exc:
                if watch is not None:
                    peer = watch.peer_failure()
                    if peer is not None:
                        raise PeerFailure(peer) from exc
                    watch.report(f"step {step}: {type(exc).__name__}: {exc}")
                raise
            if watch is not None:
                watch.beat(step)
            step_s = time.perf_counter() - t0
            dm = device.memory_stats()
            rec = {"event": "STEP_COMPLETE", "job": job_id, "worker": worker_name, "stage": idx,
                   "backend": device.backend, "engine": "device", "step": step, "schedule": cfg.pipeline.schedule,
                   "step_s": step_s, "device_step_ms": st.step_ms, "forward_s": st.forward_ms / 1e3,
                   "backward_s": st.backward_ms / 1e3, "optimizer_s": st.optimizer_ms / 1e3,
                   "compute_s": st.compute_ms / 1e3, "comm_s": st.wait_ms / 1e3,
                   "exposed_communication_s": st.exposed_p2p_ms / 1e3, "bubble_fraction": st.bubble_fraction,
                   "exposed_p2p_ms": st.exposed_p2p_ms, "idle_s": max(0.0, step_s - st.step_ms / 1e3),
                   "p2p_wait_ms": st.recv_wait_ms, "p2p_send_ms": st.send_ms, "side_stream_ms": st.side_ms,
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
    except Exception as exc:
        if watch is not None and not isinstance(exc, PeerFailure):
            watch.report(f"{type(exc).__name__}: {exc}")  # e.g. a startup OOM: the other stages stop too
        raise
    finally:
        if watch is not None:
            watch.close()
            if watch.reason is not None and joined and launched:
                watch.abandon_groups()  # NCCL work toward a failed peer never completes
        if joined and dist.is_initialized() and not groups_abandoned():
            dist.destroy_process_group()
        release_device_memory(device)
        logger.close()
