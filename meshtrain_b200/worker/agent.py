"""The worker process behind ``meshtrain join <coordinator>``.

A ``WorkerAgent`` serves one device.  At start it selects the device adapter
(``cuda:N`` / mps / cpu), probes its capabilities once, opens its data-plane
port, registers with the coordinator (cluster token) and starts heartbeats.
Then it long-polls for commands and runs each on a thread of its own:

    RUN_BENCHMARK    compute benchmark of the device     -> benchmark_result event
    PROBE_NETWORK    link probe to another worker         -> probe_result event
    START_STAGE      run one stage of a job attempt       -> stage_metrics / stage_done / stage_error events
    STOP_JOB         stop the named job (or one attempt of it)

Commands that fail report ``command_error`` with their request id.  A
START_STAGE for a new attempt of a job first stops the previous attempt on
this worker and waits for it, so its device memory is free (startup-OOM
replanning).  On a multi-GPU box run one agent per GPU (``--device cuda:0`` ...
``cuda:7``); agents of a box report one host id, which lets the planner give
their stages NCCL links.  Same commands and events as the reference's worker
(worker/worker.py:35-215).
"""

from __future__ import annotations

import socket
import threading
import time
import traceback

import httpx

from meshtrain_b200.networking.control import ControlClient
from meshtrain_b200.parallel.memory_check import is_oom
from meshtrain_b200.profiler.benchmark import benchmark_device
from meshtrain_b200.profiler.hardware import detect_hardware
from meshtrain_b200.profiler.network import measure_link
from meshtrain_b200.telemetry import EventLogger
from meshtrain_b200.worker.device import DeviceAdapter, select_device
from meshtrain_b200.worker.executor import DataPlaneServer, run_assignment
from meshtrain_b200.worker.heartbeat import Heartbeat

TIMELINE_SPANS_SENT = 20_000


def guess_advertise_host(coordinator_base: str) -> str:
    """The local address this machine uses towards the coordinator: what peers should dial."""
    host = coordinator_base.split("://", 1)[-1].rsplit(":", 1)[0]
    try:
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as probe:
            probe.connect((host, 9))  # UDP connect sends nothing; it only picks the route
            return probe.getsockname()[0]
    except OSError:
        return "127.0.0.1"


class StageRuns:
    """Stage executions on this worker, keyed by (job id, attempt), each with a stop flag."""

    def __init__(self):
        self._runs: dict[tuple[str, int], tuple[threading.Event, threading.Thread]] = {}
        self._lock = threading.Lock()

    def begin(self, job_id: str, attempt: int) -> threading.Event:
        stop = threading.Event()
        with self._lock:
            self._runs[(job_id, attempt)] = (stop, threading.current_thread())
        return stop

    def end(self, job_id: str, attempt: int) -> None:
        with self._lock:
            self._runs.pop((job_id, attempt), None)

    def stop(self, job_id: str | None = None, attempt: int | None = None, before: int | None = None) -> list:
        """Sets the stop flag of matching runs; returns their (key, thread) pairs."""
        with self._lock:
            hits = [(key, thread) for key, (flag, thread) in self._runs.items()
                    if (job_id is None or key[0] == job_id) and (attempt is None or key[1] == attempt)
                    and (before is None or key[1] < before)]
            for key, _thread in hits:
                self._runs[key][0].set()
        return hits


class WorkerAgent:
    def __init__(self, coordinator: str, token: str, *, device: str | None = None, name: str | None = None,
                 data_port: int = 29500, bind_host: str = "0.0.0.0", advertise_host: str | None = None,
                 runs_dir: str = "runs", quick_benchmark: bool = False, client: ControlClient | None = None):
        self.client = client or ControlClient(coordinator, token)
        self.token = token
        self.device: DeviceAdapter = select_device(device)
        self.hardware = detect_hardware()
        self.hardware.setdefault("host_id", self.hardware.get("hostname"))
        default_name = self.hardware.get("hostname") or "worker"
        if name is None and self.device.backend == "cuda":
            default_name = f"{default_name}-gpu{self.device.index}"
        self.name = name or default_name
        self.log = EventLogger(self.name, "-")
        self.runs_dir = runs_dir
        self.quick_benchmark = quick_benchmark
        self.dataplane = DataPlaneServer(bind_host, data_port, token=token, logger=self.log).start()
        self.capabilities = self.device.capabilities()
        self.advertise_host = advertise_host or guess_advertise_host(self.client.base)
        self.worker_id: str | None = None
        self.heartbeat: Heartbeat | None = None
        self.stages = StageRuns()
        self._halt = threading.Event()
        self.handlers = {"RUN_BENCHMARK": self._benchmark, "PROBE_NETWORK": self._probe,
                         "START_STAGE": self._start_stage, "STOP_JOB": self._stop_job}

    # ---------------------------------------------------------------- registration
    def register(self) -> str:
        reply = self.client.register({
            "name": self.name, "hardware": self.hardware, "backend": self.device.backend,
            "device": self.device.describe(), "data_host": self.advertise_host, "data_port": self.dataplane.port,
            "capabilities": self.capabilities})
        self.worker_id = self.log.worker = reply["worker_id"]
        self.log.log("REGISTERED", coordinator=self.client.base, backend=self.device.backend,
                     device=self.device.name(), data=f"{self.advertise_host}:{self.dataplane.port}")
        if self.heartbeat is None:
            self.heartbeat = Heartbeat(
                self._send_heartbeat, every_s=reply.get("heartbeat_interval_s", 3.0), forgotten=self._register_again,
                failed=lambda exc: self.log.log("HEARTBEAT_FAILED", error=str(exc)[:200])).start()
        return self.worker_id

    def _register_again(self) -> None:
        self.log.log("REREGISTER", reason="coordinator does not know this worker")
        try:
            self.register()
        except httpx.HTTPError as exc:
            self.log.log("REGISTER_FAILED", error=str(exc)[:200])

    def _memory_snapshot(self) -> dict:
        try:
            stats = self.device.memory_stats()
        except Exception:  # noqa: BLE001 - a heartbeat without memory is still a heartbeat
            return {}
        return {k: v for k, v in stats.items() if isinstance(v, (int, bool))}

    def _send_heartbeat(self) -> bool:
        """One heartbeat with the device's memory snapshot; False until the worker has an id."""
        if self.worker_id is None:
            return False
        self.client.heartbeat(self.worker_id, {"memory": self._memory_snapshot()})
        return True

    # ---------------------------------------------------------------- command loop
    def _poll_once(self) -> list[dict]:
        try:
            return self.client.poll_commands(self.worker_id, wait_s=10.0)
        except httpx.HTTPStatusError as exc:
            if exc.response.status_code == 404:
                self._register_again()
            else:
                self.log.log("COORDINATOR_ERROR", error=str(exc)[:200])
                self._halt.wait(2)
        except httpx.HTTPError as exc:
            self.log.log("COORDINATOR_UNREACHABLE", error=str(exc)[:200])
            self._halt.wait(2)
        return []

    def run_forever(self) -> None:
        while self.worker_id is None and not self._halt.is_set():
            try:
                self.register()
            except httpx.HTTPError as exc:
                self.log.log("REGISTER_FAILED", error=str(exc)[:200], retry_in_s=3)
                self._halt.wait(3)
        while not self._halt.is_set():
            for command in self._poll_once():
                threading.Thread(target=self.handle, args=(command,), daemon=True,
                                 name=f"cmd-{command.get('type')}").start()

    def stop(self) -> None:
        self._halt.set()
        self.stages.stop()
        if self.heartbeat is not None:
            self.heartbeat.stop()
        self.dataplane.close()

    def _event(self, kind: str, data: dict) -> None:
        try:
            self.client.post_event(self.worker_id, {"type": kind, "data": data})
        except httpx.HTTPError as exc:
            self.log.log("EVENT_POST_FAILED", type=kind, error=str(exc)[:200])

    def handle(self, command: dict) -> None:
        kind = command.get("type")
        try:
            handler = self.handlers.get(kind)
            if handler is None:
                raise ValueError(f"unknown command {kind!r}")
            handler(command)
        except Exception as exc:  # noqa: BLE001 - reported to the coordinator
            message = f"{type(exc).__name__}: {exc}"
            self.log.log("COMMAND_FAILED", type=kind, error=message[:300])
            if command.get("request_id"):
                self._event("command_error", {"request_id": command["request_id"], "error": message})

    # ---------------------------------------------------------------- commands
    def _benchmark(self, command: dict) -> None:
        result = benchmark_device(self.device, quick=self.quick_benchmark)
        self.log.log("BENCHMARK_DONE", gflops=round(result["matmul_gflops"], 1))
        self._event("benchmark_result", {"request_id": command.get("request_id"), "result": result})

    def _probe(self, command: dict) -> None:
        result = measure_link(command["host"], int(command["port"]), token=self.token,
                              pings=int(command.get("pings", 10)), payload_mb=float(command.get("payload_mb", 16)))
        self.log.log("PROBE_DONE", target=command.get("target"), mbps=round(result["bandwidth_Mbps"], 1))
        self._event("probe_result", {"request_id": command.get("request_id"), "result": result})

    def _stop_job(self, command: dict) -> None:
        for (job, attempt), _thread in self.stages.stop(command["job_id"], command.get("attempt")):
            self.log.log("STOP_REQUESTED", job_id=job, attempt=attempt, reason=command.get("reason"))

    def _start_stage(self, command: dict) -> None:
        job_id, attempt = command["job_id"], int(command.get("attempt", 0))
        stage = int(command["stage_index"])
        for _key, thread in self.stages.stop(job_id, before=attempt):  # free the previous attempt's memory
            if thread is not threading.current_thread():
                thread.join(timeout=60)
        stop = self.stages.begin(job_id, attempt)
        tag = {"job_id": job_id, "attempt": attempt}
        steps_done = [0]

        def forward_metrics(record: dict) -> None:
            steps_done[0] += record.get("event") == "STEP_COMPLETE"
            self._event("stage_metrics", dict(tag, record=record))

        started = time.time()
        try:
            result = run_assignment(command, device=self.device, dataplane=self.dataplane,
                                    worker_name=self.worker_id, token=self.token, metrics_callback=forward_metrics,
                                    stop_event=stop, runs_dir=self.runs_dir)
        except Exception as exc:  # noqa: BLE001 - reported to the coordinator
            if stop.is_set():
                self.log.log("STAGE_STOPPED", job_id=job_id, attempt=attempt)
                return
            self._stage_failed(tag, stage, exc, steps_done[0])
        else:
            summary = {"steps": len(result.step_metrics), "wall_s": time.time() - started,
                       "final_loss": result.losses[-1] if result.losses else None}
            self._event("stage_done", dict(tag, stage=stage, summary=summary,
                                           timeline=(result.timeline or [])[-TIMELINE_SPANS_SENT:]))
        finally:
            self.stages.end(job_id, attempt)

    def _stage_failed(self, tag: dict, stage: int, exc: Exception, steps_done: int) -> None:
        message = f"{type(exc).__name__}: {exc}"
        self.log.log("STAGE_FAILED", job_id=tag["job_id"], error=message[:500])
        if not self.log.quiet:
            traceback.print_exc()
        oom = is_oom(exc)
        report = getattr(exc, "report", None)
        if report is None and oom:
            report = {"available": self.device.available_memory()}
        from meshtrain_b200.parallel.watchdog import PeerFailure

        # a stage stopped by another rank's failure says so: the coordinator waits for that
        # rank's own report (e.g. a startup OOM to re-plan) instead of failing the job on this one
        self._event("stage_error", dict(tag, stage=stage, error=message[:1000], oom=oom,
                                        steps_completed=steps_done, memory_report=report,
                                        peer_failure=isinstance(exc, PeerFailure)))
