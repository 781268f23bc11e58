"""The coordinator: the cluster's control plane (no tensors, no training).

HTTP API, the reference's routes (coordinator/server.py:388-505); every route
except ``/health`` needs the ``X-MeshTrain-Token`` header and bodies are
capped at 8 MiB:

    POST /workers/register          hardware, device, data-plane address -> worker_id
    POST /workers/{id}/heartbeat    liveness + memory snapshot
    GET  /workers/{id}/commands     long poll (``wait`` seconds, at most 30)
    POST /workers/{id}/events       benchmark/probe results, stage metrics/done/error
    GET  /cluster/status            workers and jobs
    POST /cluster/benchmark         compute benchmark on every idle worker + directional link probes
    GET  /cluster/benchmark         benchmark progress and results
    POST /plan                      placement dry run for a config
    POST /jobs                      plan + start a job
    GET  /jobs, GET /jobs/{id}      job state (losses, per-stage metrics, attempts)
    POST /jobs/{id}/stop            stop a job

Structure: the ``Coordinator`` owns the worker registry (liveness and command
mailboxes), a ``Correlator`` that pairs commands sent to workers with the
events that answer them, at most one ``ClusterBenchmark`` run, and one
``JobSupervisor`` per job.  A supervisor places its job, starts the stages of
each placement attempt, records their metrics, and finishes the job
(COMPLETED / FAILED / STOPPED) with its run artefacts under ``runs/<job>``:
config.yaml, plan.txt, plan.json, placement_attempts.json, metrics.jsonl,
summary.json/.txt, prediction_accuracy.json, timeline.json (Chrome trace) and
timeline_report.txt.

Startup OOM replanning: a stage that runs out of memory before any step
completed shrinks its worker's budget to ``min(previous * shrink, (capacity *
shrink + reserve) / safety)`` and the job is placed again, at most
``memory.max_replans`` times; attempt n uses data-plane job id ``<job>.a<n>``
so late packets of a dead attempt cannot reach the new one.
"""

from __future__ import annotations

import hmac
import itertools
import json
import threading
import time
import uuid
from concurrent.futures import Future, ThreadPoolExecutor, TimeoutError as FutureTimeout
from pathlib import Path

import yaml
from fastapi import APIRouter, Depends, FastAPI, Header, HTTPException, Request
from fastapi.responses import JSONResponse
from pydantic import BaseModel

from meshtrain_b200.config import ConfigError, parse_config
from meshtrain_b200.coordinator.registry import WorkerRegistry
from meshtrain_b200.coordinator.scheduler import interleaved_layout, plan_job
from meshtrain_b200.coordinator.state import JobRecord, JobStatus, WorkerRecord, WorkerStatus
from meshtrain_b200.planner.cost import NetworkModel
from meshtrain_b200.profiler.benchmark import normalise_scores
from meshtrain_b200.summary import format_summary, summarize
from meshtrain_b200.telemetry import EventLogger, MetricsWriter, read_jsonl

MAX_REQUEST_BYTES = 8 * 1024 * 1024
TOKEN_HEADER = "X-MeshTrain-Token"
GB = 1024 ** 3


class RegisterRequest(BaseModel):
    name: str
    hardware: dict
    backend: str
    device: dict
    data_host: str
    data_port: int
    capabilities: dict = {}


class HeartbeatRequest(BaseModel):
    memory: dict = {}
    status: str | None = None


class EventRequest(BaseModel):
    type: str
    data: dict = {}


class JobRequest(BaseModel):
    config: dict


class BenchmarkRequest(BaseModel):
    pings: int = 10
    payload_mb: float = 16.0
    network: bool = True


class Correlator:
    """Commands that expect an answer: each gets a request id and a future the answering event resolves."""

    def __init__(self, registry: WorkerRegistry):
        self.registry = registry
        self._open: dict[str, Future] = {}
        self._lock = threading.Lock()

    def ask(self, worker_id: str, command: dict, timeout: float) -> dict | None:
        rid = uuid.uuid4().hex[:12]
        answer: Future = Future()
        with self._lock:
            self._open[rid] = answer
        try:
            self.registry.send(worker_id, dict(command, request_id=rid))
            return answer.result(timeout)
        except FutureTimeout:
            return None
        finally:
            with self._lock:
                self._open.pop(rid, None)

    def answer(self, request_id: str, data: dict) -> None:
        with self._lock:
            pending = self._open.get(request_id)
        if pending is not None and not pending.done():
            pending.set_result(dict(data))


class ClusterBenchmark:
    """One cluster benchmark: compute on every worker at once, then each directed link in turn."""

    def __init__(self, coordinator: "Coordinator", workers: list[WorkerRecord], req: BenchmarkRequest):
        self.c, self.workers, self.req = coordinator, workers, req
        self.state = {"status": "RUNNING", "started_at": time.time(), "workers": {}, "links": {}, "errors": []}

    def _ask(self, worker_id: str, command: dict, label: str):
        reply = self.c.correlator.ask(worker_id, command, self.c.command_timeout_s)
        if reply is None or "error" in reply:
            self.state["errors"].append(f"{label}: {reply.get('error') if reply else 'timed out'}")
            return None
        return reply["result"]

    def run(self) -> None:
        with ThreadPoolExecutor(max_workers=max(1, len(self.workers))) as pool:
            futures = {w.worker_id: pool.submit(self._ask, w.worker_id, {"type": "RUN_BENCHMARK"}, w.worker_id)
                       for w in self.workers}
        results = {wid: f.result() for wid, f in futures.items() if f.result() is not None}
        for wid, score in normalise_scores(results).items():
            results[wid]["compute_score"] = score
            record = self.c.registry.get(wid)
            if record is not None:
                record.benchmark = results[wid]
            self.state["workers"][wid] = results[wid]
        if self.req.network:  # serially, so the probes do not compete for the same NICs
            for src, dst in itertools.permutations(self.workers, 2):
                name = f"{src.worker_id}->{dst.worker_id}"
                probe = self._ask(src.worker_id, {"type": "PROBE_NETWORK", "target": dst.worker_id,
                                                  "host": dst.data_host, "port": dst.data_port,
                                                  "pings": self.req.pings, "payload_mb": self.req.payload_mb}, name)
                if probe is not None:
                    self.state["links"][name] = probe
        self.state.update(status="DONE", finished_at=time.time())
        self.c.log.log("BENCHMARK_DONE", workers=len(results), links=len(self.state["links"]))


def write_run_artifacts(job: JobRecord, status: JobStatus, error: str | None) -> dict | None:
    """summary.json/.txt, prediction_accuracy.json, timeline.json and timeline_report.txt of a finished job."""
    run = Path(job.run_dir)
    records = read_jsonl(run / "metrics.jsonl")
    if not records:
        return None
    summary = summarize(records)
    summary.update(status=status.value, error=error)
    if job.plan and summary.get("steps"):
        from meshtrain_b200.planner.report import prediction_accuracy

        accuracy = prediction_accuracy(job.plan, summary)
        validation = {str(r["stage"]): r["memory_validation"] for r in records
                      if r.get("memory_validation") and r.get("attempt", 0) == job.attempt}
        if validation:
            accuracy["memory_validation"] = validation
        summary["prediction_accuracy"] = accuracy
        (run / "prediction_accuracy.json").write_text(json.dumps(accuracy, indent=2, default=str))
    (run / "summary.json").write_text(json.dumps(summary, indent=2, default=str))
    if job.timelines:
        from meshtrain_b200.utils.trace_report import ascii_timeline, format_breakdown, write_run_timeline

        lanes = [(stage, worker, spans) for stage, (worker, spans) in sorted(job.timelines.items())]
        write_run_timeline(run / "timeline.json", lanes)
        steps = [span.get("step") or 0 for _s, _w, spans in lanes for span in spans]
        report = format_breakdown(summary) + "\n\n" + ascii_timeline(lanes, max(steps, default=0)) + "\n"
        (run / "timeline_report.txt").write_text(report)
    (run / "summary.txt").write_text(format_summary(summary) + "\n")
    return summary


class JobSupervisor:
    """Places one job, starts each placement attempt, tracks it and finishes it."""

    def __init__(self, coordinator: "Coordinator", job: JobRecord):
        self.c, self.job = coordinator, job
        self.metrics = MetricsWriter(Path(job.run_dir) / "metrics.jsonl")

    # -- attempts ---------------------------------------------------------------
    def launch(self, cfg, plan) -> None:
        """Writes the attempt's plan files and sends START_STAGE to each stage (coordinator lock held)."""
        job, registry = self.job, self.c.registry
        layout = interleaved_layout(cfg, plan)  # model chunks per rank for interleaved 1F1B, else None
        run = Path(job.run_dir)
        spec = cfg.build_model_spec()
        (run / "plan.txt").write_text(plan.format([spec.layer_name(i) for i in range(spec.num_layers)]) + "\n")
        (run / "plan.json").write_text(json.dumps(plan.to_dict(), indent=2))
        job.plan = plan.to_dict()
        job.stage_workers = [s.worker_id for s in plan.stages]
        job.stages_done = {}
        placement = [{"worker": s.worker_id, "layers": [s.start, s.end], "estimated_required": s.memory.required,
                      "usable": s.memory.usable} for s in plan.stages]
        for row, chunks in zip(placement, layout or []):
            row.update(chunk_ranges=chunks["chunk_ranges"], estimated_required=chunks["memory"].required,
                       usable=chunks["memory"].usable)
            row["layers"] = [chunks["chunk_ranges"][0][0], chunks["chunk_ranges"][-1][1]]
        job.attempts.append({"attempt": job.attempt, "budget_overrides": dict(job.budget_overrides),
                             "placement": placement, "state_offload": bool(getattr(plan, "state_offload", False))})
        self._write_attempts()
        workers = [registry.get(s.worker_id) for s in plan.stages]
        for w in workers:
            w.status, w.current_job = WorkerStatus.BUSY, job.job_id
        data_job = job.job_id if job.attempt == 0 else f"{job.job_id}.a{job.attempt}"
        rendezvous = None
        if cfg.network.tensor_transport == "nccl":  # NCCL store on the first stage's host, one port per attempt
            rendezvous = {"host": workers[0].data_host, "port": workers[0].data_port + 1 + job.attempt}
        n = len(plan.stages)
        for i, (stage, worker) in enumerate(zip(plan.stages, workers)):
            nxt = workers[i + 1] if i + 1 < n else None
            chunks = layout[i] if layout else None
            registry.send(worker.worker_id, {
                "type": "START_STAGE", "job_id": job.job_id, "attempt": job.attempt, "data_job_id": data_job,
                "config": job.config, "stage_index": i, "num_stages": n, "layers": placement[i]["layers"],
                "chunk_ranges": chunks and chunks["chunk_ranges"],
                "state_offload": bool(getattr(plan, "state_offload", False)),
                "memory_estimate": (chunks["memory"] if chunks else stage.memory).to_dict(), "rendezvous": rendezvous,
                "downstream": nxt and {"host": nxt.data_host, "port": nxt.data_port, "worker_id": nxt.worker_id},
                "upstream_worker": workers[i - 1].worker_id if i else None,
            })
        self.c.log.log("JOB_STARTED", job_id=job.job_id, attempt=job.attempt,
                       placement=" | ".join(f"{s.worker_name}:{s.start}-{s.end - 1}" for s in plan.stages))

    def _write_attempts(self) -> None:
        (Path(self.job.run_dir) / "placement_attempts.json").write_text(
            json.dumps(self.job.attempts, indent=2, default=str))

    def _stop_stages(self, reason: str, *, attempt: bool = False, skip_offline: bool = False) -> None:
        for wid in self.job.stage_workers:
            worker = self.c.registry.get(wid)
            if worker is None or (skip_offline and worker.status is WorkerStatus.OFFLINE):
                continue
            command = {"type": "STOP_JOB", "job_id": self.job.job_id, "reason": reason}
            if attempt:
                command["attempt"] = self.job.attempt
            self.c.registry.send(wid, command)

    def release_workers(self) -> None:
        for wid in self.job.stage_workers:
            worker = self.c.registry.get(wid)
            if worker is not None and worker.current_job == self.job.job_id:
                worker.current_job = None
                if worker.status is WorkerStatus.BUSY:
                    worker.status = WorkerStatus.ONLINE

    def shrunk_budget(self, cfg, worker_id: str, report: dict) -> int:
        """The budget a worker gets after a startup OOM (the documented replanning formula)."""
        job = self.job
        worker = self.c.registry.get(worker_id)
        backend = worker.backend if worker else "cuda"
        safety = cfg.memory.safety_factors().get(backend, cfg.memory.safety_factor)
        reserve = cfg.memory.framework_reserve_bytes().get(backend, 0)
        placed = next((s for s in job.plan.get("stages", []) if s["worker_id"] == worker_id), None)
        previous = job.budget_overrides.get(worker_id) or (placed["memory"]["total"] if placed else 0)
        shrink = cfg.memory.replan_shrink
        budget = int(previous * shrink)
        if report.get("capacity"):
            budget = min(budget, int((report["capacity"] * shrink + reserve) / safety))
        return budget

    def replan(self, worker_id: str, data: dict) -> bool:
        """After a startup OOM on ``worker_id``: shrink its budget, stop the attempt, place and launch again."""
        job = self.job
        cfg = parse_config(job.config)
        if job.attempt >= cfg.memory.max_replans:
            return False
        report = data.get("memory_report") or {}
        budget = self.shrunk_budget(cfg, worker_id, report)
        job.attempts[-1]["failure"] = {"worker": worker_id, "error": data.get("error"), "memory_report": report}
        job.budget_overrides[worker_id] = budget
        self._stop_stages("replanning after startup OOM", attempt=True)
        previous = [self.c.registry.get(wid) for wid in job.stage_workers]
        self.release_workers()
        try:
            cfg, plan = self.c.plan(job.config, job.budget_overrides,
                                    extra_workers=[w for w in previous if w and w.status is not WorkerStatus.OFFLINE])
        except ValueError:
            return False
        if not plan.stages or not plan.feasible:
            job.attempts[-1]["replan_result"] = plan.format()
            self._write_attempts()
            return False
        try:
            interleaved_layout(cfg, plan)  # the new stage count must still suit the interleaved program
        except ValueError as exc:
            job.attempts[-1]["replan_result"] = str(exc)
            self._write_attempts()
            return False
        job.attempt += 1
        self.c.log.log("JOB_REPLANNED", job_id=job.job_id, attempt=job.attempt, worker=worker_id,
                       new_budget_gb=round(budget / GB, 3))
        self.launch(cfg, plan)
        return True

    # -- endings ----------------------------------------------------------------
    def finish(self, status: JobStatus, error: str | None = None) -> None:
        job = self.job
        try:  # artefacts first: a poller must never see COMPLETED without its summary
            job.summary = write_run_artifacts(job, status, error)
        except Exception as exc:  # noqa: BLE001 - artefacts are best effort
            self.c.log.log("ARTIFACT_WRITE_FAILED", job_id=job.job_id, error=f"{type(exc).__name__}: {exc}")
        job.error, job.finished_at, job.status = error, time.time(), status
        self.release_workers()

    def fail(self, error: str) -> None:
        if self.job.status is not JobStatus.RUNNING:
            return
        self.c.log.log("JOB_FAILED", job_id=self.job.job_id, error=error)
        self._stop_stages(error, skip_offline=True)
        self.finish(JobStatus.FAILED, error)

    def stop(self) -> None:
        if self.job.status is JobStatus.RUNNING:
            self._stop_stages("stopped by user")
            self.finish(JobStatus.STOPPED, "stopped by user")

    # -- worker events ----------------------------------------------------------
    def on_metrics(self, record: dict) -> None:
        record = dict(record, attempt=self.job.attempt)
        self.metrics.write(record)
        if record.get("event") == "MEMORY_VALIDATION":
            self.job.memory_reports[str(record["stage"])] = record
            return
        self.job.last_metrics[record["stage"]] = record
        if "loss" in record:
            self.job.losses.append((record["step"], record["loss"]))

    def on_stage_done(self, worker_id: str, data: dict) -> None:
        job = self.job
        stage = int(data["stage"])
        job.stages_done[stage] = data.get("summary", {})
        if data.get("timeline"):
            job.timelines[stage] = (worker_id, data["timeline"])
        if job.status is JobStatus.RUNNING and len(job.stages_done) >= len(job.stage_workers) and all(
                i in job.stages_done for i in range(len(job.stage_workers))):
            self.c.log.log("JOB_COMPLETED", job_id=job.job_id)
            self.finish(JobStatus.COMPLETED)

    def on_stage_error(self, worker_id: str, data: dict) -> None:
        if self.job.status is not JobStatus.RUNNING:
            return
        if data.get("peer_failure"):
            self._await_root_cause(worker_id, data)
            return
        startup_oom = bool(data.get("oom")) and not data.get("steps_completed") and not self.job.losses
        if startup_oom and self.replan(worker_id, data):
            return
        hint = " (startup OOM; replanning exhausted or no placement fits)" if startup_oom else ""
        self.fail(f"stage {data.get('stage')} on {worker_id}: {data.get('error')}{hint}")

    def _await_root_cause(self, worker_id: str, data: dict) -> None:
        """A stage that stopped because another rank failed (device-engine jobs) is a consequence.

        The failed rank reports its own error (a startup OOM among them, which must reach
        the replanner) or its worker goes offline; either ends or re-plans the attempt.  If
        neither has happened within ``network.timeout_s``, this report fails the job.
        """
        job = self.job
        job.attempts[-1].setdefault("peer_failures", []).append(
            {"worker": worker_id, "stage": data.get("stage"), "error": data.get("error")})
        attempt = job.attempt
        grace = float(parse_config(job.config).network.timeout_s)

        def fallback():
            with self.c._lock:
                if job.status is JobStatus.RUNNING and job.attempt == attempt:
                    self.fail(f"stage {data.get('stage')} on {worker_id}: {data.get('error')}")

        timer = threading.Timer(grace, fallback)
        timer.daemon = True
        timer.start()

    EVENTS = {"stage_metrics": lambda self, wid, d: self.on_metrics(d["record"]),
              "stage_done": on_stage_done, "stage_error": on_stage_error}


class Coordinator:
    def __init__(self, token: str, runs_dir: str = "runs", heartbeat_timeout_s: float = 15.0,
                 command_timeout_s: float = 120.0, monitor: bool = True):
        self.token = token
        self.runs_dir = Path(runs_dir)
        self.command_timeout_s = command_timeout_s
        self.registry = WorkerRegistry(heartbeat_timeout_s)
        self.registry.on_offline.append(self._worker_offline)
        self.correlator = Correlator(self.registry)
        self.log = EventLogger("coordinator", "-")
        self.jobs: dict[str, JobRecord] = {}
        self.supervisors: dict[str, JobSupervisor] = {}
        self.benchmark: dict = {"status": "NEVER_RUN", "workers": {}, "links": {}}
        self._lock = threading.RLock()
        self._stop = threading.Event()
        if monitor:
            threading.Thread(target=self._watch_liveness, daemon=True, name="liveness").start()

    # -- liveness -------------------------------------------------------------------
    def _watch_liveness(self) -> None:
        while not self._stop.wait(0.5):
            self.registry.check_liveness()

    def _worker_offline(self, worker: WorkerRecord) -> None:
        self.log.log("WORKER_OFFLINE", worker_id=worker.worker_id,
                     silent_s=round(time.time() - worker.last_heartbeat, 1))
        reason = (f"worker {worker.worker_id} went offline (no heartbeat for "
                  f"{self.registry.heartbeat_timeout_s:.0f}s)")
        with self._lock:
            for sup in self.supervisors.values():
                if sup.job.status is JobStatus.RUNNING and worker.worker_id in sup.job.stage_workers:
                    sup.fail(reason)

    def shutdown(self) -> None:
        self._stop.set()

    # -- benchmark --------------------------------------------------------------------
    def start_benchmark(self, req: BenchmarkRequest) -> dict:
        with self._lock:
            if self.benchmark.get("status") == "RUNNING":
                return self.benchmark
            run = ClusterBenchmark(self, self.registry.idle(), req)
            self.benchmark = run.state
        threading.Thread(target=run.run, daemon=True, name="benchmark").start()
        return self.benchmark

    def network_model(self) -> NetworkModel:
        return NetworkModel.from_measurements(self.benchmark.get("links", {}))

    # -- jobs -----------------------------------------------------------------------
    def plan(self, config: dict, budget_overrides: dict | None = None, extra_workers: list | None = None):
        cfg = parse_config(config)
        workers = self.registry.idle()
        workers += [w for w in (extra_workers or []) if w not in workers]
        if not workers:
            raise ValueError("no idle online workers")
        return cfg, plan_job(cfg, workers, self.network_model(), budget_overrides=budget_overrides)

    def start_job(self, config: dict) -> JobRecord:
        cfg, plan = self.plan(config)
        if not plan.stages or (not plan.feasible and cfg.placement.enforce_memory_check):
            raise ValueError("placement infeasible:\n" + plan.format())
        layout = interleaved_layout(cfg, plan)  # refuses a microbatch count the interleaved program cannot run
        if layout and cfg.placement.enforce_memory_check:
            short = [f"stage {i}: needs {c['memory'].required / GB:.2f} GB of {c['memory'].usable / GB:.2f} GB"
                     for i, c in enumerate(layout) if not c["memory"].fits]
            if short:
                raise ValueError("interleaved placement infeasible: " + "; ".join(short))
        job_id = f"{cfg.job.name}-{time.strftime('%Y%m%d-%H%M%S')}-{uuid.uuid4().hex[:4]}"
        run_dir = self.runs_dir / job_id
        run_dir.mkdir(parents=True, exist_ok=True)
        config_out = cfg.model_dump(mode="json", by_alias=True)
        (run_dir / "config.yaml").write_text(yaml.safe_dump(config_out, sort_keys=False))  # with every default
        # workers get the config as submitted: a reference worker's strict schema rejects the keys this
        # package adds, and a config written for the reference contains none of them
        job = JobRecord(job_id, json.loads(json.dumps(config)), plan.to_dict(), run_dir=str(run_dir))
        with self._lock:
            self.jobs[job_id] = job
            sup = self.supervisors[job_id] = JobSupervisor(self, job)
            job.status = JobStatus.RUNNING
            sup.launch(cfg, plan)
        return job

    def stop_job(self, job_id: str) -> JobRecord:
        with self._lock:
            self.supervisors[job_id].stop()
        return self.jobs[job_id]

    # -- worker events -------------------------------------------------------------------
    def handle_event(self, worker_id: str, ev: EventRequest) -> None:
        data = ev.data
        if ev.type in ("benchmark_result", "probe_result", "command_error"):
            self.correlator.answer(data.get("request_id", ""), data)
            return
        sup = self.supervisors.get(data.get("job_id", ""))
        handler = JobSupervisor.EVENTS.get(ev.type)
        if sup is None or handler is None:
            return
        with self._lock:
            if int(data.get("attempt", sup.job.attempt)) != sup.job.attempt:
                return  # a late event of a superseded placement attempt
            handler(sup, worker_id, data)


def create_app(coordinator: Coordinator) -> FastAPI:
    app = FastAPI(title="meshtrain_b200 coordinator", version="1")
    app.state.coordinator = c = coordinator

    @app.middleware("http")
    async def cap_request_size(request: Request, call_next):
        size = request.headers.get("content-length")
        if size is not None and size.isdigit() and int(size) > MAX_REQUEST_BYTES:
            return JSONResponse({"detail": "request too large"}, status_code=413)
        return await call_next(request)

    def require_token(x_meshtrain_token: str | None = Header(default=None)):
        if x_meshtrain_token is None or not hmac.compare_digest(x_meshtrain_token.encode(), c.token.encode()):
            raise HTTPException(401, "invalid or missing cluster token")

    def worker(worker_id: str) -> WorkerRecord:
        record = c.registry.get(worker_id)
        if record is None:
            raise HTTPException(404, f"unknown worker {worker_id}")
        return record

    def job_of(job_id: str) -> JobRecord:
        if job_id not in c.jobs:
            raise HTTPException(404, "unknown job")
        return c.jobs[job_id]

    def bad_request(fn, *args):
        try:
            return fn(*args)
        except (ConfigError, ValueError) as exc:
            raise HTTPException(400, str(exc)) from exc

    api = APIRouter(dependencies=[Depends(require_token)])

    @api.post("/workers/register")
    def register(req: RegisterRequest):
        rec = c.registry.register(name=req.name, hardware=req.hardware, backend=req.backend, device_info=req.device,
                                  data_host=req.data_host, data_port=req.data_port, capabilities=req.capabilities)
        c.log.log("WORKER_REGISTERED", worker_id=rec.worker_id, backend=rec.backend,
                  data=f"{rec.data_host}:{rec.data_port}")
        return {"worker_id": rec.worker_id, "heartbeat_interval_s": max(1.0, c.registry.heartbeat_timeout_s / 4)}

    @api.post("/workers/{worker_id}/heartbeat")
    def heartbeat(worker_id: str, req: HeartbeatRequest):
        if not c.registry.heartbeat(worker_id, req.memory):
            raise HTTPException(404, "unknown worker; register again")
        return {"ok": True}

    @api.get("/workers/{worker_id}/commands")
    def commands(worker_id: str, wait: float = 20.0):
        worker(worker_id)
        c.registry.heartbeat(worker_id)  # a long poll is a sign of life too
        return {"commands": c.registry.poll(worker_id, min(max(wait, 0.0), 30.0))}

    @api.post("/workers/{worker_id}/events")
    def events(worker_id: str, ev: EventRequest):
        worker(worker_id)
        c.handle_event(worker_id, ev)
        return {"ok": True}

    @api.get("/cluster/status")
    def status():
        return {"workers": [w.public() for w in c.registry.all()],
                "jobs": [{"job_id": j.job_id, "status": j.status.value} for j in c.jobs.values()]}

    @api.post("/cluster/benchmark")
    def benchmark(req: BenchmarkRequest):
        return c.start_benchmark(req)

    @api.get("/cluster/benchmark")
    def benchmark_status():
        return c.benchmark

    @api.post("/plan")
    def plan(req: JobRequest):
        cfg, placement = bad_request(c.plan, req.config)
        spec = cfg.build_model_spec()
        return {"plan": placement.to_dict(),
                "text": placement.format([spec.layer_name(i) for i in range(spec.num_layers)])}

    @api.post("/jobs")
    def start(req: JobRequest):
        job = bad_request(c.start_job, req.config)
        return {**job.public(), "plan_text": (Path(job.run_dir) / "plan.txt").read_text(),
                "num_layers": parse_config(req.config).model_num_layers()}

    @api.get("/jobs")
    def jobs():
        return {"jobs": [j.public() for j in c.jobs.values()]}

    @api.get("/jobs/{job_id}")
    def job(job_id: str):
        return job_of(job_id).public()

    @api.post("/jobs/{job_id}/stop")
    def stop(job_id: str):
        job_of(job_id)
        return c.stop_job(job_id).public()

    @app.get("/health")
    def health():
        return {"ok": True}

    app.include_router(api)
    return app


def run_coordinator(host: str = "0.0.0.0", port: int = 8080, *, token: str, runs_dir: str = "runs",
                    heartbeat_timeout_s: float = 15.0) -> None:
    import uvicorn

    coordinator = Coordinator(token, runs_dir, heartbeat_timeout_s)
    print(f"meshtrain_b200 coordinator on http://{host}:{port}  (runs -> {runs_dir})", flush=True)
    uvicorn.run(create_app(coordinator), host=host, port=port, log_level="warning")
