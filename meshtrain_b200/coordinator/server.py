"""The coordinator: control plane only (no tensors, no training).

HTTP API (every route except ``/health`` needs header ``X-MeshTrain-Token``;
bodies are capped at 8 MiB), reference coordinator/server.py:1-505:

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

Startup OOM replanning: when a stage fails with out-of-memory before any step
completed, the failing worker's memory budget is shrunk to what it really
offered (``min(previous * shrink, (capacity * shrink + reserve) / safety)``)
and the job is planned again, up to ``memory.max_replans`` times; each attempt
gets its own data-plane job id ``<job>.a<n>`` so late packets of a dead attempt
cannot reach the new one.

Run artefacts under ``runs/<job>``: config.yaml, plan.txt, plan.json,
placement_attempts.json, metrics.jsonl, summary.json/.txt,
prediction_accuracy.json, timeline.json (Chrome trace) and timeline_report.txt.
"""

from __future__ import annotations

import hmac
import itertools
import json
import threading
import time
import uuid
from pathlib import Path

import yaml
from fastapi import Depends, FastAPI, Header, HTTPException, Request
from fastapi.responses import JSONResponse
from pydantic import BaseModel

from meshtrain_b200.config import ConfigError, parse_config
from meshtrain_b200.coordinator.registry import WorkerRegistry
from meshtrain_b200.coordinator.scheduler import plan_job
from meshtrain_b200.coordinator.state import JobRecord, JobStatus, WorkerRecord, WorkerStatus
from meshtrain_b200.planner.cost import NetworkModel
from meshtrain_b200.profiler.benchmark import normalise_scores
from meshtrain_b200.summary import format_summary, summarize
from meshtrain_b200.telemetry import EventLogger, MetricsWriter, read_jsonl

MAX_REQUEST_BYTES = 8 * 1024 * 1024
TOKEN_HEADER = "X-MeshTrain-Token"


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


class Coordinator:
    def __init__(self, token: str, runs_dir: str = "runs", heartbeat_timeout_s: float = 15.0,
                 command_timeout_s: float = 120.0, monitor: bool = True):
        self.token = token
        self.runs_dir = Path(runs_dir)
        self.registry = WorkerRegistry(heartbeat_timeout_s)
        self.registry.on_offline.append(self._worker_offline)
        self.jobs: dict[str, JobRecord] = {}
        self.command_timeout_s = command_timeout_s
        self.log = EventLogger("coordinator", "-")
        self._lock = threading.RLock()
        self._waiters: dict[str, tuple[threading.Event, dict]] = {}
        self.benchmark: dict = {"status": "NEVER_RUN", "workers": {}, "links": {}}
        self._writers: dict[str, MetricsWriter] = {}
        self._stop = threading.Event()
        if monitor:
            threading.Thread(target=self._monitor_loop, daemon=True, name="liveness").start()

    # ------------------------------------------------------------ liveness
    def _monitor_loop(self) -> None:
        while not self._stop.wait(0.5):
            self.registry.check_liveness()

    def _worker_offline(self, w: WorkerRecord) -> None:
        self.log.log("WORKER_OFFLINE", worker_id=w.worker_id, silent_s=round(time.time() - w.last_heartbeat, 1))
        with self._lock:
            for job in self.jobs.values():
                if job.status is JobStatus.RUNNING and w.worker_id in job.stage_workers:
                    self._fail_job(job, f"worker {w.worker_id} went offline (no heartbeat for "
                                        f"{self.registry.heartbeat_timeout_s:.0f}s)")

    def shutdown(self) -> None:
        self._stop.set()

    # ------------------------------------------------------------ request / response over the mailbox
    def _request(self, worker_id: str, command: dict, timeout: float) -> dict | None:
        rid = uuid.uuid4().hex[:12]
        done, box = threading.Event(), {}
        self._waiters[rid] = (done, box)
        self.registry.send(worker_id, {**command, "request_id": rid})
        ok = done.wait(timeout)
        self._waiters.pop(rid, None)
        return box if ok else None

    def _resolve(self, rid: str, data: dict) -> None:
        w = self._waiters.get(rid)
        if w is not None:
            w[1].update(data)
            w[0].set()

    # ------------------------------------------------------------ benchmark
    def start_benchmark(self, req: BenchmarkRequest) -> dict:
        with self._lock:
            if self.benchmark.get("status") == "RUNNING":
                return self.benchmark
            workers = self.registry.idle()
            self.benchmark = {"status": "RUNNING", "started_at": time.time(), "workers": {}, "links": {},
                              "errors": []}
        threading.Thread(target=self._run_benchmark, args=(workers, req), daemon=True, name="benchmark").start()
        return self.benchmark

    def _run_benchmark(self, workers: list[WorkerRecord], req: BenchmarkRequest) -> None:
        bench = self.benchmark
        results: dict[str, dict] = {}

        def one(w: WorkerRecord) -> None:
            r = self._request(w.worker_id, {"type": "RUN_BENCHMARK"}, self.command_timeout_s)
            if r is None or "error" in r:
                bench["errors"].append(f"{w.worker_id}: {r.get('error') if r else 'benchmark timed out'}")
            else:
                results[w.worker_id] = r["result"]

        threads = [threading.Thread(target=one, args=(w,)) for w in workers]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        for wid, score in normalise_scores(results).items():
            results[wid]["compute_score"] = score
            rec = self.registry.get(wid)
            if rec is not None:
                rec.benchmark = results[wid]
            bench["workers"][wid] = results[wid]
        if req.network:
            # one directional probe at a time, so links do not compete for the NICs
            for src, dst in itertools.permutations(workers, 2):
                r = self._request(src.worker_id, {"type": "PROBE_NETWORK", "target": dst.worker_id,
                                                  "host": dst.data_host, "port": dst.data_port, "pings": req.pings,
                                                  "payload_mb": req.payload_mb}, self.command_timeout_s)
                key = f"{src.worker_id}->{dst.worker_id}"
                if r is None or "error" in r:
                    bench["errors"].append(f"{key}: {r.get('error') if r else 'probe timed out'}")
                else:
                    bench["links"][key] = r["result"]
        bench["status"], bench["finished_at"] = "DONE", time.time()
        self.log.log("BENCHMARK_DONE", workers=len(results), links=len(bench["links"]))

    def network_model(self) -> NetworkModel:
        return NetworkModel.from_measurements(self.benchmark.get("links", {}))

    # ------------------------------------------------------------ jobs
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
        job_id = f"{cfg.job.name}-{time.strftime('%Y%m%d-%H%M%S')}-{uuid.uuid4().hex[:4]}"
        run_dir = self.runs_dir / job_id
        run_dir.mkdir(parents=True, exist_ok=True)
        dumped = cfg.model_dump(mode="json", by_alias=True)
        (run_dir / "config.yaml").write_text(yaml.safe_dump(dumped, sort_keys=False))
        job = JobRecord(job_id, dumped, plan.to_dict(), run_dir=str(run_dir))
        self._writers[job_id] = MetricsWriter(run_dir / "metrics.jsonl")
        with self._lock:
            self.jobs[job_id] = job
            job.status = JobStatus.RUNNING
            self._launch(job, cfg, plan)
        return job

    def _launch(self, job: JobRecord, cfg, plan) -> None:
        """Send START_STAGE to every stage of one placement attempt (lock held)."""
        run_dir = Path(job.run_dir)
        spec = cfg.build_model_spec()
        names = [spec.layer_name(i) for i in range(spec.num_layers)]
        (run_dir / "plan.txt").write_text(plan.format(names) + "\n")
        (run_dir / "plan.json").write_text(json.dumps(plan.to_dict(), indent=2))
        job.plan = plan.to_dict()
        job.stage_workers = [s.worker_id for s in plan.stages]
        job.stages_done = {}
        job.attempts.append({"attempt": job.attempt, "budget_overrides": dict(job.budget_overrides),
                             "placement": [{"worker": s.worker_id, "layers": [s.start, s.end],
                                            "estimated_required": s.memory.required, "usable": s.memory.usable}
                                           for s in plan.stages]})
        (run_dir / "placement_attempts.json").write_text(json.dumps(job.attempts, indent=2, default=str))
        data_job = job.job_id if job.attempt == 0 else f"{job.job_id}.a{job.attempt}"
        for s in plan.stages:
            w = self.registry.get(s.worker_id)
            w.status, w.current_job = WorkerStatus.BUSY, job.job_id
        n = len(plan.stages)
        nccl = cfg.network.tensor_transport == "nccl"
        first = self.registry.get(plan.stages[0].worker_id)
        rendezvous = {"host": first.data_host, "port": first.data_port + 1 + job.attempt} if nccl else None
        for i, s in enumerate(plan.stages):
            nxt = self.registry.get(plan.stages[i + 1].worker_id) if i + 1 < n else None
            self.registry.send(s.worker_id, {
                "type": "START_STAGE", "job_id": job.job_id, "attempt": job.attempt, "data_job_id": data_job,
                "config": job.config, "stage_index": i, "num_stages": n, "layers": [s.start, s.end],
                "memory_estimate": s.memory.to_dict(), "rendezvous": rendezvous,
                "downstream": ({"host": nxt.data_host, "port": nxt.data_port, "worker_id": nxt.worker_id}
                               if nxt else None),
                "upstream_worker": plan.stages[i - 1].worker_id if i else None,
            })
        self.log.log("JOB_STARTED", job_id=job.job_id, attempt=job.attempt,
                     placement=" | ".join(f"{s.worker_name}:{s.start}-{s.end - 1}" for s in plan.stages))

    def _replan(self, job: JobRecord, worker_id: str, data: dict) -> bool:
        """Startup OOM on ``worker_id``: shrink its budget to what it measured and plan again."""
        cfg = parse_config(job.config)
        if job.attempt >= cfg.memory.max_replans:
            return False
        w = self.registry.get(worker_id)
        backend = w.backend if w else "cuda"
        sf = cfg.memory.safety_factors().get(backend, cfg.memory.safety_factor)
        fw = cfg.memory.framework_reserve_bytes().get(backend, 0)
        st = next((s for s in job.plan.get("stages", []) if s["worker_id"] == worker_id), None)
        prev = job.budget_overrides.get(worker_id) or (st["memory"]["total"] if st else 0)
        shrink = cfg.memory.replan_shrink
        new_total = int(prev * shrink)
        report = data.get("memory_report") or {}
        if report.get("capacity"):
            new_total = min(new_total, int((report["capacity"] * shrink + fw) / sf))
        job.attempts[-1]["failure"] = {"worker": worker_id, "error": data.get("error"), "memory_report": report}
        job.budget_overrides[worker_id] = new_total
        for wid in job.stage_workers:
            self.registry.send(wid, {"type": "STOP_JOB", "job_id": job.job_id, "attempt": job.attempt,
                                     "reason": "replanning after startup OOM"})
        own = [self.registry.get(wid) for wid in job.stage_workers]
        self._release(job)
        try:
            cfg, plan = self.plan(job.config, job.budget_overrides,
                                  extra_workers=[x for x in own if x and x.status is not WorkerStatus.OFFLINE])
        except ValueError:
            return False
        if not plan.stages or not plan.feasible:
            job.attempts[-1]["replan_result"] = plan.format()
            (Path(job.run_dir) / "placement_attempts.json").write_text(json.dumps(job.attempts, indent=2,
                                                                                  default=str))
            return False
        job.attempt += 1
        self.log.log("JOB_REPLANNED", job_id=job.job_id, attempt=job.attempt, worker=worker_id,
                     new_budget_gb=round(new_total / 1024 ** 3, 3))
        self._launch(job, cfg, plan)
        return True

    def _release(self, job: JobRecord) -> None:
        for wid in job.stage_workers:
            w = self.registry.get(wid)
            if w is not None and w.current_job == job.job_id:
                w.current_job = None
                if w.status is WorkerStatus.BUSY:
                    w.status = WorkerStatus.ONLINE

    def _finish(self, job: JobRecord, status: JobStatus, error: str | None = None) -> None:
        # artefacts first: a client polling /jobs/{id} must never see COMPLETED without a summary
        try:
            job.summary = self._write_artifacts(job, status, error)
        except Exception as exc:  # noqa: BLE001 - artefacts are best effort
            self.log.log("ARTIFACT_WRITE_FAILED", job_id=job.job_id, error=f"{type(exc).__name__}: {exc}")
        job.error, job.finished_at = error, time.time()
        job.status = status
        self._release(job)

    def _write_artifacts(self, job: JobRecord, status: JobStatus, error: str | None) -> dict | None:
        run = Path(job.run_dir)
        records = read_jsonl(run / "metrics.jsonl")
        if not records:
            return None
        s = summarize(records)
        s["status"], s["error"] = status.value, error
        if job.plan and s.get("steps"):
            from meshtrain_b200.planner.report import prediction_accuracy

            acc = prediction_accuracy(job.plan, s)
            mem = {str(r["stage"]): r["memory_validation"] for r in records
                   if r.get("memory_validation") and r.get("attempt", 0) == job.attempt}
            if mem:
                acc["memory_validation"] = mem
            s["prediction_accuracy"] = acc
            (run / "prediction_accuracy.json").write_text(json.dumps(acc, indent=2, default=str))
        (run / "summary.json").write_text(json.dumps(s, indent=2, default=str))
        if job.timelines:
            from meshtrain_b200.utils.trace_report import ascii_timeline, format_breakdown, write_run_timeline

            lanes = [(idx, wk, spans) for idx, (wk, spans) in sorted(job.timelines.items())]
            write_run_timeline(run / "timeline.json", lanes)
            last = max((sp.get("step") or 0) for _, _, spans in lanes for sp in spans) if any(
                spans for _, _, spans in lanes) else 0
            (run / "timeline_report.txt").write_text(format_breakdown(s) + "\n\n" + ascii_timeline(lanes, last)
                                                     + "\n")
        (run / "summary.txt").write_text(format_summary(s) + "\n")
        return s

    def _fail_job(self, job: JobRecord, error: str) -> None:
        if job.status is not JobStatus.RUNNING:
            return
        self.log.log("JOB_FAILED", job_id=job.job_id, error=error)
        for wid in job.stage_workers:
            w = self.registry.get(wid)
            if w is not None and w.status is not WorkerStatus.OFFLINE:
                self.registry.send(wid, {"type": "STOP_JOB", "job_id": job.job_id, "reason": error})
        self._finish(job, JobStatus.FAILED, error)

    def stop_job(self, job_id: str) -> JobRecord:
        job = self.jobs[job_id]
        with self._lock:
            if job.status is JobStatus.RUNNING:
                for wid in job.stage_workers:
                    self.registry.send(wid, {"type": "STOP_JOB", "job_id": job_id, "reason": "stopped by user"})
                self._finish(job, JobStatus.STOPPED, "stopped by user")
        return job

    # ------------------------------------------------------------ worker events
    def handle_event(self, worker_id: str, ev: EventRequest) -> None:
        d = ev.data
        if ev.type in ("benchmark_result", "probe_result", "command_error"):
            self._resolve(d.get("request_id", ""), d)
            return
        job = self.jobs.get(d.get("job_id", ""))
        if job is None:
            return
        with self._lock:
            if int(d.get("attempt", job.attempt)) != job.attempt:
                return  # late event of a superseded attempt
            if ev.type == "stage_metrics":
                rec = dict(d["record"])
                rec["attempt"] = job.attempt
                self._writers[job.job_id].write(rec)
                if rec.get("event") == "MEMORY_VALIDATION":
                    job.memory_reports[str(rec["stage"])] = rec
                    return
                job.last_metrics[rec["stage"]] = rec
                if "loss" in rec:
                    job.losses.append((rec["step"], rec["loss"]))
            elif ev.type == "stage_done":
                job.stages_done[int(d["stage"])] = d.get("summary", {})
                if d.get("timeline"):
                    job.timelines[int(d["stage"])] = (worker_id, d["timeline"])
                if job.status is JobStatus.RUNNING and all(i in job.stages_done
                                                           for i in range(len(job.stage_workers))):
                    self.log.log("JOB_COMPLETED", job_id=job.job_id)
                    self._finish(job, JobStatus.COMPLETED)
            elif ev.type == "stage_error":
                if job.status is not JobStatus.RUNNING:
                    return
                startup_oom = bool(d.get("oom")) and not d.get("steps_completed") and not job.losses
                if startup_oom and self._replan(job, worker_id, d):
                    return
                hint = " (startup OOM; replanning exhausted or no placement fits)" if startup_oom else ""
                self._fail_job(job, f"stage {d.get('stage')} on {worker_id}: {d.get('error')}{hint}")


def create_app(coordinator: Coordinator) -> FastAPI:
    app = FastAPI(title="meshtrain_b200 coordinator", version="1")
    app.state.coordinator = c = coordinator

    @app.middleware("http")
    async def cap_request_size(request: Request, call_next):
        size = request.headers.get("content-length")
        if size is not None and size.isdigit() and int(size) > MAX_REQUEST_BYTES:
            return JSONResponse({"detail": "request too large"}, status_code=413)
        return await call_next(request)

    def auth(x_meshtrain_token: str | None = Header(default=None)):
        if x_meshtrain_token is None or not hmac.compare_digest(x_meshtrain_token.encode(), c.token.encode()):
            raise HTTPException(401, "invalid or missing cluster token")

    def known(worker_id: str) -> WorkerRecord:
        w = c.registry.get(worker_id)
        if w is None:
            raise HTTPException(404, f"unknown worker {worker_id}")
        return w

    guarded = [Depends(auth)]

    @app.get("/health")
    def health():
        return {"ok": True}

    @app.post("/workers/register", dependencies=guarded)
    def register(req: RegisterRequest):
        w = c.registry.register(name=req.name, hardware=req.hardware, backend=req.backend, device_info=req.device,
                                data_host=req.data_host, data_port=req.data_port, capabilities=req.capabilities)
        c.log.log("WORKER_REGISTERED", worker_id=w.worker_id, backend=w.backend, data=f"{w.data_host}:{w.data_port}")
        return {"worker_id": w.worker_id, "heartbeat_interval_s": max(1.0, c.registry.heartbeat_timeout_s / 4)}

    @app.post("/workers/{worker_id}/heartbeat", dependencies=guarded)
    def heartbeat(worker_id: str, req: HeartbeatRequest):
        if not c.registry.heartbeat(worker_id, req.memory):
            raise HTTPException(404, "unknown worker; register again")
        return {"ok": True}

    @app.get("/workers/{worker_id}/commands", dependencies=guarded)
    def commands(worker_id: str, wait: float = 20.0):
        known(worker_id)
        c.registry.heartbeat(worker_id)
        return {"commands": c.registry.poll(worker_id, min(max(wait, 0.0), 30.0))}

    @app.post("/workers/{worker_id}/events", dependencies=guarded)
    def events(worker_id: str, ev: EventRequest):
        known(worker_id)
        c.handle_event(worker_id, ev)
        return {"ok": True}

    @app.get("/cluster/status", dependencies=guarded)
    def status():
        return {"workers": [w.public() for w in c.registry.all()],
                "jobs": [{"job_id": j.job_id, "status": j.status.value} for j in c.jobs.values()]}

    @app.post("/cluster/benchmark", dependencies=guarded)
    def benchmark(req: BenchmarkRequest):
        return c.start_benchmark(req)

    @app.get("/cluster/benchmark", dependencies=guarded)
    def benchmark_status():
        return c.benchmark

    @app.post("/plan", dependencies=guarded)
    def plan(req: JobRequest):
        try:
            cfg, p = c.plan(req.config)
        except (ConfigError, ValueError) as exc:
            raise HTTPException(400, str(exc)) from exc
        spec = cfg.build_model_spec()
        return {"plan": p.to_dict(), "text": p.format([spec.layer_name(i) for i in range(spec.num_layers)])}

    @app.post("/jobs", dependencies=guarded)
    def start(req: JobRequest):
        try:
            job = c.start_job(req.config)
        except (ConfigError, ValueError) as exc:
            raise HTTPException(400, str(exc)) from exc
        text = (Path(job.run_dir) / "plan.txt").read_text()
        return {**job.public(), "plan_text": text, "num_layers": parse_config(req.config).model_num_layers()}

    @app.get("/jobs", dependencies=guarded)
    def jobs():
        return {"jobs": [j.public() for j in c.jobs.values()]}

    @app.get("/jobs/{job_id}", dependencies=guarded)
    def job(job_id: str):
        if job_id not in c.jobs:
            raise HTTPException(404, "unknown job")
        return c.jobs[job_id].public()

    @app.post("/jobs/{job_id}/stop", dependencies=guarded)
    def stop(job_id: str):
        if job_id not in c.jobs:
            raise HTTPException(404, "unknown job")
        return c.stop_job(job_id).public()

    return app


def run_coordinator(host: str = "0.0.0.0", port: int = 8080, *, token: str, runs_dir: str = "runs",
                    heartbeat_timeout_s: float = 15.0) -> None:
    import uvicorn

    coordinator = Coordinator(token, runs_dir, heartbeat_timeout_s)
    print(f"meshtrain_b200 coordinator on http://{host}:{port}  (runs -> {runs_dir})", flush=True)
    uvicorn.run(create_app(coordinator), host=host, port=port, log_level="warning")
