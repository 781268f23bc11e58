"""``meshtrain`` command line (reference cli.py:1-645; same commands and flags).

Simple form:
    meshtrain start                   first machine: coordinator + worker, prints a join code
    meshtrain join TOKEN@HOST         every other machine
    meshtrain status | jobs | benchmark | plan CONFIG | train CONFIG | dashboard | console

Explicit form:
    meshtrain coordinator start [--port 8080]
    meshtrain worker join HOST:PORT [--device cuda:N|mps|cpu] [--name NAME]
    meshtrain cluster status | cluster benchmark [--output FILE]
    meshtrain inspect placement CONFIG
    meshtrain train CONFIG --local    every stage local: processes over pipes/TCP, or one
                                      GPU per stage over NCCL when network.tensor_transport is nccl
    meshtrain experiment correctness|placement|capacity|transformer|device-correctness
    meshtrain results record RUN_DIR --section NAME

Coordinator address and token: --coordinator/--token, then $MESHTRAIN_COORDINATOR /
$MESHTRAIN_TOKEN, then the cluster remembered in ~/.meshtrain/cluster.json.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import shutil
import sys
import time

from meshtrain_b200.terminal import banner, heading, paint, table

DEFAULT_TOKEN = "meshtrain-dev-token"
DEFAULT_PORT = 8080


# ---------------------------------------------------------------- remembered cluster
class ClusterMemory:
    """``<MESHTRAIN_HOME or ~/.meshtrain>/cluster.json``: the last cluster joined or started.

    It holds the cluster token, so it is created readable by its owner only.
    """

    FILE = "cluster.json"

    @classmethod
    def path(cls) -> str:
        home = os.environ.get("MESHTRAIN_HOME") or os.path.join(os.path.expanduser("~"), ".meshtrain")
        return os.path.join(home, cls.FILE)

    @classmethod
    def read(cls) -> dict:
        try:
            with open(cls.path()) as f:
                data = json.load(f)
        except (OSError, ValueError):
            return {}
        return data if isinstance(data, dict) else {}

    @classmethod
    def write(cls, coordinator: str, token: str) -> None:
        target = cls.path()
        os.makedirs(os.path.dirname(target), exist_ok=True)
        fd = os.open(target, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
        with os.fdopen(fd, "w") as f:
            json.dump({"coordinator": coordinator, "token": token}, f)


state_path, load_saved, save_cluster = ClusterMemory.path, ClusterMemory.read, ClusterMemory.write

_JOIN_TARGET = re.compile(r"^(?:(?P<token>[^@]*)@)?(?:https?://)?(?P<host>[^/:]*)(?::(?P<port>\d+))?/?$")


def parse_join_target(target: str) -> tuple[str, str | None]:
    """``TOKEN@HOST[:PORT]`` or ``HOST[:PORT]`` (optionally with http://) -> ("HOST:PORT", token or None)."""
    token = None
    if "@" in target:  # the token may itself contain '@': split at the last one
        token, target = target.rsplit("@", 1)
    m = _JOIN_TARGET.match(target)
    if m is None or not m.group("host"):
        raise ValueError("missing coordinator address")
    return f"{m.group('host')}:{m.group('port') or DEFAULT_PORT}", token or None


def lan_ip() -> str:
    """This machine's address on its default route (a UDP connect sends no packet)."""
    import socket

    try:
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as probe:
            probe.connect(("10.255.255.255", 1))
            return probe.getsockname()[0]
    except OSError:
        return "127.0.0.1"


def _first_set(*candidates):
    return next((c for c in candidates if c), None)


def resolve_token(args=None) -> str:
    """--token, then $MESHTRAIN_TOKEN, then the remembered cluster, then the insecure default (with a warning)."""
    token = _first_set(getattr(args, "token", None), os.environ.get("MESHTRAIN_TOKEN"), load_saved().get("token"))
    if token is None:
        print(f"warning: no --token / $MESHTRAIN_TOKEN, using the insecure default {DEFAULT_TOKEN!r}",
              file=sys.stderr)
        token = DEFAULT_TOKEN
    return token


def client_from(args=None):
    """A control-plane client for --coordinator / $MESHTRAIN_COORDINATOR / the remembered cluster / localhost."""
    from meshtrain_b200.networking.control import ControlClient

    address = _first_set(getattr(args, "coordinator", None), os.environ.get("MESHTRAIN_COORDINATOR"),
                         load_saved().get("coordinator")) or f"127.0.0.1:{DEFAULT_PORT}"
    return ControlClient(address, resolve_token(args))


def _gb(n) -> str:
    return f"{n / 1024 ** 3:.1f} GB" if n else "-"


def _load_raw(path: str) -> dict:
    from meshtrain_b200.config import load_config

    return load_config(path).model_dump(mode="json", by_alias=True)


# ---------------------------------------------------------------- coordinator / worker
def cmd_coordinator_start(args) -> int:
    from meshtrain_b200.coordinator.server import run_coordinator

    run_coordinator(args.host, args.port, token=resolve_token(args), runs_dir=args.runs_dir,
                    heartbeat_timeout_s=args.heartbeat_timeout)
    return 0


def _serve_as_worker(args, coordinator: str, token: str) -> int:
    """Runs this process as a worker of ``coordinator`` until Ctrl-C."""
    from meshtrain_b200.worker.agent import WorkerAgent

    options = {key: getattr(args, key) for key in ("device", "name", "data_port", "advertise_host", "runs_dir",
                                                     "quick_benchmark") if hasattr(args, key)}
    agent = WorkerAgent(coordinator, token, **options)
    try:
        agent.run_forever()
    except KeyboardInterrupt:
        pass
    finally:
        agent.stop()
    return 0


def cmd_worker_join(args) -> int:
    address, code_token = parse_join_target(args.coordinator_address)
    token = code_token or resolve_token(args)
    save_cluster(address, token)
    return _serve_as_worker(args, address, token)


JOIN_CODE_ALPHABET = "abcdefghjkmnpqrstuvwxyz23456789"  # no characters that are easy to misread


def _wait_until_serving(client, process, attempts: int = 150) -> bool:
    import httpx

    for _ in range(attempts):
        if process.poll() is not None:
            return False
        try:
            client.status()
            return True
        except httpx.HTTPError:
            time.sleep(0.1)
    return False


def cmd_start(args) -> int:
    """This machine becomes the cluster: a coordinator subprocess, a join code, and (unless --no-worker) a worker."""
    import secrets
    import subprocess

    from meshtrain_b200.networking.control import ControlClient

    print(banner() + "\n", flush=True)
    token = _first_set(args.token, os.environ.get("MESHTRAIN_TOKEN")) or \
        "".join(secrets.choice(JOIN_CODE_ALPHABET) for _ in range(10))
    argv = [sys.executable, "-m", "meshtrain_b200.cli", "coordinator", "start", "--host", args.host, "--port",
            str(args.port), "--runs-dir", args.runs_dir]
    coordinator = subprocess.Popen(argv, env=dict(os.environ, MESHTRAIN_TOKEN=token))
    address = f"127.0.0.1:{args.port}"
    client = ControlClient(address, token)
    try:
        if not _wait_until_serving(client, coordinator):
            print(f"error: coordinator exited (is port {args.port} in use?)", file=sys.stderr)
            return 1
        save_cluster(address, token)
        args.advertise_host = args.advertise_host or lan_ip()  # remote stages dial this machine's LAN address
        suffix = "" if args.port == DEFAULT_PORT else f":{args.port}"
        print("\n".join(["", heading("cluster started"), "", "  " + paint("on every other machine run:", "accent"),
                         "", f"      meshtrain join {token}@{args.advertise_host}{suffix}", "",
                         "  then, anywhere in the cluster:", "      meshtrain status", "      meshtrain dashboard",
                         "      meshtrain train configs/local_cpu_mlp.yaml", ""]), flush=True)
        if args.no_worker:
            return coordinator.wait() or 0
        return _serve_as_worker(args, address, token)
    except KeyboardInterrupt:
        return 0
    finally:
        client.close()
        coordinator.terminate()
        try:
            coordinator.wait(10)
        except subprocess.TimeoutExpired:
            coordinator.kill()


def cmd_local_cluster(args) -> int:
    """A coordinator plus N CPU worker processes on this machine (for trying the control plane)."""
    import subprocess

    token = resolve_token(args) if (args.token or os.environ.get("MESHTRAIN_TOKEN")) else "local-cluster"
    env = {**os.environ, "MESHTRAIN_TOKEN": token}
    procs = [subprocess.Popen([sys.executable, "-m", "meshtrain_b200.cli", "coordinator", "start", "--host",
                               "127.0.0.1", "--port", str(args.port), "--runs-dir", args.runs_dir], env=env)]
    address = f"127.0.0.1:{args.port}"
    save_cluster(address, token)
    try:
        time.sleep(1.0)
        for i in range(args.workers):
            procs.append(subprocess.Popen([sys.executable, "-m", "meshtrain_b200.cli", "worker", "join", address,
                                           "--device", args.device, "--name", f"local{i}", "--data-port", "0",
                                           "--advertise-host", "127.0.0.1", "--runs-dir", args.runs_dir], env=env))
        print(f"local cluster at {address} with {args.workers} worker(s); Ctrl-C stops it", flush=True)
        procs[0].wait()
    except KeyboardInterrupt:
        pass
    finally:
        for p in procs[::-1]:
            p.terminate()
        for p in procs:
            try:
                p.wait(10)
            except subprocess.TimeoutExpired:
                p.kill()
    return 0


# ---------------------------------------------------------------- cluster views
def _worker_cells(w: dict) -> dict:
    device = w.get("device") or {}
    memory = "-" if w["backend"] == "cpu" else _gb(device.get("memory_total")) + ("*" if device.get("unified_memory") else "")
    score = (w.get("benchmark") or {}).get("compute_score")
    return {"WORKER": w["worker_id"], "BACKEND": w["backend"].upper(), "DEVICE": device.get("name", ""),
            "MEMORY": memory, "RAM": _gb(w.get("ram_total")), "SCORE": "-" if score is None else f"{score:.2f}",
            "STATUS": w["status"]}


# (columns, widths) for wide and narrow terminals
STATUS_LAYOUTS = ((("WORKER", "BACKEND", "DEVICE", "MEMORY", "RAM", "SCORE", "STATUS"), (18, 7, 25, 11, 9, 6, 9)),
                  (("WORKER", "BACKEND", "DEVICE", "STATUS"), (18, 7, 24, 9)))


def format_status(status: dict) -> str:
    workers = status["workers"]
    alive = [w for w in workers if w["status"] in ("ONLINE", "BUSY")]
    columns, widths = STATUS_LAYOUTS[0 if shutil.get_terminal_size((110, 24)).columns >= 100 else 1]
    cells = [_worker_cells(w) for w in workers]
    out = [heading("cluster", f"{len(alive)}/{len(workers)} workers online"), "",
           table(list(columns), [[c[col] for col in columns] for c in cells], list(widths))]
    if not workers:
        out.append(paint("no workers yet: run `meshtrain join CODE` on another machine", "dim"))
    out += [f"  {w['worker_id']} -> {paint(w['current_job'], 'warn')}" for w in workers if w.get("current_job")]
    if status.get("jobs"):
        out += ["", heading("jobs")] + [f"  {j['job_id']}  {paint(j['status'], 'dim')}" for j in status["jobs"]]
    return "\n".join(out)


def cmd_status(args) -> int:
    c = client_from(args)
    try:
        print(format_status(c.status()))
        print(paint(f"coordinator: {c.base}", "dim"))
    finally:
        c.close()
    return 0


def _job_cells(job: dict) -> list:
    losses = dict(job.get("losses", []))
    per_stage = job.get("last_metrics", {})
    stage0 = per_stage[min(per_stage, key=int)] if per_stage else {}
    step_s = stage0.get("step_s", (job.get("summary") or {}).get("mean_step_s"))
    last_loss = f"{losses[max(losses)]:.5g}" if losses else "-"
    return [job["job_id"], job["status"], len(losses), last_loss, "-" if step_s is None else f"{step_s * 1000:.1f}"]


def format_jobs(jobs: list[dict]) -> str:
    newest_first = sorted(jobs, key=lambda j: j.get("created_at", 0), reverse=True)
    out = [heading("training runs", f"{len(jobs)} recorded"), "",
           table(["RUN", "STATUS", "STEPS", "LOSS", "STEP ms"], [_job_cells(j) for j in newest_first],
                 [34, 10, 6, 10, 10])]
    if not jobs:
        out.append(paint("no runs yet: meshtrain train CONFIG", "dim"))
    out += [paint(f"  {j['job_id']}: {j['error']}", "bad") for j in jobs if j.get("error")]
    return "\n".join(out)


def cmd_jobs(args) -> int:
    c = client_from(args)
    try:
        print(format_jobs(c.jobs()["jobs"]))
    finally:
        c.close()
    return 0


def cmd_console(args) -> int:
    from meshtrain_b200.terminal import run_console

    run_console(args)
    return 0


def cmd_dashboard(args) -> int:
    from meshtrain_b200.dashboard import run_dashboard

    run_dashboard(client_from(args), args.port)
    return 0


def format_benchmark(b: dict) -> str:
    from meshtrain_b200.profiler.network import format_matrix

    by_score = sorted(b.get("workers", {}).items(), key=lambda kv: -kv[1]["compute_score"])
    rows = [[wid, r["backend"].upper(), f"{r['matmul_gflops']:.1f}", f"{r['mlp_forward_s'] * 1e3:.2f}",
             f"{r['mlp_backward_s'] * 1e3:.2f}", f"{r['compute_score']:.2f}"] for wid, r in by_score]
    out = [heading("cluster benchmark", f"status: {b.get('status')}"), "",
           table(["WORKER", "BACKEND", "MATMUL GFLOP/s", "FWD ms", "BWD ms", "SCORE"], rows, [18, 7, 14, 10, 10, 6])]
    names = sorted(b.get("workers", {}))
    probes = {tuple(key.split("->")): probe for key, probe in b.get("links", {}).items()}
    if names and probes:
        matrices = (("bandwidth", "bandwidth_Mbps", lambda v: f"{v:.0f}Mbps"),
                    ("latency", "latency_s", lambda v: f"{v * 1000:.2f}ms"))
        for title, key, fmt in matrices:
            out += ["", heading(title, "row -> column"),
                    format_matrix(names, {pair: p[key] for pair, p in probes.items()},
                                  lambda v, fmt=fmt: "?" if v is None else fmt(v))]
    out += [paint(f"error: {e}", "bad") for e in b.get("errors", [])]
    return "\n".join(out)


def cmd_cluster_benchmark(args) -> int:
    client = client_from(args)
    try:
        client.start_benchmark({"pings": args.pings, "payload_mb": args.payload_mb, "network": not args.no_network})
        print(heading("benchmarking cluster", "compute + worker-to-worker links"), flush=True)
        result = client.benchmark_status()
        while result.get("status") == "RUNNING":
            time.sleep(1)
            result = client.benchmark_status()
    finally:
        client.close()
    print(format_benchmark(result))
    if args.output:
        with open(args.output, "w") as f:
            json.dump(result, f, indent=2)
    return 1 if result.get("errors") else 0


def cmd_benchmark(args) -> int:
    if args.what == "cluster":
        return cmd_cluster_benchmark(args)
    os.environ.setdefault("MESHTRAIN_QUIET", "1")
    from meshtrain_b200.experiments import pipeline_bench

    if args.cluster:
        if not args.config:
            print("error: --cluster needs --config", file=sys.stderr)
            return 2
        r = pipeline_bench.run_cluster_benchmark(client_from(args), _load_raw(args.config))
    else:
        model, batch, mbs = None, args.batch_size, args.microbatches
        if args.config:
            from meshtrain_b200.config import load_config

            cfg = load_config(args.config)
            model, batch, mbs = cfg.model_spec_dict(), cfg.training.batch_size, cfg.training.num_microbatches
        devices = args.devices.split(",") if args.devices else None
        r = pipeline_bench.run_local_benchmark(model, num_stages=len(devices) if devices else args.stages,
                                               batch_size=batch, num_microbatches=mbs, steps=args.steps,
                                               bandwidth_mbps=args.bandwidth_mbps or None,
                                               latency_ms=args.latency_ms, devices=devices,
                                               compression=None if args.compression == "none" else args.compression)
    print(r["markdown"])
    return 0


# ---------------------------------------------------------------- plan / train
def cmd_plan(args) -> int:
    c = client_from(args)
    try:
        resp = c.plan(_load_raw(args.config))
    finally:
        c.close()
    print(resp["text"])
    return 0 if resp["plan"]["feasible"] else 1


def cmd_inspect_placement(args) -> int:
    from meshtrain_b200.config import load_config
    from meshtrain_b200.planner.report import format_placement

    cfg = load_config(args.config)
    if args.offline:
        from meshtrain_b200.api import plan_device_pipeline

        spec = cfg.build_model_spec()
        tc = cfg.training
        from meshtrain_b200.parallel.placement import config_mode

        mode = config_mode(cfg.offload)
        args_plan = (spec, args.offline, tc.num_microbatches, tc.microbatch_size or tc.batch_size,
                     cfg.pipeline.schedule, tc.optimizer)
        try:
            plan = plan_device_pipeline(*args_plan, offload=mode == "host").to_dict()
        except RuntimeError:
            if mode != "auto":
                raise
            print("optimizer state: does not fit on the GPUs; offloaded to host memory (offload: auto)")
            plan = plan_device_pipeline(*args_plan, offload=True).to_dict()
    else:
        c = client_from(args)
        try:
            plan = c.plan(cfg.model_dump(mode="json", by_alias=True))["plan"]
        finally:
            c.close()
        spec = cfg.build_model_spec()
    print(format_placement(plan, [spec.layer_name(i) for i in range(spec.num_layers)]))
    if args.offline and args.offline > 1 and cfg.pipeline.schedule == "1f1b":
        from meshtrain_b200.api import forecast_interleaving, layer_costs

        rows = forecast_interleaving(layer_costs(spec), args.offline, cfg.training.num_microbatches)
        if rows:
            print("\nInterleaved 1F1B forecast (simulated from per-unit FLOPs; p2p and kernel-size effects "
                  "left out):")
            print("  chunks/GPU  bubble  step vs 1 chunk  largest/mean rank work")
            for r in rows:
                print(f"  {r['chunks']:>10}  {100 * r['bubble_fraction']:5.1f}%  {r['relative_step']:15.3f}  "
                      f"{r['rank_imbalance']:22.3f}")
    return 0 if plan["feasible"] else 1


def cmd_train(args) -> int:
    if args.local:
        from meshtrain_b200.config import load_config

        cfg = load_config(args.config)
        if cfg.network.tensor_transport == "nccl":
            return _train_local_device(args, cfg)
        return _train_local_host(args, cfg)
    c = client_from(args)
    raw = _load_raw(args.config)
    print(heading("planning", args.config), flush=True)
    job = c.start_job(raw)
    print(job["plan_text"])
    print(f"training started: job {job['job_id']}  (metrics -> {job['run_dir']}/metrics.jsonl)\n", flush=True)
    seen = 0
    log_every, steps = raw["training"]["log_every"], raw["training"]["steps"]
    try:
        while True:
            j = c.job(job["job_id"])
            last = j["last_metrics"]
            for step, loss in j["losses"][seen:]:
                if step % log_every == 0 or step == steps - 1:
                    comm = sum(m.get("comm_s", 0) for m in last.values())
                    sent = sum(m.get("bytes_sent", 0) for m in last.values())
                    step_s = max((m.get("step_s", 0) for m in last.values()), default=0)
                    print(f"step {step:<6} loss {loss:.4f}   step {step_s * 1000:.0f} ms   comm {comm * 1000:.0f} ms"
                          f"   sent {sent / 1e6:.2f} MB", flush=True)
            seen = len(j["losses"])
            if j["status"] != "RUNNING":
                break
            time.sleep(0.5)
    except KeyboardInterrupt:
        print("stopping job ...")
        c.stop_job(job["job_id"])
        return 130
    finally:
        c.close()
    print("\n" + heading("training " + j["status"]) + (paint(f": {j['error']}", "bad") if j.get("error") else ""))
    if j.get("summary"):
        from meshtrain_b200.summary import format_summary

        print(format_summary(j["summary"]))
    return 0 if j["status"] == "COMPLETED" else 1


def _local_host_stages(args, cfg) -> list:
    from meshtrain_b200.parallel.local import LocalStage

    if cfg.placement.stages:
        return [LocalStage(tuple(st.layers), st.device or "cpu") for st in cfg.placement.stages]
    count = args.stages or cfg.placement.num_stages or 2
    total = cfg.model_num_layers()
    edges = [total * i // count for i in range(count + 1)]
    return [LocalStage((a, b), args.device) for a, b in zip(edges, edges[1:])]


def _train_local_host(args, cfg) -> int:
    """Every stage as a process on this machine (host runtime over pipes or loopback TCP)."""
    from meshtrain_b200.parallel.local import run_local_pipeline
    from meshtrain_b200.summary import format_summary, summarize
    from meshtrain_b200.telemetry import MetricsWriter, new_run_id
    from meshtrain_b200.utils.trace_report import ascii_timeline, format_breakdown, write_run_timeline

    stages = _local_host_stages(args, cfg)
    run_id = new_run_id(cfg.job.name)
    run_dir = os.path.join(cfg.job.runs_dir, run_id)
    layout = " | ".join(f"stage{i} {st.device} layers {st.layers[0]}-{st.layers[1] - 1}" for i, st in enumerate(stages))
    print(f"local run {run_id}: {layout}", flush=True)
    transport = "tcp" if cfg.network.tensor_transport == "tcp" else "pipe"
    results = run_local_pipeline(cfg.model_spec_dict(), stages, cfg.pipeline_settings(run_id), seed=cfg.job.seed,
                                 optimizer=cfg.training.optimizer, lr=cfg.training.learning_rate, transport=transport,
                                 capture_params=True, torch_threads=args.threads)
    records = [rec for r in results for rec in r.step_metrics]
    metrics = MetricsWriter(os.path.join(run_dir, "metrics.jsonl"))
    for rec in records:
        metrics.write(rec)
    losses = results[0].losses
    every = cfg.training.log_every
    for step, loss in enumerate(losses):
        if step % every == 0 or step == len(losses) - 1:
            print(f"step {step:<6} loss {loss:.4f}")
    summary = summarize(records)
    moved = {r.stage_index: all(bool((r.initial_params[k] != r.final_params[k]).any()) for k in r.initial_params)
             for r in results}
    summary.update(parameters_changed=moved, loss_decreased=len(losses) > 1 and losses[-1] < losses[0])
    with open(os.path.join(run_dir, "summary.json"), "w") as f:
        json.dump(summary, f, indent=2, default=str)
    lanes = [(r.stage_index, r.worker, r.timeline or []) for r in results]
    trace = write_run_timeline(os.path.join(run_dir, "timeline.json"), lanes)
    print("\n\n".join(["", format_summary(summary), format_breakdown(summary),
                        ascii_timeline(lanes, step=len(losses) - 1)]))
    print(f"parameters changed per stage: {moved}\ntimeline: {trace} (chrome://tracing or ui.perfetto.dev)\n"
          f"metrics: {run_dir}/metrics.jsonl")
    ok = (summary["loss_decreased"] or len(losses) < 2) and all(moved.values())
    return 0 if ok else 1


def _device_rank(cfg_dict: dict, run_dir: str, partition):
    """One rank of ``train --local`` with the device engine (runs in a spawned process)."""
    from meshtrain_b200.api import PipelineTrainer
    from meshtrain_b200.config import parse_config

    cfg = parse_config(cfg_dict)
    tc = cfg.training
    from meshtrain_b200.parallel.placement import config_mode

    offload_options = dict(prefetch_ahead=cfg.offload.prefetch_ahead, chunk_mb=cfg.offload.chunk_mb,
                           device_budget_gb=cfg.offload.device_budget_gb)
    offload, mode = None, config_mode(cfg.offload)
    if mode == "host":
        from meshtrain_b200.parallel.offload import HostOffload

        offload = HostOffload(**offload_options)
    elif mode == "auto":
        offload = "auto"  # the trainer's startup memory estimate decides
    tr = PipelineTrainer(cfg.model_spec_dict(), num_microbatches=tc.num_microbatches, schedule=cfg.pipeline.schedule,
                         optimizer=tc.optimizer, lr=tc.learning_rate, weight_decay=tc.weight_decay, seed=cfg.job.seed,
                         partition=partition, max_inflight=cfg.pipeline.max_inflight_microbatches, offload=offload,
                         microbatch_size=tc.microbatch_size or tc.batch_size,
                         virtual_stages=cfg.pipeline.virtual_stages, recompute=tc.activation_recompute,
                         offload_options=offload_options)
    records = []
    seq = getattr(tr.spec, "seq_len", 1)
    offset = 0
    if tc.resume_from:
        from meshtrain_b200.checkpoint import load_stage_checkpoint

        offset = load_stage_checkpoint(tc.resume_from, tr.engine)
    ckpt_dir = tc.checkpoint_dir or os.path.join(run_dir, "checkpoints")
    measured = []  # timed steps since the start, for pipeline.rebalance_after_steps
    from meshtrain_b200.utils.timeline import Timeline

    timeline = Timeline(f"rank{tr.rank}", tr.stage)  # device spans (CUDA events) of every step
    walls: list[float] = []
    for step in range(offset, offset + tc.steps):
        after = cfg.pipeline.rebalance_after_steps
        if after and step - offset == after and tr.engine.offload is None:
            moves = tr.rebalance(measured[1:] or measured)  # the first step also warms up
            if moves and tr.rank == 0:
                print(f"rebalanced after {after} steps: units {[u for u, _a, _b in moves]} moved; "
                      f"stages now {tr.ranges}", flush=True)
        x, y = tr.spec.make_batch(step, tc.batch_size)
        t0 = time.perf_counter()
        wall0 = timeline.now()
        st = tr.step(step, x, y, timed=True)
        timeline.add_device_spans(st.spans, step, wall0)
        walls.append(wall0)
        if len(walls) > 256:  # keep the trace to the last 256 steps
            timeline.drop_before(walls[-256])
        measured.append(st)
        rec = {"event": "STEP_COMPLETE", "stage": tr.stage, "step": step, "engine": "device",
               "worker": f"rank{tr.rank}", "backend": tr.device.type, "step_s": time.perf_counter() - t0,
               "device_step_ms": st.step_ms, "compute_s": st.compute_ms / 1e3, "comm_s": st.wait_ms / 1e3,
               "bubble_fraction": st.bubble_fraction, "exposed_p2p_ms": st.exposed_p2p_ms,
               "bytes_sent": st.bytes_sent, "bytes_received": st.bytes_received}
        if tr.is_last:
            rec["loss"] = tr.loss_value(st)
            rec["tokens_per_s"] = tc.batch_size * seq / rec["step_s"]
            if step % tc.log_every == 0 or step == tc.steps - 1:
                print(f"step {step:<6} loss {rec['loss']:.4f}   {st.step_ms:.1f} ms (device)   "
                      f"bubble {100 * st.bubble_fraction:.1f}%   exposed p2p {st.exposed_p2p_ms:.2f} ms", flush=True)
        if tc.checkpoint_every and (step + 1) % tc.checkpoint_every == 0:
            from meshtrain_b200.checkpoint import save_stage_checkpoint

            save_stage_checkpoint(ckpt_dir, tr.engine, step + 1)
        records.append(rec)
    ranges = tr.ranges
    tr.close()
    return {"records": records, "ranges": ranges, "stage": tr.stage, "worker": f"rank{tr.rank}",
            "timeline": timeline.export()}


def _train_local_device(args, cfg) -> int:
    """One GPU per stage on this machine, activations over NCCL (gloo on a CPU-only host)."""
    import torch

    from meshtrain_b200.parallel.spawn import spawn_ranks
    from meshtrain_b200.summary import format_summary, summarize
    from meshtrain_b200.telemetry import MetricsWriter, new_run_id

    if cfg.placement.stages:
        partition = [list(s.layers) for s in cfg.placement.stages]
    else:
        partition = "topology_aware" if cfg.placement.strategy in ("topology_aware", "auto") else "balanced"
    k = len(partition) if isinstance(partition, list) else (args.stages or cfg.placement.num_stages or
                                                           max(1, torch.cuda.device_count()))
    run_id = new_run_id(cfg.job.name)
    run_dir = os.path.join(cfg.job.runs_dir, run_id)
    os.makedirs(run_dir, exist_ok=True)
    print(f"local device run {run_id}: {k} stage(s)", flush=True)
    out = spawn_ranks(_device_rank, k, cfg.model_dump(mode="json", by_alias=True), run_dir, partition,
                      timeout_s=cfg.network.timeout_s * 20)
    writer = MetricsWriter(os.path.join(run_dir, "metrics.jsonl"))
    for r in out:
        for rec in r["records"]:
            writer.write(rec)
    summary = summarize([rec for r in out for rec in r["records"]])
    summary["stage_layers"] = out[0]["ranges"]
    with open(os.path.join(run_dir, "summary.json"), "w") as f:
        json.dump(summary, f, indent=2, default=str)
    from meshtrain_b200.utils.trace_report import write_run_timeline

    trace = write_run_timeline(os.path.join(run_dir, "timeline.json"),
                               [(r["stage"], r["worker"], r["timeline"]) for r in out])
    print("\n" + format_summary(summary))
    print(f"metrics: {run_dir}/metrics.jsonl\ntimeline: {trace} (chrome://tracing or ui.perfetto.dev)")
    return 0


# ---------------------------------------------------------------- experiments / results
def _experiment_correctness(args):
    from meshtrain_b200.experiments.correctness import run_experiment1

    print(run_experiment1(args.transport))


def _experiment_placement(args):
    from meshtrain_b200.experiments.placement import run_experiment4

    print(run_experiment4(cluster_file=args.cluster))


def _experiment_capacity(args):
    from meshtrain_b200.experiments.capacity import run_experiment5

    client = client_from(args) if args.mode == "hardware" else None
    print(run_experiment5(mode=args.mode, cluster_file=args.cluster, steps=args.steps, client=client))


def _experiment_device_correctness(args):
    from meshtrain_b200.experiments.device_correctness import format_device_correctness, run_device_correctness

    result = run_device_correctness(args.devices.split(","), steps=args.steps)
    print(format_device_correctness(result))
    return 0 if result["passed"] else 1


def _experiment_transformer(args):
    from meshtrain_b200.experiments.transformer import run_experiment_transformer

    print(run_experiment_transformer())


EXPERIMENTS = {"correctness": _experiment_correctness, "placement": _experiment_placement,
               "capacity": _experiment_capacity, "device-correctness": _experiment_device_correctness,
               "transformer": _experiment_transformer}


def cmd_experiment(args) -> int:
    os.environ.setdefault("MESHTRAIN_QUIET", "1")
    return EXPERIMENTS[args.name](args) or 0


def cmd_results_record(args) -> int:
    from meshtrain_b200.experiments.record import record_run

    status = None
    try:
        status = client_from(args).status()
    except Exception:  # noqa: BLE001 - record without device names
        pass
    print(record_run(args.run_dir, args.section, reference_steps=args.reference_steps, cluster_status=status))
    return 0


# ---------------------------------------------------------------- parser
def _flag(*names, **kw):
    return names, kw


WORKER_FLAGS = (
    _flag("--device", default="auto", help="auto | cuda | cuda:N | mps | cpu"),
    _flag("--name", help="worker name (default: hostname[-gpuN])"),
    _flag("--data-port", type=int, default=29500, help="data-plane TCP port (0 = any)"),
    _flag("--advertise-host", help="address peers use to reach this machine"),
    _flag("--runs-dir", default="runs"),
    _flag("--quick-benchmark", action="store_true"),
)
CLUSTER_BENCH_FLAGS = (
    _flag("--pings", type=int, default=10),
    _flag("--payload-mb", type=float, default=16.0),
    _flag("--no-network", action="store_true"),
    _flag("--output", help="write the raw results as JSON"),
)
PIPELINE_BENCH_FLAGS = (
    _flag("what", nargs="?", default="cluster", choices=["cluster", "pipeline"]),
    _flag("--config", help="pipeline: model/training config"),
    _flag("--stages", type=int, default=3),
    _flag("--devices", help="pipeline: one device per stage, e.g. cpu,cpu,cpu"),
    _flag("--microbatches", type=int, default=8),
    _flag("--batch-size", type=int, default=32),
    _flag("--steps", type=int, default=8),
    _flag("--bandwidth-mbps", type=float, default=100.0, help="emulated link bandwidth (0 = unthrottled)"),
    _flag("--latency-ms", type=float, default=1.0),
    _flag("--compression", choices=["none", "bf16", "fp16"], default="none",
          help="pipeline: fp32 boundary tensors as 16-bit floats on the links (lossy)"),
    _flag("--cluster", action="store_true", help="pipeline: run the modes as cluster jobs"),
)

# (command path, handler, help, flags); every command also takes --token / --coordinator
COMMANDS = (
    (("coordinator", "start"), "cmd_coordinator_start", None,
     (_flag("--host", default="0.0.0.0"), _flag("--port", type=int, default=DEFAULT_PORT),
      _flag("--runs-dir", default="runs"), _flag("--heartbeat-timeout", type=float, default=15.0))),
    (("start",), "cmd_start", "start a cluster here: coordinator + local worker",
     (_flag("--host", default="0.0.0.0"), _flag("--port", type=int, default=DEFAULT_PORT),
      _flag("--no-worker", action="store_true", help="only the coordinator")) + WORKER_FLAGS),
    (("join",), "cmd_worker_join", "join a cluster: meshtrain join TOKEN@HOST[:PORT]",
     (_flag("coordinator_address", metavar="TOKEN@HOST[:PORT]"),) + WORKER_FLAGS),
    (("worker", "join"), "cmd_worker_join", None,
     (_flag("coordinator_address", metavar="[TOKEN@]HOST[:PORT]"),) + WORKER_FLAGS),
    (("local-cluster",), "cmd_local_cluster", "coordinator + N CPU workers on this machine",
     (_flag("--workers", type=int, default=3), _flag("--port", type=int, default=DEFAULT_PORT),
      _flag("--device", default="cpu"), _flag("--runs-dir", default="runs"))),
    (("status",), "cmd_status", "cluster workers", ()),
    (("cluster", "status"), "cmd_status", None, ()),
    (("jobs",), "cmd_jobs", "runs: status, loss, step time", ()),
    (("console",), "cmd_console", "interactive prompt", ()),
    (("dashboard",), "cmd_dashboard", "live metrics in a local browser", (_flag("--port", type=int, default=8081),)),
    (("cluster", "benchmark"), "cmd_cluster_benchmark", None, CLUSTER_BENCH_FLAGS),
    (("benchmark",), "cmd_benchmark", "measure the cluster or the pipeline modes",
     CLUSTER_BENCH_FLAGS + PIPELINE_BENCH_FLAGS),
    (("plan",), "cmd_plan", "preview a placement", (_flag("config"),)),
    (("inspect", "placement"), "cmd_inspect_placement", "detailed placement of a config",
     (_flag("config"), _flag("--offline", type=int, metavar="N_GPUS", default=0,
                             help="plan for N local B200s without a coordinator"))),
    (("train",), "cmd_train", "train from a YAML config",
     (_flag("config"), _flag("--local", action="store_true", help="run every stage on this machine"),
      _flag("--stages", type=int, help="--local: number of stages when the config names none"),
      _flag("--device", default="cpu", help="--local host runtime: device of auto-split stages"),
      _flag("--threads", type=int, default=None, help="--local host runtime: torch threads per stage"))),
    (("results", "record"), "cmd_results_record", "add a finished run to the results file",
     (_flag("run_dir"), _flag("--section", required=True), _flag("--reference-steps", type=int, default=20))),
    (("experiment",), "cmd_experiment", "correctness and placement experiments",
     (_flag("name", choices=["correctness", "placement", "capacity", "transformer", "device-correctness"]),
      _flag("--devices", default="cpu,cpu", help="device-correctness: one device per stage"),
      _flag("--transport", default="tcp", choices=["pipe", "tcp"]),
      _flag("--mode", default="emulated", choices=["emulated", "hardware", "b200"]),
      _flag("--cluster", help="JSON written by `cluster benchmark --output`"),
      _flag("--steps", type=int, default=5))),
)


def build_parser() -> argparse.ArgumentParser:
    """The command tree of ``COMMANDS``; --token / --coordinator work before or after the command."""
    shared = argparse.ArgumentParser(add_help=False)
    shared.add_argument("--token", default=argparse.SUPPRESS, help="cluster token (default $MESHTRAIN_TOKEN)")
    shared.add_argument("--coordinator", default=argparse.SUPPRESS, help="coordinator HOST:PORT")
    root = argparse.ArgumentParser(prog="meshtrain", description="pipeline-parallel training across machines and GPUs")
    root.add_argument("--token", default=None, help="cluster token (default $MESHTRAIN_TOKEN)")
    root.add_argument("--coordinator", default=None, help="coordinator HOST:PORT")
    groups = {(): root.add_subparsers(dest="command", required=True)}
    handlers = globals()
    for path, handler, help_text, flags in COMMANDS:
        for depth in range(1, len(path)):  # intermediate nouns ("coordinator", "cluster", ...)
            if path[:depth] not in groups:
                noun = groups[path[:depth - 1]].add_parser(path[depth - 1])
                groups[path[:depth]] = noun.add_subparsers(dest="action", required=True)
        extra = {"help": help_text} if help_text else {}
        cmd = groups[path[:-1]].add_parser(path[-1], parents=[shared], **extra)
        for names, kw in flags:
            cmd.add_argument(*names, **kw)
        defaults = {"func": handlers[handler]}
        if handler in ("cmd_cluster_benchmark",):
            defaults["what"] = "cluster"
        cmd.set_defaults(**defaults)
    return root


def main(argv: list[str] | None = None) -> int:
    parser = build_parser()
    args = parser.parse_args(argv)
    try:
        return int(args.func(args) or 0)
    except KeyboardInterrupt:
        return 130
    except Exception as exc:  # noqa: BLE001 - one-line error for the user, not a traceback
        import httpx

        from meshtrain_b200.config import ConfigError

        if isinstance(exc, (ConfigError, FileNotFoundError, ValueError, httpx.HTTPError)):
            detail = ""
            if isinstance(exc, httpx.HTTPStatusError):
                try:
                    detail = ": " + str(exc.response.json().get("detail"))
                except ValueError:
                    pass
            print(paint(f"error: {exc}{detail}", "bad"), file=sys.stderr)
            return 2
        raise


if __name__ == "__main__":
    sys.exit(main())
