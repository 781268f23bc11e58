"""Whole-cluster runs on one host: the coordinator's HTTP app served in a thread,
workers as separate processes started through the CLI, the TCP data plane
between them.  Covers the benchmark -> plan -> train path, the device engine
over gloo, a worker dying mid-job, and startup-OOM replanning."""

import os
import socket
import subprocess
import sys
import threading
import time
from pathlib import Path

import pytest
import uvicorn

from meshtrain_b200.coordinator.server import Coordinator, create_app
from meshtrain_b200.networking.control import ControlClient
from meshtrain_b200.telemetry import read_jsonl

ROOT = Path(__file__).resolve().parents[2]
TOKEN = "local-cluster-secret"


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def eventually(predicate, timeout: float, every: float = 0.25, what: str = "condition"):
    give_up = time.monotonic() + timeout
    while time.monotonic() < give_up:
        value = predicate()
        if value:
            return value
        time.sleep(every)
    raise TimeoutError(f"{what} not reached within {timeout}s")


class LocalCluster:
    """A coordinator in this process plus CPU worker processes joined through the CLI."""

    def __init__(self, tmp: Path, heartbeat_timeout_s: float = 3.0):
        self.tmp = tmp
        self.port = free_port()
        self.coordinator = Coordinator(TOKEN, runs_dir=str(tmp / "runs"), heartbeat_timeout_s=heartbeat_timeout_s)
        config = uvicorn.Config(create_app(self.coordinator), host="127.0.0.1", port=self.port, log_level="error")
        self.server = uvicorn.Server(config)
        self.thread = threading.Thread(target=self.server.run, daemon=True)
        self.client = ControlClient(f"127.0.0.1:{self.port}", TOKEN)
        self.workers: dict[str, subprocess.Popen] = {}

    def __enter__(self):
        self.thread.start()

        def up():
            try:
                return self.client.status() is not None
            except Exception:  # noqa: BLE001 - not listening yet
                return False
        eventually(up, 20, 0.1, "coordinator up")
        return self

    def __exit__(self, *exc):
        for proc in self.workers.values():
            proc.kill()
            proc.wait()
        self.server.should_exit = True
        self.thread.join(5)
        self.coordinator.shutdown()
        self.client.close()

    def join(self, name: str, *, data_port: int = 0, env: dict | None = None) -> subprocess.Popen:
        environment = dict(os.environ, MESHTRAIN_TOKEN=TOKEN, OMP_NUM_THREADS="1", MESHTRAIN_QUIET="1",
                           MESHTRAIN_HOME=str(self.tmp / "home"),
                           PYTHONPATH=os.pathsep.join([str(ROOT), os.environ.get("PYTHONPATH", "")]), **(env or {}))
        argv = [sys.executable, "-m", "meshtrain_b200.cli", "worker", "join", f"127.0.0.1:{self.port}",
                "--device", "cpu", "--name", name, "--data-port", str(data_port), "--advertise-host", "127.0.0.1",
                "--quick-benchmark", "--runs-dir", str(self.tmp / "worker-runs")]
        self.workers[name] = subprocess.Popen(argv, env=environment, stdout=subprocess.DEVNULL,
                                              stderr=subprocess.PIPE)
        return self.workers[name]

    def online(self, count: int, timeout: float = 90) -> list[dict]:
        def ready():
            found = [w for w in self.client.status()["workers"] if w["status"] == "ONLINE"]
            return found if len(found) >= count else None
        return eventually(ready, timeout, 0.2, f"{count} workers online")

    def finished(self, job_id: str, timeout: float = 240) -> dict:
        return eventually(lambda: (lambda j: j if j["status"] != "RUNNING" else None)(self.client.job(job_id)),
                          timeout, 0.3, f"job {job_id} finished")


@pytest.fixture
def cluster(tmp_path):
    with LocalCluster(tmp_path) as c:
        yield c


MLP_JOB = {"job": {"name": "e2e"}, "model": {"type": "mlp"},
           "training": {"batch_size": 64, "microbatch_size": 16, "learning_rate": 0.001, "optimizer": "adam",
                        "steps": 30, "log_every": 10},
           "placement": {"strategy": "auto", "num_stages": 3}, "workers": {"allow": ["cpu"]},
           "network": {"timeout_s": 20, "connect_timeout_s": 20}}


def test_benchmark_plan_and_train_on_three_workers(cluster):
    for name in ("red", "green", "blue"):
        cluster.join(name)
    cluster.online(3)
    cluster.client.start_benchmark({"pings": 3, "payload_mb": 2})
    bench = eventually(lambda: (lambda b: b if b["status"] != "RUNNING" else None)(cluster.client.benchmark_status()),
                       180, 0.5, "benchmark done")
    assert bench["status"] == "DONE" and not bench["errors"], bench.get("errors")
    assert len(bench["workers"]) == 3 and len(bench["links"]) == 3 * 2  # every directed pair
    assert max(r["compute_score"] for r in bench["workers"].values()) == pytest.approx(1.0)
    assert len(cluster.client.plan(MLP_JOB)["plan"]["stages"]) == 3

    job = cluster.finished(cluster.client.start_job(MLP_JOB)["job_id"])
    assert job["status"] == "COMPLETED", job["error"]
    losses = [loss for _step, loss in job["losses"]]
    assert len(losses) == 30 and losses[-1] < losses[0]
    assert {int(s) for s in job["summary"]["stages"]} == {0, 1, 2}
    steps = [r for r in read_jsonl(os.path.join(job["run_dir"], "metrics.jsonl")) if r.get("event") == "STEP_COMPLETE"]
    assert {r["stage"] for r in steps} == {0, 1, 2}
    for artefact in ("config.yaml", "plan.txt", "plan.json", "placement_attempts.json", "summary.json",
                     "summary.txt", "prediction_accuracy.json", "timeline.json", "timeline_report.txt"):
        assert os.path.exists(os.path.join(job["run_dir"], artefact)), artefact
    assert {w["status"] for w in cluster.client.status()["workers"]} == {"ONLINE"}  # released after the job


def test_device_engine_job_over_gloo(cluster):
    """``tensor_transport: nccl`` jobs run the device engine; on CPU workers its ranks use gloo."""
    for name in ("dev0", "dev1"):
        cluster.join(name, data_port=free_port())
    cluster.online(2)
    config = {"job": {"name": "dev"}, "network": {"tensor_transport": "nccl", "timeout_s": 60},
              "model": {"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
              "training": {"batch_size": 8, "microbatch_size": 2, "steps": 6, "optimizer": "adam",
                           "learning_rate": 0.001, "log_every": 2},
              "placement": {"strategy": "equal", "num_stages": 2}, "workers": {"allow": ["cpu"]}}
    job = cluster.finished(cluster.client.start_job(config)["job_id"])
    assert job["status"] == "COMPLETED", job["error"]
    losses = [loss for _step, loss in job["losses"]]
    assert len(losses) == 6 and min(losses) > 0


def test_a_worker_that_dies_fails_the_job_and_frees_the_rest(cluster):
    for name in ("left", "right"):
        cluster.join(name)
    cluster.online(2)
    config = dict(MLP_JOB, training=dict(MLP_JOB["training"], steps=100_000),
                  placement={"strategy": "equal", "num_stages": 2})
    started = cluster.client.start_job(config)
    time.sleep(3)
    victim = started["plan"]["stages"][1]["worker_id"]
    cluster.workers[victim].kill()
    t0 = time.monotonic()
    job = cluster.finished(started["job_id"], timeout=60)
    assert job["status"] == "FAILED" and job["error"]
    assert time.monotonic() - t0 < 45
    survivor = next(w for w in cluster.client.status()["workers"] if w["worker_id"] != victim)
    eventually(lambda: cluster.client.status() and any(
        w["worker_id"] == survivor["worker_id"] and w["status"] == "ONLINE" for w in cluster.client.status()["workers"]),
        30, 0.3, "survivor back online")


def test_startup_oom_replans_with_fewer_layers_on_the_small_worker(cluster):
    cluster.join("roomy")
    cluster.join("tiny", env={"MESHTRAIN_EMULATE_DEVICE_MEMORY_GB": "0.12"})
    cluster.online(2)
    # ~29M parameters: half of them with Adam state exceeds the 0.12 GB the small worker reports
    config = {"job": {"name": "replan"},
              "model": {"type": "tiny_transformer", "layers": 6, "hidden_size": 512, "heads": 8, "vocab_size": 4096,
                        "seq_len": 32},
              "training": {"batch_size": 8, "microbatch_size": 4, "learning_rate": 0.001, "optimizer": "adam",
                           "steps": 3, "log_every": 1},
              "placement": {"strategy": "auto", "num_stages": 2, "enforce_memory_check": False},
              "memory": {"max_replans": 3, "probe_allocation": False},
              "workers": {"allow": ["cpu"]}, "network": {"timeout_s": 30, "connect_timeout_s": 30}}
    job = cluster.finished(cluster.client.start_job(config)["job_id"], timeout=300)
    if job["status"] != "COMPLETED":
        pytest.skip(f"host memory too small for this scenario: {job['error']}")
    assert job["attempt"] >= 1
    first, last = job["attempts"][0], job["attempts"][-1]
    assert "failure" in first and first["failure"]["worker"].startswith("tiny")

    def layers_on(attempt, prefix):
        return sum(b - a for p in attempt["placement"] if p["worker"].startswith(prefix) for a, b in [p["layers"]])
    assert layers_on(last, "tiny") < layers_on(first, "tiny")


def test_device_engine_startup_oom_replans(cluster):
    """A device-engine (``tensor_transport: nccl``) job whose stage does not fit the worker's
    memory: the stage's startup check fails before any rank sends or receives, every rank
    tears its process group down, and the coordinator places the job again with fewer
    layers on that worker; the same worker processes run the new attempt's process group."""
    cluster.join("roomy", data_port=free_port())
    cluster.join("tiny", data_port=free_port(), env={"MESHTRAIN_EMULATE_DEVICE_MEMORY_GB": "0.12"})
    cluster.online(2)
    # ~21M parameters; the engine keeps 16 bytes per fp32 parameter (weights, gradients, two
    # Adam moments), so half of the blocks exceed the 0.12 GB the small worker reports
    config = {"job": {"name": "dev-replan"},
              "model": {"type": "gpt", "layers": 6, "hidden_size": 512, "heads": 8, "vocab_size": 4096,
                        "seq_len": 32},
              "training": {"batch_size": 8, "microbatch_size": 4, "learning_rate": 0.001, "optimizer": "adam",
                           "steps": 3, "log_every": 1},
              "placement": {"strategy": "auto", "num_stages": 2, "enforce_memory_check": False},
              "memory": {"max_replans": 3, "probe_allocation": False},
              "workers": {"allow": ["cpu"]}, "network": {"tensor_transport": "nccl", "timeout_s": 60}}
    job = cluster.finished(cluster.client.start_job(config)["job_id"], timeout=300)
    assert job["status"] == "COMPLETED", job["error"]
    assert job["attempt"] >= 1
    first, last = job["attempts"][0], job["attempts"][-1]
    assert first["failure"]["worker"].startswith("tiny")
    assert first["failure"]["memory_report"]["engine"] == "device"

    def layers_on(attempt, prefix):
        return sum(b - a for p in attempt["placement"] if p["worker"].startswith(prefix) for a, b in [p["layers"]])
    assert layers_on(last, "tiny") < layers_on(first, "tiny")
    assert len(job["losses"]) == 3


def test_interleaved_device_engine_job(cluster):
    """``pipeline.virtual_stages: 2`` on a device-engine job: the coordinator cuts the model into
    four pieces for two workers (each holds two, linked in a ring) and the job trains exactly
    like the same job with one contiguous range per worker."""
    for name in ("ring0", "ring1"):
        cluster.join(name, data_port=free_port())
    cluster.online(2)
    base = {"network": {"tensor_transport": "nccl", "timeout_s": 60},
            "model": {"type": "gpt", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
            "training": {"batch_size": 8, "microbatch_size": 2, "steps": 4, "optimizer": "adam",
                         "learning_rate": 0.001, "log_every": 1},
            "placement": {"strategy": "equal", "num_stages": 2}, "workers": {"allow": ["cpu"]}}
    plain = cluster.finished(cluster.client.start_job({**base, "job": {"name": "plain"}})["job_id"])
    assert plain["status"] == "COMPLETED", plain["error"]
    ring = cluster.finished(cluster.client.start_job(
        {**base, "job": {"name": "ring"}, "pipeline": {"schedule": "1f1b", "virtual_stages": 2}})["job_id"])
    assert ring["status"] == "COMPLETED", ring["error"]
    chunks = [p["chunk_ranges"] for p in ring["attempts"][0]["placement"]]
    assert len(chunks) == 2 and all(len(c) == 2 for c in chunks)
    assert sorted(tuple(r) for c in chunks for r in c)[0][0] == 0
    assert [loss for _s, loss in ring["losses"]] == pytest.approx([loss for _s, loss in plain["losses"]], rel=1e-5)


def test_interleaved_job_needs_microbatches_divisible_by_stages(cluster):
    for name in ("odd0", "odd1"):
        cluster.join(name, data_port=free_port())
    cluster.online(2)
    config = {"job": {"name": "odd"}, "network": {"tensor_transport": "nccl"},
              "model": {"type": "gpt", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
              "training": {"batch_size": 6, "microbatch_size": 2, "steps": 1},
              "pipeline": {"virtual_stages": 2}, "placement": {"strategy": "equal", "num_stages": 2},
              "workers": {"allow": ["cpu"]}}
    import httpx

    with pytest.raises(httpx.HTTPStatusError) as refused:
        cluster.client.start_job(config)
    assert refused.value.response.status_code == 400
    assert "multiple of the number of stages" in refused.value.response.text


REFERENCE = ROOT / "baseline" / "_ref"


@pytest.mark.skipif(not (REFERENCE / "meshtrain").is_dir(), reason="the reference is not installed under baseline/_ref")
def test_reference_worker_joins_and_runs_a_stage(cluster):
    """A worker of the reference's own build joins this coordinator (same routes, token header and
    commands), takes the second stage of a job and talks MSHT to a worker of this package; the job
    trains like one process."""
    from meshtrain_b200.parallel.local import reference_step
    from meshtrain_b200.parallel.pipeline import PipelineSettings

    cluster.join("ours0", data_port=free_port())
    env = dict(os.environ, MESHTRAIN_TOKEN=TOKEN, OMP_NUM_THREADS="1", MESHTRAIN_QUIET="1", PYTHONPATH=str(REFERENCE))
    cluster.workers["refw"] = subprocess.Popen(
        [sys.executable, "-m", "meshtrain.cli", "join", f"{TOKEN}@127.0.0.1:{cluster.port}", "--device", "cpu",
         "--name", "refw", "--data-port", str(free_port()), "--advertise-host", "127.0.0.1", "--quick-benchmark",
         "--runs-dir", str(cluster.tmp / "ref-runs")],
        env=env, cwd=str(cluster.tmp), stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
    cluster.online(2)
    config = {"job": {"name": "mixed"}, "model": {"type": "mlp"},
              "training": {"batch_size": 32, "microbatch_size": 8, "learning_rate": 0.001, "optimizer": "adam",
                           "steps": 5, "log_every": 1},
              "placement": {"strategy": "manual", "stages": [{"worker": "ours0", "layers": [0, 3]},
                                                            {"worker": "refw", "layers": [3, 7]}]},
              "workers": {"allow": ["cpu"]}, "network": {"timeout_s": 30, "connect_timeout_s": 30}}
    job = cluster.finished(cluster.client.start_job(config)["job_id"], timeout=180)
    assert job["status"] == "COMPLETED", job["error"]
    assert job["stage_workers"] == ["ours0", "refw"]
    settings = PipelineSettings("oracle", steps=5, batch_size=32, num_microbatches=4)
    oracle, _, _ = reference_step({"type": "mlp"}, settings, optimizer="adam", lr=0.001, steps=5)
    assert [loss for _step, loss in job["losses"]] == pytest.approx(oracle, rel=1e-6)


@pytest.mark.skipif(not (REFERENCE / "meshtrain").is_dir(), reason="the reference is not installed under baseline/_ref")
def test_worker_joins_the_reference_coordinator(tmp_path):
    """The other way round: a worker of this package joins the reference's own coordinator and runs the
    last stage of its job next to a reference worker."""
    from meshtrain_b200.parallel.local import reference_step
    from meshtrain_b200.parallel.pipeline import PipelineSettings

    port = free_port()
    ref_env = dict(os.environ, MESHTRAIN_TOKEN=TOKEN, OMP_NUM_THREADS="1", MESHTRAIN_QUIET="1",
                   PYTHONPATH=str(REFERENCE))
    procs = [subprocess.Popen([sys.executable, "-m", "meshtrain.cli", "coordinator", "start", "--host", "127.0.0.1",
                               "--port", str(port), "--runs-dir", str(tmp_path / "runs"), "--heartbeat-timeout", "5"],
                              env=ref_env, cwd=str(tmp_path), stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)]
    client = ControlClient(f"127.0.0.1:{port}", TOKEN)
    try:
        def up():
            try:
                return client.status() is not None
            except Exception:  # noqa: BLE001 - not listening yet
                return False
        eventually(up, 60, 0.2, "reference coordinator up")
        ours_env = dict(os.environ, MESHTRAIN_TOKEN=TOKEN, OMP_NUM_THREADS="1", MESHTRAIN_QUIET="1",
                        MESHTRAIN_HOME=str(tmp_path / "home"),
                        PYTHONPATH=os.pathsep.join([str(ROOT), os.environ.get("PYTHONPATH", "")]))
        procs.append(subprocess.Popen(
            [sys.executable, "-m", "meshtrain_b200.cli", "worker", "join", f"127.0.0.1:{port}", "--device", "cpu",
             "--name", "ours0", "--data-port", str(free_port()), "--advertise-host", "127.0.0.1", "--quick-benchmark",
             "--runs-dir", str(tmp_path / "our-runs")], env=ours_env, cwd=str(tmp_path),
            stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL))
        procs.append(subprocess.Popen(
            [sys.executable, "-m", "meshtrain.cli", "join", f"{TOKEN}@127.0.0.1:{port}", "--device", "cpu",
             "--name", "refw", "--data-port", str(free_port()), "--advertise-host", "127.0.0.1", "--quick-benchmark",
             "--runs-dir", str(tmp_path / "ref-runs")], env=ref_env, cwd=str(tmp_path),
            stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL))
        eventually(lambda: len([w for w in client.status()["workers"] if w["status"] == "ONLINE"]) >= 2, 90, 0.5,
                   "two workers online")
        config = {"job": {"name": "mixed"}, "model": {"type": "mlp"},
                  "training": {"batch_size": 32, "microbatch_size": 8, "learning_rate": 0.001, "optimizer": "adam",
                               "steps": 5, "log_every": 1},
                  "placement": {"strategy": "manual", "stages": [{"worker": "refw", "layers": [0, 3]},
                                                                {"worker": "ours0", "layers": [3, 7]}]},
                  "workers": {"allow": ["cpu"]}, "network": {"timeout_s": 30, "connect_timeout_s": 30}}
        job_id = client.start_job(config)["job_id"]
        job = eventually(lambda: (lambda j: j if j["status"] != "RUNNING" else None)(client.job(job_id)), 180, 0.5,
                         "job finished")
        assert job["status"] == "COMPLETED", job.get("error")
        settings = PipelineSettings("oracle", steps=5, batch_size=32, num_microbatches=4)
        oracle, _, _ = reference_step({"type": "mlp"}, settings, optimizer="adam", lr=0.001, steps=5)
        assert [loss for _step, loss in job["losses"]] == pytest.approx(oracle, rel=1e-6)
    finally:
        client.close()
        for proc in procs:
            proc.kill()
            proc.wait()
