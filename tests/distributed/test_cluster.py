"""End to end on one host: the real coordinator (HTTP, in a thread) and worker
processes started through the CLI, with the TCP data plane between them."""

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

TOKEN = "cluster-test-token"
ROOT = Path(__file__).resolve().parents[2]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def cluster(tmp_path):
    port = _free_port()
    coord = Coordinator(TOKEN, runs_dir=str(tmp_path / "runs"), heartbeat_timeout_s=3.0)
    server = uvicorn.Server(uvicorn.Config(create_app(coord), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    client = ControlClient(f"127.0.0.1:{port}", TOKEN)
    for _ in range(100):
        try:
            client.status()
            break
        except Exception:  # noqa: BLE001
            time.sleep(0.1)
    procs = []

    def start_worker(name, data_port=0):
        env = {**os.environ, "MESHTRAIN_TOKEN": TOKEN, "OMP_NUM_THREADS": "1", "MESHTRAIN_QUIET": "1",
               "MESHTRAIN_HOME": str(tmp_path / "home"),
               "PYTHONPATH": os.pathsep.join([str(ROOT), os.environ.get("PYTHONPATH", "")])}
        p = subprocess.Popen([sys.executable, "-m", "meshtrain_b200.cli", "worker", "join", f"127.0.0.1:{port}",
                              "--device", "cpu", "--name", name, "--data-port", str(data_port), "--advertise-host",
                              "127.0.0.1", "--quick-benchmark", "--runs-dir", str(tmp_path / "worker-runs")],
                             env=env, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
        procs.append(p)
        return p

    def wait_online(n, timeout=90):
        t0 = time.time()
        ws = []
        while time.time() - t0 < timeout:
            ws = [w for w in client.status()["workers"] if w["status"] == "ONLINE"]
            if len(ws) >= n:
                return ws
            time.sleep(0.2)
        raise TimeoutError(f"only {len(ws)} workers online")

    yield client, coord, start_worker, wait_online
    for p in procs:
        p.kill()
        p.wait()
    server.should_exit = True
    th.join(5)
    coord.shutdown()
    client.close()


def _wait_job(client, job_id, timeout=240):
    t0 = time.time()
    while time.time() - t0 < timeout:
        j = client.job(job_id)
        if j["status"] != "RUNNING":
            return j
        time.sleep(0.3)
    raise TimeoutError("job did not finish")


CFG = {"job": {"name": "e2e"}, "model": {"type": "mlp"},
       "training": {"batch_size": 64, "microbatch_size": 16, "learning_rate": 0.001, "optimizer": "adam",
                    "steps": 30, "log_every": 10},
       "placement": {"strategy": "auto", "num_stages": 3}, "workers": {"allow": ["cpu"]},
       "network": {"timeout_s": 20, "connect_timeout_s": 20}}


def test_three_workers_benchmark_plan_and_train(cluster):
    client, coord, start_worker, wait_online = cluster
    for n in ("alpha", "beta", "gamma"):
        start_worker(n)
    wait_online(3)
    client.start_benchmark({"pings": 3, "payload_mb": 2})
    t0 = time.time()
    while client.benchmark_status()["status"] == "RUNNING" and time.time() - t0 < 180:
        time.sleep(0.5)
    b = client.benchmark_status()
    assert b["status"] == "DONE" and not b["errors"], b.get("errors")
    assert len(b["workers"]) == 3 and len(b["links"]) == 6
    assert max(r["compute_score"] for r in b["workers"].values()) == pytest.approx(1.0)
    plan = client.plan(CFG)
    assert len(plan["plan"]["stages"]) == 3
    job = client.start_job(CFG)
    j = _wait_job(client, job["job_id"])
    assert j["status"] == "COMPLETED", j["error"]
    losses = [loss for _, loss in j["losses"]]
    assert len(losses) == 30 and losses[-1] < losses[0]
    s = j["summary"]
    assert set(map(int, s["stages"])) == {0, 1, 2}
    recs = read_jsonl(os.path.join(j["run_dir"], "metrics.jsonl"))
    assert {r["stage"] for r in recs if r.get("event") == "STEP_COMPLETE"} == {0, 1, 2}
    for f in ("summary.json", "prediction_accuracy.json", "timeline.json", "timeline_report.txt"):
        assert os.path.exists(os.path.join(j["run_dir"], f)), f
    assert all(w["status"] == "ONLINE" for w in client.status()["workers"])


def test_device_engine_job_over_gloo(cluster):
    """``tensor_transport: nccl`` jobs run the device engine; on CPU workers the ranks use gloo."""
    client, coord, start_worker, wait_online = cluster
    ports = [_free_port() for _ in range(2)]
    start_worker("d0", ports[0])
    start_worker("d1", ports[1])
    wait_online(2)
    cfg = {"job": {"name": "dev"}, "network": {"tensor_transport": "nccl", "timeout_s": 60},
           "model": {"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
           "training": {"batch_size": 8, "microbatch_size": 2, "steps": 6, "optimizer": "adam",
                        "learning_rate": 0.001, "log_every": 2},
           "placement": {"strategy": "equal", "num_stages": 2}, "workers": {"allow": ["cpu"]}}
    job = client.start_job(cfg)
    j = _wait_job(client, job["job_id"])
    assert j["status"] == "COMPLETED", j["error"]
    losses = [loss for _, loss in j["losses"]]
    assert len(losses) == 6 and all(l > 0 for l in losses)


def test_killed_worker_fails_the_job(cluster):
    client, coord, start_worker, wait_online = cluster
    procs = {n: start_worker(n) for n in ("k1", "k2")}
    wait_online(2)
    cfg = {**CFG, "training": {**CFG["training"], "steps": 100000}, "placement": {"strategy": "equal",
                                                                                   "num_stages": 2}}
    job = client.start_job(cfg)
    time.sleep(3)
    victim = job["plan"]["stages"][1]["worker_id"]
    procs[victim].kill()
    t0 = time.time()
    j = _wait_job(client, job["job_id"], timeout=60)
    assert j["status"] == "FAILED" and j["error"]
    assert time.time() - t0 < 45
