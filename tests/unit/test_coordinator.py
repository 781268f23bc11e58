import json
import time
from pathlib import Path

import pytest
from fastapi.testclient import TestClient

from meshtrain_b200.coordinator.registry import WorkerRegistry
from meshtrain_b200.coordinator.scheduler import live_cuda_budget, worker_profile
from meshtrain_b200.coordinator.server import Coordinator, create_app
from meshtrain_b200.coordinator.state import WorkerRecord, WorkerStatus

TOKEN = "t0k3n"
H = {"X-MeshTrain-Token": TOKEN}
GB = 1024 ** 3
CFG = {"job": {"name": "unit"}, "model": {"type": "mlp"},
       "training": {"batch_size": 32, "microbatch_size": 8, "steps": 3, "optimizer": "adam"},
       "placement": {"strategy": "equal", "num_stages": 2}, "workers": {"allow": ["cpu"]}}


@pytest.fixture
def env(tmp_path):
    coord = Coordinator(TOKEN, runs_dir=str(tmp_path / "runs"), heartbeat_timeout_s=60, monitor=False)
    client = TestClient(create_app(coord))
    yield coord, client
    coord.shutdown()


def _register(client, name, backend="cpu", port=1000, memory=8 * GB, host="h1"):
    r = client.post("/workers/register", headers=H, json={
        "name": name, "hardware": {"hostname": host, "ram_total": memory, "ram_available": memory},
        "backend": backend, "device": {"memory_total": memory}, "data_host": "127.0.0.1", "data_port": port})
    assert r.status_code == 200, r.text
    return r.json()["worker_id"]


def test_auth_health_and_size_cap(env):
    _, client = env
    assert client.get("/health").json() == {"ok": True}
    assert client.get("/cluster/status").status_code == 401
    assert client.get("/cluster/status", headers={"X-MeshTrain-Token": "nope"}).status_code == 401
    big = client.post("/plan", headers={**H, "content-length": str(9 * 1024 * 1024)}, content=b"{}")
    assert big.status_code == 413


def test_register_heartbeat_and_reregistration(env):
    coord, client = env
    a = _register(client, "node a")
    assert a == "node-a"
    b = _register(client, "node a", port=1001)  # same name, other address: distinct worker
    assert b != a
    assert _register(client, "node a") == a  # restart of the same worker keeps its id
    assert client.post(f"/workers/{a}/heartbeat", headers=H, json={"memory": {"free": 5}}).json() == {"ok": True}
    assert coord.registry.get(a).memory == {"free": 5}
    assert client.post("/workers/ghost/heartbeat", headers=H, json={}).status_code == 404
    st = client.get("/cluster/status", headers=H).json()
    assert {w["worker_id"] for w in st["workers"]} == {a, b}


def test_long_poll_delivers_bursts():
    reg = WorkerRegistry()
    w = reg.register(name="w", hardware={}, backend="cpu", device_info={}, data_host="h", data_port=1)
    t0 = time.monotonic()
    assert reg.poll(w.worker_id, 0.2) == [] and time.monotonic() - t0 >= 0.19
    reg.send(w.worker_id, {"type": "A"})
    reg.send(w.worker_id, {"type": "B"})
    assert [c["type"] for c in reg.poll(w.worker_id, 1)] == ["A", "B"]


def test_liveness_marks_offline_and_fails_running_job(env):
    coord, client = env
    a, b = _register(client, "a", port=1), _register(client, "b", port=2)
    job = client.post("/jobs", headers=H, json={"config": CFG}).json()
    assert job["status"] == "RUNNING"
    coord.registry.get(b).last_heartbeat -= 120
    gone = coord.registry.check_liveness()
    assert [w.worker_id for w in gone] == [b]
    j = client.get(f"/jobs/{job['job_id']}", headers=H).json()
    assert j["status"] == "FAILED" and "offline" in j["error"]
    assert coord.registry.get(a).status is WorkerStatus.ONLINE  # released


def _stage_commands(client, wid):
    return [c for c in client.get(f"/workers/{wid}/commands", headers=H, params={"wait": 0}).json()["commands"]
            if c["type"] == "START_STAGE"]


def test_job_lifecycle_and_artifacts(env):
    coord, client = env
    ws = [_register(client, n, port=i) for i, n in enumerate(("a", "b"))]
    plan = client.post("/plan", headers=H, json={"config": CFG}).json()
    assert len(plan["plan"]["stages"]) == 2 and "Stage 0" in plan["text"]
    job = client.post("/jobs", headers=H, json={"config": CFG}).json()
    jid = job["job_id"]
    cmds = {w: _stage_commands(client, w) for w in ws}
    assigned = {c[0]["stage_index"]: (w, c[0]) for w, c in cmds.items()}
    assert assigned[0][1]["downstream"]["port"] == coord.registry.get(assigned[1][0]).data_port
    assert assigned[1][1]["downstream"] is None and assigned[1][1]["data_job_id"] == jid
    for stage, (w, _) in assigned.items():
        for step in range(3):
            rec = {"event": "STEP_COMPLETE", "stage": stage, "step": step, "step_s": 0.1, "worker": w,
                   "backend": "cpu", "compute_s": 0.05, "memory": {"device_peak": 10}}
            if stage == 0:
                rec["loss"] = 2.0 - 0.1 * step
            client.post(f"/workers/{w}/events", headers=H,
                        json={"type": "stage_metrics", "data": {"job_id": jid, "attempt": 0, "record": rec}})
    spans = [{"category": "FORWARD_COMPUTE", "start": 1.0, "end": 1.1, "thread": "main", "step": 2,
              "microbatch": 0, "args": None}]
    for stage, (w, _) in assigned.items():
        client.post(f"/workers/{w}/events", headers=H, json={"type": "stage_done", "data": {
            "job_id": jid, "attempt": 0, "stage": stage, "summary": {}, "timeline": spans}})
    j = client.get(f"/jobs/{jid}", headers=H).json()
    assert j["status"] == "COMPLETED", j
    assert [l for _, l in j["losses"]] == pytest.approx([2.0, 1.9, 1.8])
    run = Path(j["run_dir"])
    for f in ("config.yaml", "plan.txt", "plan.json", "placement_attempts.json", "metrics.jsonl", "summary.json",
              "summary.txt", "prediction_accuracy.json", "timeline.json", "timeline_report.txt"):
        assert (run / f).exists(), f
    assert all(w.status is WorkerStatus.ONLINE for w in coord.registry.all())


def test_startup_oom_replans_with_smaller_budget(env):
    coord, client = env
    ws = [_register(client, n, port=i) for i, n in enumerate(("a", "b", "c"))]
    cfg = {**CFG, "placement": {"strategy": "auto"}}
    job = client.post("/jobs", headers=H, json={"config": cfg}).json()
    jid = job["job_id"]
    first = job["plan"]["stages"][0]["worker_id"]
    client.post(f"/workers/{first}/events", headers=H, json={"type": "stage_error", "data": {
        "job_id": jid, "attempt": 0, "stage": 0, "error": "CUDA out of memory", "oom": True, "steps_completed": 0,
        "memory_report": {"capacity": 1 * GB}}})
    j = client.get(f"/jobs/{jid}", headers=H).json()
    assert j["status"] == "RUNNING" and j["attempt"] == 1
    assert len(j["attempts"]) == 2 and j["attempts"][0]["failure"]["worker"] == first
    sf, fw = 0.85, int(0.25 * GB)
    assert coord.jobs[jid].budget_overrides[first] == min(int(8 * GB * 0.85), int((GB * 0.85 + fw) / sf))
    cmds = [c for w in ws for c in client.get(f"/workers/{w}/commands", headers=H,
                                              params={"wait": 0}).json()["commands"]]
    starts = [c for c in cmds if c["type"] == "START_STAGE" and c["attempt"] == 1]
    assert starts and all(c["data_job_id"] == f"{jid}.a1" for c in starts)
    assert any(c["type"] == "STOP_JOB" and c.get("attempt") == 0 for c in cmds)
    # a late event of attempt 0 is ignored
    client.post(f"/workers/{first}/events", headers=H, json={"type": "stage_error", "data": {
        "job_id": jid, "attempt": 0, "stage": 1, "error": "late", "oom": False}})
    assert client.get(f"/jobs/{jid}", headers=H).json()["status"] == "RUNNING"
    # OOM after training started is a plain failure
    client.post(f"/workers/{first}/events", headers=H, json={"type": "stage_error", "data": {
        "job_id": jid, "attempt": 1, "stage": 0, "error": "out of memory", "oom": True, "steps_completed": 4}})
    j = client.get(f"/jobs/{jid}", headers=H).json()
    assert j["status"] == "FAILED" and "out of memory" in j["error"]


def test_stop_job_and_unknown_job(env):
    coord, client = env
    _register(client, "a", port=1)
    _register(client, "b", port=2)
    jid = client.post("/jobs", headers=H, json={"config": CFG}).json()["job_id"]
    assert client.post(f"/jobs/{jid}/stop", headers=H).json()["status"] == "STOPPED"
    assert client.get("/jobs/none", headers=H).status_code == 404
    assert client.post("/jobs", headers=H, json={"config": {"model": {"type": "nope"}}}).status_code == 400


@pytest.mark.parametrize("memory,available", [
    ({}, None), ({"free": 0}, 0), ({"free": GB, "reserved": 2 * GB, "allocated": GB}, 2 * GB),
    ({"free": 10 * GB}, 4 * GB), ({"free": 0, "reserved": 6 * GB, "allocated": 2 * GB}, 0)])
def test_live_cuda_memory_budget(memory, available):
    assert live_cuda_budget(4 * GB, memory) == available
    w = WorkerRecord("w", "w", {"hostname": "h"}, "cuda", {"memory_total": 4 * GB}, "127.0.0.1", 1, memory=memory)
    p = worker_profile(w)
    assert p.memory_total == 4 * GB and p.memory_available == available and p.host == "h"


def test_nccl_jobs_get_device_links_and_rendezvous(env):
    coord, client = env
    ws = [_register(client, f"g{i}", backend="cuda", port=100 + 10 * i, memory=180 * GB, host="box")
          for i in range(2)]
    cfg = {"job": {"name": "dev"}, "network": {"tensor_transport": "nccl"},
           "model": {"type": "gpt", "layers": 4, "hidden_size": 256, "heads": 4, "vocab_size": 1000, "seq_len": 128,
                     "dtype": "bfloat16"},
           "training": {"batch_size": 8, "microbatch_size": 2, "steps": 2, "optimizer": "adam"},
           "placement": {"strategy": "topology_aware", "num_stages": 2}, "workers": {"allow": ["cuda"]}}
    job = client.post("/jobs", headers=H, json={"config": cfg}).json()
    assert job["plan"]["boundaries"][0]["forward"]["kind"] == "nccl"
    starts = [c for w in ws for c in client.get(f"/workers/{w}/commands", headers=H,
                                                params={"wait": 0}).json()["commands"]]
    assert {c["rendezvous"]["port"] for c in starts} == {starts[0]["rendezvous"]["port"]}
