import json
import os
from pathlib import Path

import httpx
import pytest
import yaml
from fastapi.testclient import TestClient

from meshtrain_b200 import cli
from meshtrain_b200.config import ConfigError, load_config, parse_config
from meshtrain_b200.networking.control import ControlClient
from meshtrain_b200.terminal import Console, heading, paint, table, tools_help

ROOT = Path(__file__).resolve().parents[2]


@pytest.mark.parametrize("target,expect", [
    ("tok@10.0.0.2", ("10.0.0.2:8080", "tok")), ("10.0.0.2:9000", ("10.0.0.2:9000", None)),
    ("abc@http://host:81", ("host:81", "abc")), ("@h", ("h:8080", None))])
def test_join_target_parsing(target, expect):
    assert cli.parse_join_target(target) == expect


def test_remembered_cluster_is_private(tmp_path, monkeypatch):
    monkeypatch.setenv("MESHTRAIN_HOME", str(tmp_path))
    cli.save_cluster("h:1", "secret")
    assert cli.load_saved() == {"coordinator": "h:1", "token": "secret"}
    assert oct(os.stat(cli.state_path()).st_mode & 0o777) == "0o600"
    monkeypatch.delenv("MESHTRAIN_TOKEN", raising=False)
    assert cli.resolve_token() == "secret"


def test_parser_accepts_reference_command_lines():
    p = cli.build_parser()
    for argv in (["start", "--no-worker"], ["join", "t@h"], ["worker", "join", "h:1", "--device", "cuda:3"],
                 ["coordinator", "start", "--port", "9"], ["cluster", "status"], ["status"], ["jobs"],
                 ["cluster", "benchmark", "--output", "x.json"], ["benchmark", "pipeline", "--stages", "2"],
                 ["plan", "c.yaml"], ["inspect", "placement", "c.yaml", "--offline", "8"],
                 ["train", "c.yaml", "--local", "--stages", "3"], ["results", "record", "runs/x", "--section", "s"],
                 ["experiment", "capacity", "--mode", "b200"], ["dashboard", "--port", "9999"], ["console"]):
        assert callable(p.parse_args(argv).func), argv


@pytest.mark.parametrize("path", sorted((ROOT / "configs").glob("*.yaml")))
def test_shipped_configs_validate(path):
    cfg = load_config(path)
    assert cfg.model_num_layers() > 0


def test_config_rejects_unknown_keys_and_bad_batches():
    with pytest.raises(ConfigError):
        parse_config({"model": {"type": "mlp"}, "bogus": 1})
    with pytest.raises(ConfigError):
        parse_config({"model": {"type": "mlp"}, "training": {"batch_size": 10, "microbatch_size": 3}})
    with pytest.raises(ConfigError):
        parse_config({"model": {"type": "gpt", "hidden_size": 100, "heads": 3}})
    cfg = parse_config({"model": {"type": "mlp"}, "transport": {"async": False}})
    assert cfg.transport.async_ is False


def test_inspect_placement_offline_for_b200(tmp_path, capsys):
    c = {"model": {"type": "gpt", "layers": 8, "hidden_size": 512, "heads": 8, "vocab_size": 1024, "seq_len": 256,
                   "dtype": "bfloat16"}, "training": {"batch_size": 16, "microbatch_size": 2, "optimizer": "adam"},
         "pipeline": {"schedule": "1f1b"}}
    p = tmp_path / "c.yaml"
    p.write_text(yaml.safe_dump(c))
    assert cli.main(["inspect", "placement", str(p), "--offline", "4"]) == 0
    out = capsys.readouterr().out
    assert "Stage 3" in out or "stage 3" in out.lower()


def test_status_and_jobs_formatting():
    status = {"workers": [{"worker_id": "gpu0", "backend": "cuda", "device": {"name": "NVIDIA B200",
                                                                             "memory_total": 180 * 1024 ** 3},
                           "ram_total": 2 ** 40, "benchmark": {"compute_score": 1.0}, "status": "ONLINE",
                           "current_job": None}],
              "jobs": [{"job_id": "j1", "status": "COMPLETED"}]}
    out = cli.format_status(status)
    assert "gpu0" in out and "180.0 GB" in out and "1/1 workers" in out
    jobs = cli.format_jobs([{"job_id": "j1", "status": "FAILED", "losses": [[0, 2.0], [1, 1.5]],
                             "last_metrics": {"0": {"step_s": 0.25}}, "error": "boom", "created_at": 1}])
    assert "1.5" in jobs and "250.0" in jobs and "boom" in jobs


def test_terminal_helpers_without_tty(monkeypatch):
    monkeypatch.setenv("NO_COLOR", "1")
    assert paint("x", "bad") == "x"
    t = table(["A", "B"], [["ONLINE", "a-very-long-value"]], [6, 8])
    assert "a-ver..." in t and "ONLINE" in t
    assert "TRAINING" in tools_help() and heading("a", "b") == "a  b"


def test_console_dispatches_and_survives_errors():
    calls = []

    def runner(argv):
        calls.append(argv)
        if argv[0] == "boom":
            raise RuntimeError("bad")

    class A:
        coordinator, token = "h:1", "t"

    con = Console(A(), runner=runner)
    assert con.onecmd("status") is False
    assert calls[-1] == ["status", "--coordinator", "h:1", "--token", "t"]
    assert con.onecmd("boom") is False
    assert con.onecmd("start") is False and len(calls) == 2
    assert con.onecmd("exit") is True


def test_dashboard_proxies_snapshot_and_checks_host():
    def handler(request: httpx.Request):
        if request.url.path == "/cluster/status":
            return httpx.Response(200, json={"workers": [{"worker_id": "w"}], "jobs": []})
        if request.url.path == "/jobs":
            return httpx.Response(200, json={"jobs": [{"job_id": "j"}]})
        return httpx.Response(404)

    from meshtrain_b200.dashboard import create_app

    client = ControlClient("127.0.0.1:1", "t", transport=httpx.MockTransport(handler))
    app = TestClient(create_app(client), base_url="http://127.0.0.1")
    snap = app.get("/api/snapshot").json()
    assert snap["workers"][0]["worker_id"] == "w" and snap["jobs"][0]["job_id"] == "j"
    assert "meshtrain_b200" in app.get("/").text
    evil = TestClient(create_app(client), base_url="http://evil.example")
    assert evil.get("/api/snapshot").status_code == 400
