"""``meshtrain start`` + ``meshtrain join TOKEN@HOST:PORT`` as real processes."""

import os
import signal
import socket
import subprocess
import sys
import time
from pathlib import Path

from meshtrain_b200.networking.control import ControlClient

ROOT = Path(__file__).resolve().parents[2]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_start_then_join(tmp_path):
    port, token = _port(), "joincode42"
    env = {**os.environ, "MESHTRAIN_HOME": str(tmp_path / "home"), "MESHTRAIN_QUIET": "1", "OMP_NUM_THREADS": "1",
           "PYTHONPATH": os.pathsep.join([str(ROOT), os.environ.get("PYTHONPATH", "")])}
    env.pop("MESHTRAIN_TOKEN", None)
    start = subprocess.Popen([sys.executable, "-m", "meshtrain_b200.cli", "start", "--no-worker", "--port", str(port),
                              "--host", "127.0.0.1", "--token", token, "--runs-dir", str(tmp_path / "runs"),
                              "--advertise-host", "127.0.0.1"], env=env, stdout=subprocess.PIPE,
                             stderr=subprocess.STDOUT, start_new_session=True)
    join = None
    client = ControlClient(f"127.0.0.1:{port}", token)
    try:
        for _ in range(300):
            try:
                client.status()
                break
            except Exception:  # noqa: BLE001
                time.sleep(0.1)
        join = subprocess.Popen([sys.executable, "-m", "meshtrain_b200.cli", "join", f"{token}@127.0.0.1:{port}",
                                 "--device", "cpu", "--name", "joiner", "--data-port", "0", "--advertise-host",
                                 "127.0.0.1"], env=env, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL,
                                start_new_session=True)
        workers = []
        for _ in range(600):
            workers = client.status()["workers"]
            if workers:
                break
            time.sleep(0.1)
        assert [w["worker_id"] for w in workers] == ["joiner"]
        assert workers[0]["status"] == "ONLINE"
        bad = ControlClient(f"127.0.0.1:{port}", "wrong-token")
        try:
            bad.status()
            raise AssertionError("a wrong token must be rejected")
        except Exception as exc:  # noqa: BLE001
            assert "401" in str(exc)
        finally:
            bad.close()
    finally:
        client.close()
        for p in (join, start):
            if p is not None:
                os.killpg(p.pid, signal.SIGTERM)
                try:
                    p.wait(15)
                except subprocess.TimeoutExpired:
                    os.killpg(p.pid, signal.SIGKILL)
                    p.wait(5)
    out = start.stdout.read().decode()
    assert f"meshtrain join {token}@127.0.0.1:{port}" in out
