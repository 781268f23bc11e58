"""HTTP client for the coordinator's control-plane API (token in ``X-MeshTrain-Token``).

One method per endpoint (reference networking/control.py:22-82).
"""

from __future__ import annotations

import httpx

TOKEN_HEADER = "X-MeshTrain-Token"


def normalize_address(addr: str) -> str:
    addr = addr.strip()
    if not addr.startswith(("http://", "https://")):
        addr = "http://" + addr
    return addr.rstrip("/")


class ControlClient:
    def __init__(self, address: str, token: str | None = None, timeout: float = 10.0, transport=None):
        self.base = normalize_address(address)
        headers = {TOKEN_HEADER: token} if token else {}
        self.http = httpx.Client(base_url=self.base, headers=headers, timeout=timeout, transport=transport)

    def _get(self, path: str, **params):
        r = self.http.get(path, params=params or None)
        r.raise_for_status()
        return r.json()

    def _post(self, path: str, body=None, timeout: float | None = None):
        r = self.http.post(path, json=body if body is not None else {}, timeout=timeout or self.http.timeout)
        r.raise_for_status()
        return r.json()

    def register(self, info: dict) -> dict:
        return self._post("/workers/register", info)

    def heartbeat(self, worker_id: str, info: dict | None = None) -> dict:
        return self._post(f"/workers/{worker_id}/heartbeat", info or {})

    def poll_commands(self, worker_id: str, wait_s: float = 5.0) -> list[dict]:
        r = self.http.get(f"/workers/{worker_id}/commands", params={"wait": wait_s}, timeout=wait_s + 10.0)
        r.raise_for_status()
        return r.json().get("commands", [])

    def post_event(self, worker_id: str, event: dict) -> dict:
        return self._post(f"/workers/{worker_id}/events", event)

    def status(self) -> dict:
        return self._get("/cluster/status")

    def start_benchmark(self, options: dict | None = None) -> dict:
        return self._post("/cluster/benchmark", options or {})

    def benchmark_status(self) -> dict:
        return self._get("/cluster/benchmark")

    def plan(self, config: dict) -> dict:
        return self._post("/plan", {"config": config}, timeout=120.0)

    def start_job(self, config: dict) -> dict:
        return self._post("/jobs", {"config": config}, timeout=120.0)

    def jobs(self) -> dict:
        return self._get("/jobs")

    def job(self, job_id: str) -> dict:
        return self._get(f"/jobs/{job_id}")

    def stop_job(self, job_id: str) -> dict:
        return self._post(f"/jobs/{job_id}/stop")

    def close(self) -> None:
        self.http.close()
