"""Read-only browser view of a running coordinator.

``meshtrain dashboard`` serves ``dashboard.html`` on 127.0.0.1 plus one JSON
route, ``/api/snapshot``: workers and jobs fetched from the coordinator with
the cluster token.  The browser never sees the token, and only requests whose
Host header is localhost / 127.0.0.1 are answered, so another web page cannot
read the snapshot through DNS rebinding.  The page polls the snapshot every
two seconds (the reference's dashboard, dashboard.py:1-41, has the same two
routes).
"""

from __future__ import annotations

from contextlib import asynccontextmanager
from pathlib import Path

import httpx
from fastapi import FastAPI, HTTPException
from fastapi.responses import FileResponse
from starlette.middleware.trustedhost import TrustedHostMiddleware

PAGE = Path(__file__).with_name("dashboard.html")
LOCAL_HOSTS = ["localhost", "127.0.0.1"]


class SnapshotSource:
    """Everything the page shows, in one call to the coordinator pair of routes."""

    def __init__(self, client):
        self.client = client

    def __call__(self) -> dict:
        try:
            workers = self.client.status()["workers"]
            jobs = self.client.jobs()["jobs"]
        except httpx.HTTPError as exc:
            raise HTTPException(502, f"coordinator unreachable: {exc}") from exc
        return {"coordinator": self.client.base, "workers": workers, "jobs": jobs}


def create_app(client) -> FastAPI:
    snapshot = SnapshotSource(client)

    @asynccontextmanager
    async def closing_client(_app):
        yield
        client.close()

    app = FastAPI(lifespan=closing_client, docs_url=None, redoc_url=None, openapi_url=None)
    app.add_middleware(TrustedHostMiddleware, allowed_hosts=LOCAL_HOSTS)
    app.add_api_route("/", lambda: FileResponse(PAGE, headers={"Cache-Control": "no-store"}), methods=["GET"])
    app.add_api_route("/api/snapshot", snapshot, methods=["GET"])
    return app


def run_dashboard(client, port: int = 8081) -> None:
    import uvicorn

    print(f"dashboard: http://127.0.0.1:{port}  (Ctrl-C to close)", flush=True)
    uvicorn.run(create_app(client), host="127.0.0.1", port=port, log_level="warning")
