"""Read-only browser dashboard for a running coordinator (reference dashboard.py:1-41).

Serves ``dashboard.html`` on 127.0.0.1 and one JSON route, ``/api/snapshot``,
which proxies the coordinator's status and jobs with the cluster token, so the
token never reaches the browser.  Host-header checking keeps other sites from
reading it through DNS rebinding.
"""

from __future__ import annotations

from contextlib import asynccontextmanager
from pathlib import Path

import httpx
from fastapi import FastAPI, HTTPException
from fastapi.responses import FileResponse
from starlette.middleware.trustedhost import TrustedHostMiddleware

PAGE = Path(__file__).with_name("dashboard.html")


def create_app(client) -> FastAPI:
    @asynccontextmanager
    async def lifespan(app):
        yield
        client.close()

    app = FastAPI(lifespan=lifespan, docs_url=None, redoc_url=None, openapi_url=None)
    app.add_middleware(TrustedHostMiddleware, allowed_hosts=["localhost", "127.0.0.1"])

    @app.get("/")
    def index():
        return FileResponse(PAGE, headers={"Cache-Control": "no-store"})

    @app.get("/api/snapshot")
    def snapshot():
        try:
            status = client.status()
            return {"coordinator": client.base, "workers": status["workers"], "jobs": client.jobs()["jobs"]}
        except httpx.HTTPError as exc:
            raise HTTPException(502, f"coordinator unreachable: {exc}") from exc

    return app


def run_dashboard(client, port: int = 8081) -> None:
    import uvicorn

    print(f"dashboard: http://127.0.0.1:{port}  (Ctrl-C to close)", flush=True)
    uvicorn.run(create_app(client), host="127.0.0.1", port=port, log_level="warning")
