"""Live orchestrator state over HTTP (reference orchestrator/state_server.py).

``OrchestratorRunState`` is updated by the rollout loop (current step,
policy step, queue depth, last metrics, a bounded ring of recent events);
``maybe_state_server`` starts a FastAPI app on ``state_server.host:port``
in a daemon thread when ``orchestrator.state_server.enabled``.  Routes:
``/api/state``, ``/api/events?after=<seq>``, ``/api/health``, and the
dashboard's run API (``/api/runs/...``) for the run directory.
"""

from __future__ import annotations

import threading
import time
from collections import deque
from datetime import datetime, timezone
from pathlib import Path
from typing import Any


class OrchestratorRunState:
    def __init__(self, run_dir: Path, max_events: int = 2000):
        self.run_dir = Path(run_dir)
        self._lock = threading.Lock()
        self._events: deque = deque(maxlen=max_events)
        self._seq = 0
        self.state: dict[str, Any] = {"status": "starting", "step": None, "policy_step": None, "queue_depth": 0,
                                      "metrics": {}, "started_at": datetime.now(timezone.utc).isoformat()}

    def update(self, **fields) -> None:
        with self._lock:
            self.state.update(fields)
            self.state["updated_at"] = datetime.now(timezone.utc).isoformat()

    def event(self, name: str, **payload) -> None:
        with self._lock:
            self._seq += 1
            self._events.append({"seq": self._seq, "timestamp": datetime.now(timezone.utc).isoformat(),
                                 "event": name, **payload})

    def snapshot(self) -> dict[str, Any]:
        with self._lock:
            return dict(self.state)

    def events(self, after: int = 0) -> list[dict[str, Any]]:
        with self._lock:
            return [e for e in self._events if e["seq"] > after]


def build_state_app(run_state: OrchestratorRunState, cors: list[str] | None = None):
    from fastapi import FastAPI

    from ..dashboard.server import RunRegistry, build_app

    app = FastAPI(title="wavelet_b200 orchestrator state")
    if cors:
        from fastapi.middleware.cors import CORSMiddleware

        app.add_middleware(CORSMiddleware, allow_origins=cors, allow_methods=["GET"], allow_headers=["*"])

    @app.get("/api/health")
    def health():
        return {"ok": True}

    @app.get("/api/state")
    def state():
        return run_state.snapshot()

    @app.get("/api/events")
    def events(after: int = 0):
        return {"events": run_state.events(after)}

    app.mount("/runs", build_app(RunRegistry(runs=[run_state.run_dir])))
    return app


class StateServerHandle:
    def __init__(self, server, thread):
        self.server, self.thread = server, thread

    def close(self, timeout: float = 5.0) -> None:
        self.server.should_exit = True
        self.thread.join(timeout)


def maybe_state_server(cfg, run_state: OrchestratorRunState) -> StateServerHandle | None:
    sc = getattr(cfg.orchestrator, "state_server", None)
    if sc is None or not sc.enabled:
        return None
    import uvicorn

    server = uvicorn.Server(uvicorn.Config(build_state_app(run_state, sc.cors_allow_origins), host=sc.host,
                                           port=sc.port, log_level=sc.log_level))
    t = threading.Thread(target=server.run, daemon=True, name="state-server")
    t.start()
    for _ in range(100):
        if server.started:
            break
        time.sleep(0.05)
    return StateServerHandle(server, t)
