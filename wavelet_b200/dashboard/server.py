"""Read-only run dashboard: a run registry and a JSON API over run directories
(reference dashboard/server.py:24-379).  Nothing under a run is modified.

Routes (prefix ``/api``): ``health``, ``runs``, ``current`` and per run
``summary``, ``config``, ``metrics/keys``, ``series``, ``nodes``, ``evals``,
``rollouts``, ``rollouts/rows``, ``queue``, ``timeline``, ``events``,
``samples``, ``logs``, ``logs/{name}``, ``episodes``.  ``/`` serves the
static UI (``dashboard/static``).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

from .store import MetricTable, read_jsonl

API = "/api"
SOURCES = {"trainer": "metrics.jsonl", "orchestrator": "orchestrator_metrics.jsonl", "eval": "eval_metrics.jsonl"}


def is_run_dir(p: Path) -> bool:
    return p.is_dir() and any((p / n).exists() for n in ("metrics.jsonl", "run_metadata.json", "heartbeat.json",
                                                          "orchestrator_metrics.jsonl", "configs"))


class RunReader:
    def __init__(self, path: Path):
        self.path = Path(path)
        self.tables: dict[str, MetricTable] = {}

    @property
    def run_id(self) -> str:
        return self.path.name

    def _json(self, name: str) -> Any:
        p = self.path / name
        try:
            return json.loads(p.read_text())
        except (OSError, json.JSONDecodeError):
            return None

    def table(self, source: str) -> MetricTable:
        if source not in SOURCES:
            raise KeyError(f"unknown source {source!r} (one of {sorted(SOURCES)})")
        t = self.tables.get(source)
        if t is None:
            t = self.tables[source] = MetricTable(self.path / SOURCES[source])
        return t

    def summary(self) -> dict[str, Any]:
        hb = self._json("heartbeat.json") or {}
        meta = self._json("run_metadata.json") or {}
        t = self.table("trainer")
        t.refresh()
        ckpts = sorted(int(p.name.split("-")[1]) for p in self.path.glob("checkpoint-*")
                       if p.name.split("-")[1].isdigit() and (p / "STABLE").exists())
        return {"run_id": self.run_id, "path": str(self.path), "status": hb.get("status"), "step": hb.get("step"),
                "heartbeat": hb.get("timestamp"), "metadata": meta, "last_metrics": t.last,
                "checkpoints": ckpts, "num_metric_rows": len(t.steps)}

    def config(self) -> dict[str, Any]:
        d = self.path / "configs" / "latest" / "resolved"
        out = {}
        if d.exists():
            for p in sorted(d.glob("*.yaml")):
                out[p.name] = p.read_text()
        return out

    def metric_keys(self) -> dict[str, list[str]]:
        return {s: self.table(s).keys() for s in SOURCES}

    def series(self, source, keys, **kw) -> dict[str, Any]:
        return self.table(source).series(keys, **kw)

    def nodes(self) -> dict[str, Any]:
        hb = self._json("heartbeat.json") or {}
        last = self.table("trainer").last or {}
        return {"ranks": hb.get("ranks") or [], "node_metrics": {k: v for k, v in last.items() if k.startswith("node/")}}

    def evals(self) -> dict[str, Any]:
        envs = {}
        d = self.path / "evals"
        if d.exists():
            for env in sorted(p for p in d.iterdir() if p.is_dir()):
                envs[env.name] = sorted(int(p.stem.split("-")[1]) for p in env.glob("step-*.jsonl"))
        return {"metrics": read_jsonl(self.path / "eval_metrics.jsonl"), "envs": envs}

    def _queue_dir(self) -> Path:
        return self.path / "rollouts"

    def rollouts(self) -> list[dict[str, Any]]:
        out = []
        q = self._queue_dir()
        for d in sorted(q.glob("step-*")) if q.exists() else []:
            man = {}
            try:
                man = json.loads((d / "manifest.json").read_text())
            except (OSError, json.JSONDecodeError):
                pass
            out.append({"step": int(d.name.split("-")[1]), "stable": (d / "STABLE").exists(),
                        "claimed": (d / "claim.json").exists(), "consumed": (d / "consumed.json").exists(),
                        "manifest": man})
        return out

    def rollout_rows(self, step: int, offset: int = 0, limit: int = 50) -> dict[str, Any]:
        rows = read_jsonl(self._queue_dir() / f"step-{step:06d}" / "rollouts.jsonl")
        return {"step": step, "total": len(rows), "rows": rows[offset : offset + limit]}

    def queue(self) -> dict[str, Any]:
        r = self.rollouts()
        return {"published": len(r), "stable": sum(x["stable"] for x in r), "consumed": sum(x["consumed"] for x in r),
                "pending": [x["step"] for x in r if x["stable"] and not x["consumed"]],
                "events": read_jsonl(self.path / "events" / "queue.jsonl", 200)}

    def timeline(self) -> list[dict[str, Any]]:
        items = [{"kind": "event", "timestamp": e.get("timestamp"), "name": e.get("event"), "step": e.get("step")}
                 for e in read_jsonl(self.path / "events.jsonl")]
        pol = self.path / "policies"
        for d in sorted(pol.glob("step-*")) if pol.exists() else []:
            items.append({"kind": "policy", "name": d.name, "step": int(d.name.split("-")[1]),
                          "stable": (d / "STABLE").exists()})
        return sorted(items, key=lambda x: (x.get("timestamp") or "", x.get("step") or 0))

    def logs(self) -> list[str]:
        d = self.path / "logs" / "latest"
        return sorted(p.name for p in d.glob("*.log")) if d.exists() else []

    def log_tail(self, name: str, lines: int = 500) -> str:
        d = (self.path / "logs" / "latest").resolve()
        p = (d / name).resolve()
        if p.parent != d or not p.exists():
            raise FileNotFoundError(name)
        return "\n".join(p.read_text(errors="replace").splitlines()[-lines:])


class RunRegistry:
    def __init__(self, roots: list[Path] = (), runs: list[Path] = ()):
        self.roots = [Path(r) for r in roots]
        self.explicit = [Path(r) for r in runs]
        self.readers: dict[str, RunReader] = {}

    def discover(self) -> list[str]:
        paths = list(self.explicit)
        for root in self.roots:
            if root.exists():
                paths += [p for p in sorted(root.iterdir()) if is_run_dir(p)]
        for p in paths:
            rid = p.name
            if rid not in self.readers:
                self.readers[rid] = RunReader(p)
        return sorted(self.readers)

    def get(self, rid: str) -> RunReader | None:
        if rid not in self.readers:
            self.discover()
        return self.readers.get(rid)


def build_app(registry: RunRegistry, static_dir: Path | None = None):
    from fastapi import FastAPI, HTTPException, Query
    from fastapi.responses import FileResponse, PlainTextResponse

    app = FastAPI(title="wavelet_b200 dashboard")

    def reader(rid: str) -> RunReader:
        r = registry.get(rid)
        if r is None:
            raise HTTPException(404, f"unknown run {rid}")
        return r

    @app.get(f"{API}/health")
    def health():
        return {"ok": True}

    @app.get(f"{API}/runs")
    def runs():
        return {"runs": [registry.get(r).summary() for r in registry.discover()]}

    @app.get(f"{API}/current")
    def current():
        ids = registry.discover()
        if not ids:
            return {"run": None}
        latest = max(ids, key=lambda r: (registry.get(r).summary().get("heartbeat") or ""))
        return {"run": latest}

    @app.get(API + "/runs/{rid}/summary")
    def summary(rid: str):
        return reader(rid).summary()

    @app.get(API + "/runs/{rid}/config")
    def config(rid: str):
        return reader(rid).config()

    @app.get(API + "/runs/{rid}/metrics/keys")
    def keys(rid: str):
        return reader(rid).metric_keys()

    @app.get(API + "/runs/{rid}/series")
    def series(rid: str, source: str = "trainer", keys: str = "", limit: int = Query(0, ge=0, le=100_000),
               start: float | None = None, end: float | None = None, after: float | None = None,
               points: int = Query(0, ge=0, le=20_000)):
        try:
            return reader(rid).series(source, [k for k in keys.split(",") if k], start=start, end=end, after=after,
                                      limit=limit, points=points)
        except KeyError as e:
            raise HTTPException(400, str(e)) from None

    @app.get(API + "/runs/{rid}/nodes")
    def nodes(rid: str):
        return reader(rid).nodes()

    @app.get(API + "/runs/{rid}/evals")
    def evals(rid: str):
        return reader(rid).evals()

    @app.get(API + "/runs/{rid}/rollouts")
    def rollouts(rid: str):
        return {"batches": reader(rid).rollouts()}

    @app.get(API + "/runs/{rid}/rollouts/rows")
    def rollout_rows(rid: str, step: int, offset: int = Query(0, ge=0), limit: int = Query(50, ge=1, le=1000)):
        return reader(rid).rollout_rows(step, offset, limit)

    @app.get(API + "/runs/{rid}/episodes")
    def episodes(rid: str, limit: int = Query(50, ge=1, le=1000)):
        r = reader(rid)
        steps = [b["step"] for b in r.rollouts() if b["stable"]]
        return r.rollout_rows(steps[-1], 0, limit) if steps else {"rows": [], "total": 0}

    @app.get(API + "/runs/{rid}/live")
    def live_list(rid: str, limit: int = Query(200, ge=1, le=2000)):
        from ..orchestrator.live import list_episodes

        return {"episodes": list_episodes(reader(rid).path, limit)}

    @app.get(API + "/runs/{rid}/live/{eid}")
    def live_one(rid: str, eid: str):
        from ..orchestrator.live import read_episode

        doc = read_episode(reader(rid).path, eid)
        if doc is None:
            raise HTTPException(404, eid)
        return doc

    @app.get(API + "/runs/{rid}/queue")
    def queue(rid: str):
        return reader(rid).queue()

    @app.get(API + "/runs/{rid}/timeline")
    def timeline(rid: str):
        return {"items": reader(rid).timeline()}

    @app.get(API + "/runs/{rid}/events")
    def events(rid: str, limit: int = Query(500, ge=1, le=100_000)):
        return {"events": read_jsonl(reader(rid).path / "events.jsonl", limit)}

    @app.get(API + "/runs/{rid}/samples")
    def samples(rid: str, limit: int = Query(100, ge=1, le=10_000)):
        return {"samples": read_jsonl(reader(rid).path / "samples.jsonl", limit)}

    @app.get(API + "/runs/{rid}/logs")
    def logs(rid: str):
        return {"logs": reader(rid).logs()}

    @app.get(API + "/runs/{rid}/logs/{name}", response_class=PlainTextResponse)
    def log(rid: str, name: str, lines: int = Query(500, ge=1, le=100_000)):
        try:
            return reader(rid).log_tail(name, lines)
        except FileNotFoundError:
            raise HTTPException(404, name) from None

    if static_dir is not None and Path(static_dir).is_dir():
        index = Path(static_dir) / "index.html"

        @app.get("/")
        def root():
            return FileResponse(index)

    return app


def default_static_dir() -> Path:
    return Path(__file__).resolve().parent / "static"
