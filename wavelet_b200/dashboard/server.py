"""Read-only run dashboard: a run registry and a JSON API over run directories
(reference dashboard/server.py:24-379).  Nothing under a run is modified.

Routes (prefix ``/api``): ``health``, ``runs``, ``current`` and per run
``summary``, ``config``, ``metrics/keys``, ``series`` (sources ``trainer``,
``orchestrator``, ``eval`` and the external trackers ``wandb`` / ``trackio``),
``external``, ``nodes``, ``evals``, ``evals/{step}/{env}/rows`` (filtered,
sorted, paged), ``rollouts``, ``rollouts/rows``, ``queue``, ``timeline``,
``events``, ``samples``, ``logs``, ``logs/{name}``, ``episodes``,
``episodes/{id}``, ``live``, ``live/{id}``.  ``/`` serves the static UI
(``dashboard/static``).
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


def _num(v: Any) -> float | None:
    return float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else None


def eval_row(i: int, r: dict[str, Any]) -> dict[str, Any]:
    """An evaluation rollout as a table row (native and verifiers-package rows)."""
    traj = r.get("trajectory") or []
    n = sum(len(((st or {}).get("tokens") or {}).get("completion_ids") or []) for st in traj) if traj \
        else len(r.get("completion_ids") or [])
    return {"row_index": i, "example_id": None if r.get("example_id") is None else str(r.get("example_id")),
            "reward": _num(r.get("reward")), "error": r.get("error"), "is_truncated": bool(r.get("is_truncated")),
            "completion_len": n, "row": r}


ROLLOUT_SORT_KEYS = ("row_index", "reward", "advantage", "completion_token_count", "input_token_count",
                     "logprob_mean", "logprob_min", "group_key", "env", "example_id", "policy_step", "turn_count")


def rollout_row(i: int, r: dict[str, Any], full: bool = False) -> dict[str, Any]:
    """A rollout record as a compact table row (the record itself with ``full``)."""
    md = r.get("metadata") or {}
    lps = [x for x in (r.get("inference_logprobs") or []) if isinstance(x, (int, float))]
    mask = r.get("loss_mask") or []
    adv = r.get("advantage")
    text = " ".join(str(m.get("content") or "") for m in (r.get("completion") or []) if isinstance(m, dict))
    out = {"row_index": i, "reward": _num(r.get("reward")), "advantage": _num(adv) if not isinstance(adv, list)
           else (sum(adv) / len(adv) if adv else None),
           "completion_token_count": md.get("completion_token_count", sum(bool(x) for x in mask)),
           "input_token_count": len(r.get("input_ids") or []),
           "logprob_mean": sum(lps) / len(lps) if lps else None, "logprob_min": min(lps) if lps else None,
           "group_key": None if md.get("group") is None else str(md.get("group")),
           "env": md.get("env") or r.get("source"), "example_id": None if md.get("example_id") is None
           else str(md.get("example_id")), "policy_step": md.get("policy_step"),
           "is_truncated": bool(md.get("is_truncated")), "turn_count": md.get("turn_count"),
           "stop_condition": md.get("stop_condition") or md.get("finish_reason"), "text": text[:3000]}
    if full:
        out["row"] = r
    return out


def filter_rows(rows: list[dict[str, Any]], *, example_id: str | None = None, min_reward: float | None = None,
                max_reward: float | None = None, truncated: bool | None = None,
                has_error: bool | None = None, env: str | None = None, group_key: str | None = None,
                advantage_sign: str | None = None, search: str | None = None) -> list[dict[str, Any]]:
    out = []
    for r in rows:
        rw = r.get("reward")
        if example_id is not None and r.get("example_id") != example_id:
            continue
        if env is not None and r.get("env") != env:
            continue
        if group_key is not None and r.get("group_key") != group_key:
            continue
        if advantage_sign is not None:
            a = r.get("advantage")
            sign = "zero" if not a else ("positive" if a > 0 else "negative")
            if sign != advantage_sign:
                continue
        if search and search.lower() not in str(r.get("text", "")).lower():
            continue
        if min_reward is not None and (rw is None or rw < min_reward):
            continue
        if max_reward is not None and (rw is None or rw > max_reward):
            continue
        if truncated is not None and bool(r.get("is_truncated")) != truncated:
            continue
        if has_error is not None and (r.get("error") is not None) != has_error:
            continue
        out.append(r)
    return out


def summarize(values: list[float]) -> dict[str, Any]:
    if not values:
        return {"count": 0}
    v = sorted(values)
    return {"count": len(v), "mean": sum(v) / len(v), "min": v[0], "max": v[-1], "median": v[len(v) // 2]}


EVAL_SORT_KEYS = ("row_index", "reward", "completion_len", "example_id")


class RunReader:
    def __init__(self, path: Path):
        self.path = Path(path)
        self.tables: dict[str, MetricTable] = {}
        self._external = None

    def resolved_config(self) -> dict[str, Any]:
        """The run's resolved config (the first role file of the latest launch)."""
        import yaml

        d = self.path / "configs" / "latest" / "resolved"
        for name in ("rl.yaml", "sft.yaml", "rl_trainer.yaml", "rl_inference.yaml"):
            p = d / name
            if p.is_file():
                try:
                    return yaml.safe_load(p.read_text()) or {}
                except yaml.YAMLError:
                    return {}
        return {}

    def external(self):
        from .external import ExternalSources

        if self._external is None:
            self._external = ExternalSources(self.path, self.resolved_config())
        return self._external

    def external_status(self) -> list[dict[str, Any]]:
        return self.external().status()

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
        from .external import SOURCES as EXTERNAL

        if source in EXTERNAL:
            return self.external().table(source)
        if source not in SOURCES:
            raise KeyError(f"unknown source {source!r} (one of {sorted(SOURCES) + list(EXTERNAL)})")
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
        out = {s: self.table(s).keys() for s in SOURCES}
        for s in self.external().ready():  # trackers a run also logs to, once fetched
            out[s] = self.table(s).keys()
        return out

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

    def eval_rows(self, step: int, env: str, *, sort: str = "row_index", descending: bool = False,
                  offset: int = 0, limit: int = 50, **filters) -> dict[str, Any]:
        """One evaluation's rollouts, filtered, sorted and paged, with reward statistics."""
        d = (self.path / "evals").resolve()
        p = (d / env / f"step-{step}.jsonl").resolve()
        if p.parent.parent != d or not p.is_file():
            return {"available": False, "reason": f"no eval rollouts for step {step} env {env}"}
        rows = [eval_row(i, r) for i, r in enumerate(read_jsonl(p))]
        kept = filter_rows(rows, **filters)
        key = sort if sort in EVAL_SORT_KEYS else "row_index"
        have = sorted((r for r in kept if r.get(key) is not None), key=lambda r: r[key], reverse=descending)
        kept = have + [r for r in kept if r.get(key) is None]  # rows without the key last, either order
        rewards = [r["reward"] for r in rows if r["reward"] is not None]
        return {"available": True, "step": step, "env": env, "total": len(rows), "filtered": len(kept),
                "stats": {"reward": summarize(rewards),
                          "errors": sum(r["error"] is not None for r in rows),
                          "truncated": sum(r["is_truncated"] for r in rows)},
                "rows": kept[offset : offset + limit]}

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

    def rollout_rows(self, step: int, offset: int = 0, limit: int = 50, *, view: bool = False, sort: str = "row_index",
                     descending: bool = False, full: bool = False, **filters) -> dict[str, Any]:
        """A queue step's rollout records; ``view`` returns compact rows that
        can be filtered and sorted (with reward / advantage statistics)."""
        rows = read_jsonl(self._queue_dir() / f"step-{step:06d}" / "rollouts.jsonl")
        if not view:
            return {"step": step, "total": len(rows), "rows": rows[offset : offset + limit]}
        vs = [rollout_row(i, r, full) for i, r in enumerate(rows)]
        kept = filter_rows(vs, **filters)
        key = sort if sort in ROLLOUT_SORT_KEYS else "row_index"
        have = sorted((r for r in kept if r.get(key) is not None), key=lambda r: r[key], reverse=descending)
        kept = have + [r for r in kept if r.get(key) is None]
        return {"step": step, "total": len(vs), "filtered": len(kept),
                "stats": {"reward": summarize([r["reward"] for r in vs if r["reward"] is not None]),
                          "advantage": summarize([r["advantage"] for r in vs if r["advantage"] is not None]),
                          "truncated": sum(r["is_truncated"] for r in vs)},
                "rows": kept[offset : offset + limit]}

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

    @app.get(API + "/runs/{rid}/evals/{step}/{env}/rows")
    def eval_rows(rid: str, step: int, env: str, sort: str = "row_index", order: str = "asc",
                  offset: int = Query(0, ge=0), limit: int = Query(50, ge=1, le=500), example_id: str | None = None,
                  min_reward: float | None = None, max_reward: float | None = None, truncated: bool | None = None,
                  has_error: bool | None = None):
        return reader(rid).eval_rows(step, env, sort=sort, descending=order == "desc", offset=offset, limit=limit,
                                     example_id=example_id, min_reward=min_reward, max_reward=max_reward,
                                     truncated=truncated, has_error=has_error)

    @app.get(API + "/runs/{rid}/external")
    def external(rid: str):
        return reader(rid).external_status()

    @app.get(API + "/runs/{rid}/episodes/{eid}")
    def episode(rid: str, eid: str):
        from ..orchestrator.live import read_episode

        doc = read_episode(reader(rid).path, eid)
        if doc is None:
            raise HTTPException(404, "episode snapshot unavailable")
        return doc

    @app.get(API + "/runs/{rid}/rollouts")
    def rollouts(rid: str):
        return {"batches": reader(rid).rollouts()}

    @app.get(API + "/runs/{rid}/rollouts/rows")
    def rollout_rows(rid: str, step: int, offset: int = Query(0, ge=0), limit: int = Query(50, ge=1, le=1000),
                     view: bool = False, sort: str = "row_index", order: str = "asc", full: bool = False,
                     env: str | None = None, group_key: str | None = None, example_id: str | None = None,
                     min_reward: float | None = None, max_reward: float | None = None, truncated: bool | None = None,
                     advantage_sign: str | None = None, search: str | None = None):
        if not view:
            return reader(rid).rollout_rows(step, offset, limit)
        return reader(rid).rollout_rows(step, offset, limit, view=True, sort=sort, descending=order == "desc",
                                        full=full, env=env, group_key=group_key, example_id=example_id,
                                        min_reward=min_reward, max_reward=max_reward, truncated=truncated,
                                        advantage_sign=advantage_sign, search=search)

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
