"""Metric history from trackers a run also logs to (ref dashboard/external.py).

Two providers, both read-only and best effort:

* ``wandb`` — the W&B run whose id the monitor persisted in
  ``wandb_run_id.txt`` (project / entity from the run's resolved config),
  read through ``wandb.Api().run(path).scan_history()``;
* ``trackio`` — Trackio's SQLite store under ``TRACKIO_DIR`` (default
  ``~/.cache/huggingface/trackio``), table ``metrics(run_name, step,
  timestamp, metrics)``; the run name and project come from the run's
  ``trackio_run.json`` sidecar or its W&B name / project settings.

A fetch runs on a background thread and is repeated after
``refresh_seconds``; readers always get the last good table and a status
(``unavailable`` / ``loading`` / ``ready`` / ``error``), so a slow or broken
tracker never blocks the dashboard's own files.
"""

from __future__ import annotations

import json
import os
import sqlite3
import threading
import time
from pathlib import Path
from typing import Any, Callable

from .store import MetricTable

SOURCES = ("wandb", "trackio")
REFRESH_SECONDS = 120.0
TRACKIO_SIDECAR = "trackio_run.json"


class RowsTable(MetricTable):
    """A metric table built from rows in memory (no file behind it)."""

    def __init__(self, rows: list[dict[str, Any]] | None = None):
        super().__init__(Path(os.devnull))
        for r in rows or []:
            self._append(r)

    def refresh(self) -> None:
        return


class ExternalSource:
    def __init__(self, name: str, fetch: Callable[[], list[dict[str, Any]]], available: bool, reason: str,
                 refresh_seconds: float = REFRESH_SECONDS):
        self.name, self.available, self.reason = name, available, reason
        self._fetch = fetch
        self._every = refresh_seconds
        self._table = RowsTable()
        self._lock = threading.Lock()
        self._thread: threading.Thread | None = None
        self._fetched_at: float | None = None
        self._error: str | None = None

    def table(self) -> MetricTable:
        self._maybe_refresh()
        with self._lock:
            return self._table

    def status(self) -> dict[str, Any]:
        self._maybe_refresh()
        with self._lock:
            if not self.available:
                state = "unavailable"
            elif self._fetched_at is None:
                state = "error" if self._error else "loading"
            else:
                state = "ready"
            return {"source": self.name, "status": state, "reason": self.reason, "error": self._error,
                    "rows": len(self._table.steps), "keys": len(self._table.cols),
                    "fetched_at": self._fetched_at,
                    "refreshing": self._thread is not None and self._thread.is_alive()}

    def _maybe_refresh(self) -> None:
        if not self.available:
            return
        with self._lock:
            if self._thread is not None and self._thread.is_alive():
                return
            if self._fetched_at is not None and time.time() - self._fetched_at < self._every:
                return
            if self._error is not None and self._fetched_at is None and self._thread is not None:
                return  # a failed first fetch is not retried on every request
            self._thread = threading.Thread(target=self.refresh_now, name=f"dashboard-{self.name}", daemon=True)
            self._thread.start()

    def refresh_now(self) -> None:
        try:
            table = RowsTable(self._fetch())
        except Exception as exc:  # noqa: BLE001 - reported as the source's status
            with self._lock:
                self._error = f"{type(exc).__name__}: {exc}"
            return
        with self._lock:
            self._table, self._error, self._fetched_at = table, None, time.time()


def _settings(cfg: dict[str, Any]) -> dict[str, Any]:
    return ((cfg or {}).get("monitor") or {}).get("wandb") or {}


def wandb_run_path(run_dir: Path, cfg: dict[str, Any]) -> str | None:
    try:
        rid = (Path(run_dir) / "wandb_run_id.txt").read_text(encoding="utf-8").strip()
    except OSError:
        return None
    if not rid:
        return None
    if "/" in rid:
        return rid
    w = _settings(cfg)
    project = w.get("project") or "wavelet"
    return f"{w['entity']}/{project}/{rid}" if w.get("entity") else f"{project}/{rid}"


def fetch_wandb_history(path: str, api: Any | None = None) -> list[dict[str, Any]]:
    if api is None:
        import wandb  # type: ignore

        api = wandb.Api(timeout=30)
    rows = []
    for rec in api.run(path).scan_history():
        row: dict[str, Any] = {}
        for k, v in rec.items():
            if k == "_step":
                row["step"] = v
            elif k == "_timestamp" and isinstance(v, (int, float)):
                row["timestamp"] = v
            elif not k.startswith("_"):
                row[k] = v
        rows.append(row)
    return rows


def wandb_source(run_dir: Path, cfg: dict[str, Any], api: Any | None = None) -> ExternalSource:
    w = _settings(cfg)
    path = wandb_run_path(run_dir, cfg)
    if not w.get("enabled") or w.get("mode") == "disabled":
        ok, why = False, "monitor.wandb is disabled for this run"
    elif path is None:
        ok, why = False, "no wandb_run_id.txt in the run directory"
    else:
        ok, why = True, f"W&B run {path}"
    return ExternalSource("wandb", lambda: fetch_wandb_history(path or "", api), ok, why)


def trackio_root() -> Path:
    env = os.environ.get("TRACKIO_DIR")
    return Path(env).expanduser() if env else Path.home() / ".cache" / "huggingface" / "trackio"


def trackio_identity(run_dir: Path, cfg: dict[str, Any]) -> tuple[str | None, str]:
    """(project, run name) of a run: the sidecar first, else the W&B names."""
    try:
        side = json.loads((Path(run_dir) / TRACKIO_SIDECAR).read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError):
        side = {}
    if isinstance(side, dict) and (side.get("run") or side.get("name")):
        return (str(side["project"]) if side.get("project") else None, str(side.get("run") or side.get("name")))
    w = _settings(cfg)
    return w.get("project"), w.get("name") or Path(run_dir).name


def _databases(root: Path, project: str | None) -> list[Path]:
    if not root.is_dir():
        return []
    if project:
        p = root / f"{project}.db"
        return [p] if p.is_file() else []
    return sorted(root.glob("*.db"))


def _query(db: Path, sql: str, args: tuple) -> list[tuple]:
    con = sqlite3.connect(f"file:{db}?mode=ro", uri=True)
    try:
        return con.execute(sql, args).fetchall()
    except sqlite3.DatabaseError:
        return []
    finally:
        con.close()


def fetch_trackio_history(dbs: list[Path], run: str) -> list[dict[str, Any]]:
    for db in dbs:
        rows = []
        for ts, step, metrics in _query(db, "SELECT timestamp, step, metrics FROM metrics WHERE run_name = ? "
                                            "ORDER BY step, id", (run,)):
            try:
                payload = json.loads(metrics) if isinstance(metrics, str) else None
            except json.JSONDecodeError:
                continue
            if isinstance(payload, dict):
                rows.append({"step": step, "timestamp": ts, **payload})
        if rows:
            return rows
    return []


def trackio_source(run_dir: Path, cfg: dict[str, Any], root: Path | None = None) -> ExternalSource:
    root = root or trackio_root()
    project, run = trackio_identity(run_dir, cfg)
    dbs = _databases(root, project)
    if not dbs:
        ok, why = False, f"no Trackio database under {root}"
    elif not any(_query(db, "SELECT 1 FROM metrics WHERE run_name = ? LIMIT 1", (run,)) for db in dbs):
        ok, why = False, f"run '{run}' not found in Trackio"
    else:
        ok, why = True, f"Trackio run {run} ({root})"
    return ExternalSource("trackio", lambda: fetch_trackio_history(dbs, run), ok, why)


class ExternalSources:
    """Both providers of one run directory."""

    def __init__(self, run_dir: Path, cfg: dict[str, Any], *, wandb_api: Any | None = None,
                 trackio_dir: Path | None = None):
        self.sources = {"wandb": wandb_source(run_dir, cfg, wandb_api),
                        "trackio": trackio_source(run_dir, cfg, trackio_dir)}

    def table(self, name: str) -> MetricTable:
        return self.sources[name].table()

    def status(self) -> list[dict[str, Any]]:
        return [self.sources[n].status() for n in SOURCES]

    def ready(self) -> list[str]:
        return [n for n in SOURCES if self.sources[n].status()["status"] == "ready"]
