"""Live episode traces (reference orchestrator/live.py:1-401).

Each rollout episode that is being generated has one small JSON document,
``<run>/traces/live/<id>.json``, rewritten atomically (temporary file +
rename) at every phase, next to a ``<id>.meta.json`` index entry (status,
phase, env, step, times, writer identity) that a dashboard lists without
opening the documents.  Documents are bounded so a misbehaving environment
cannot flood the disk: at most ``MAX_EVENTS`` events, strings cut at
``MAX_TEXT`` characters, containers at ``MAX_ITEMS`` items, ``MAX_BYTES`` per
document (older events dropped first).  When an episode ends (``completed``,
``error``, ``cancelled``) finished documents beyond the newest ``KEEP`` are
pruned.  ``episode_abandoned`` recognises an episode whose writer process on
this host died (its pid now has another start time, or is gone) without
expiring a slow one.

``LiveEpisode`` works as a sync or async context manager and registers
itself as the current episode of the task (a context variable), so hooks deep
inside an environment can add events with ``current_episode()``;
``install_environment_hooks`` wraps an environment's rollout / scoring
methods to record their start, end and errors.
"""

from __future__ import annotations

import asyncio
import contextvars
import functools
import inspect
import json
import math
import os
import socket
import time
import uuid
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

MAX_EVENTS = 128
MAX_TEXT = 8192
MAX_ITEMS = 128
MAX_BYTES = 256 * 1024
KEEP = 256
_META_KEYS = ("format_version", "id", "pid", "hostname", "process_start", "env", "kind", "status", "phase", "step",
              "policy_step", "example_id", "parent_id", "started_at", "finished_at")
_current: contextvars.ContextVar["LiveEpisode | None"] = contextvars.ContextVar("wavelet_live_episode", default=None)


def _now() -> str:
    return datetime.now(timezone.utc).isoformat()


def bounded(value: Any, depth: int = 0) -> Any:
    """A JSON-safe, size-bounded copy of ``value``."""
    if depth > 8:
        return "…"
    if value is None or isinstance(value, (bool, int)):
        return value
    if isinstance(value, float):
        return value if math.isfinite(value) else str(value)
    if isinstance(value, str):
        return value if len(value) <= MAX_TEXT else value[:MAX_TEXT] + f"… [{len(value) - MAX_TEXT} more]"
    if isinstance(value, BaseException):
        return bounded(f"{type(value).__name__}: {value}")
    if isinstance(value, dict):
        items = list(value.items())
        out = {str(k): bounded(v, depth + 1) for k, v in items[:MAX_ITEMS]}
        if len(items) > MAX_ITEMS:
            out["…"] = f"{len(items) - MAX_ITEMS} more"
        return out
    if isinstance(value, (list, tuple, set)):
        seq = list(value)
        out = [bounded(v, depth + 1) for v in seq[:MAX_ITEMS]]
        if len(seq) > MAX_ITEMS:
            out.append(f"… {len(seq) - MAX_ITEMS} more")
        return out
    if hasattr(value, "__dataclass_fields__"):
        return bounded({k: getattr(value, k) for k in value.__dataclass_fields__}, depth + 1)
    return bounded(repr(value), depth + 1)


def _atomic_json(path: Path, obj: dict) -> None:
    tmp = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    tmp.write_text(json.dumps(obj, sort_keys=True, separators=(",", ":")))
    os.replace(tmp, path)


def process_start(pid: int) -> str | None:
    """Start time of a local process (clock ticks since boot) or None."""
    try:
        return Path(f"/proc/{pid}/stat").read_text().rsplit(")", 1)[1].split()[19]
    except (OSError, IndexError):
        return None


def episode_abandoned(meta: dict[str, Any]) -> bool:
    """A running episode whose writer on this host is gone (a pid reused by
    another process counts as gone); episodes of other hosts are never judged."""
    if meta.get("status") != "running" or meta.get("hostname") != socket.gethostname():
        return False
    pid = meta.get("pid")
    if not isinstance(pid, int):
        return False
    start = meta.get("process_start")
    now = process_start(pid)
    return now is None or (start is not None and now != start)


class LiveEpisode:
    def __init__(self, run_dir: Path, env: str = "", kind: str = "train", *, step: int | None = None,
                 policy_step: int | None = None, example_id: str | None = None, parent_id: str | None = None,
                 enabled: bool = True):
        self.enabled = enabled
        self.dir = Path(run_dir) / "traces" / "live"
        self.id = uuid.uuid4().hex
        self.path = self.dir / f"{self.id}.json"
        pid = os.getpid()
        self.data: dict[str, Any] = {
            "format_version": 1, "id": self.id, "pid": pid, "hostname": socket.gethostname(),
            "process_start": process_start(pid), "env": env, "kind": kind, "status": "running", "phase": None,
            "step": step, "policy_step": policy_step, "example_id": example_id, "parent_id": parent_id,
            "started_at": _now(), "finished_at": None, "events": [],
        }
        self._token = None
        self._alock = None

    # ---------------------------------------------------------- recording
    def event(self, phase: str, **fields: Any) -> None:
        ev = self.data["events"]
        ev.append({"at": _now(), "phase": phase, **{k: bounded(v) for k, v in fields.items()}})
        del ev[:-MAX_EVENTS]
        self.data["phase"] = phase
        self._publish()

    def finish(self, status: str = "completed", **fields: Any) -> None:
        if self.data["status"] != "running":
            return
        self.data.update({k: bounded(v) for k, v in fields.items()})
        self.data["status"] = status
        self.data["finished_at"] = _now()
        self._publish()

    def _publish(self) -> None:
        if not self.enabled:
            return
        try:
            self.dir.mkdir(parents=True, exist_ok=True)
            doc = self.data
            raw = json.dumps(doc, separators=(",", ":"))
            while len(raw) > MAX_BYTES and doc["events"]:
                doc["events"] = doc["events"][len(doc["events"]) // 2 + 1:]
                doc["truncated"] = True
                raw = json.dumps(doc, separators=(",", ":"))
            _atomic_json(self.path, doc)
            meta = {k: doc.get(k) for k in _META_KEYS}
            meta["updated_at"] = _now()
            meta["revision"] = time.time_ns()
            _atomic_json(self.dir / f"{self.id}.meta.json", meta)
            if doc["status"] != "running":
                prune_finished(self.dir)
        except OSError:
            pass  # tracing never fails a rollout

    # ---------------------------------------------------------- contexts
    def __enter__(self) -> "LiveEpisode":
        self._token = _current.set(self)
        self.event("episode_started")
        return self

    def __exit__(self, et, ev, tb) -> None:
        try:
            if ev is None:
                self.finish("completed")
            else:
                self.finish("cancelled" if isinstance(ev, asyncio.CancelledError) else "error", error=ev)
        finally:
            if self._token is not None:
                _current.reset(self._token)

    async def __aenter__(self) -> "LiveEpisode":
        self._alock = asyncio.Lock()
        self._token = _current.set(self)
        await self.aevent("episode_started")
        return self

    async def __aexit__(self, et, ev, tb) -> None:
        try:
            async with self._alock:
                if ev is None:
                    await asyncio.to_thread(self.finish, "completed")
                else:
                    status = "cancelled" if isinstance(ev, asyncio.CancelledError) else "error"
                    await asyncio.to_thread(self.finish, status, error=ev)
        finally:
            if self._token is not None:
                _current.reset(self._token)

    async def aevent(self, phase: str, **fields: Any) -> None:
        async with self._alock:
            await asyncio.to_thread(self.event, phase, **fields)


def current_episode() -> LiveEpisode | None:
    return _current.get()


def prune_finished(live_dir: Path, keep: int = KEEP) -> int:
    """Delete finished (or abandoned) episodes beyond the newest ``keep``."""
    done = []
    for m in list(Path(live_dir).glob("*.meta.json"))[:4096]:
        try:
            meta = json.loads(m.read_text())
        except (OSError, ValueError):
            continue
        if meta.get("status") != "running" or episode_abandoned(meta):
            done.append((str(meta.get("updated_at", "")), m))
    done.sort()
    n = 0
    for _, m in done[:-keep] if keep > 0 else done:
        for p in (m, m.with_name(m.name.removesuffix(".meta.json") + ".json")):
            try:
                p.unlink()
            except OSError:
                pass
        n += 1
    return n


def list_episodes(run_dir: Path, limit: int = 200) -> list[dict[str, Any]]:
    """Index entries, running first then newest, each with ``abandoned``."""
    out = []
    for m in Path(run_dir, "traces", "live").glob("*.meta.json"):
        try:
            meta = json.loads(m.read_text())
        except (OSError, ValueError):
            continue
        meta["abandoned"] = episode_abandoned(meta)
        out.append(meta)
    out.sort(key=lambda x: (x.get("status") != "running" or x["abandoned"], str(x.get("updated_at", ""))),
             reverse=False)
    running = [x for x in out if x.get("status") == "running" and not x["abandoned"]]
    rest = sorted((x for x in out if x not in running), key=lambda x: str(x.get("updated_at", "")), reverse=True)
    return (sorted(running, key=lambda x: str(x.get("started_at", ""))) + rest)[:limit]


def read_episode(run_dir: Path, episode_id: str) -> dict[str, Any] | None:
    if not episode_id.isalnum():
        return None
    p = Path(run_dir, "traces", "live", f"{episode_id}.json")
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


_HOOK_METHODS = ("rollout", "run_rollout", "env_response", "score", "score_rollout", "score_group")
_MARK = "_wavelet_live_hooked"


def install_environment_hooks(env: Any) -> Any:
    """Wrap an environment's rollout / scoring methods so the current live
    episode records ``<method>_started`` / ``<method>_finished`` (with the
    error when one is raised); outside an episode the methods run untouched.
    Idempotent."""
    for name in _HOOK_METHODS:
        fn = getattr(env, name, None)
        if fn is None or not callable(fn) or getattr(fn, _MARK, False):
            continue
        if inspect.iscoroutinefunction(fn):
            @functools.wraps(fn)
            async def wrapped(*a, __fn=fn, __name=name, **kw):
                ep = current_episode()
                if ep is not None:
                    await ep.aevent(f"{__name}_started") if ep._alock else ep.event(f"{__name}_started")
                try:
                    out = await __fn(*a, **kw)
                except BaseException as e:
                    if ep is not None:
                        ep.event(f"{__name}_failed", error=e)
                    raise
                if ep is not None:
                    ep.event(f"{__name}_finished")
                return out
        else:
            @functools.wraps(fn)
            def wrapped(*a, __fn=fn, __name=name, **kw):
                ep = current_episode()
                if ep is not None:
                    ep.event(f"{__name}_started")
                try:
                    out = __fn(*a, **kw)
                except BaseException as e:
                    if ep is not None:
                        ep.event(f"{__name}_failed", error=e)
                    raise
                if ep is not None:
                    ep.event(f"{__name}_finished", result=out if isinstance(out, (int, float, str)) else None)
                return out
        setattr(wrapped, _MARK, True)
        setattr(env, name, wrapped)
    return env
