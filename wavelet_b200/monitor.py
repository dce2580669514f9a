"""Run monitor: metrics, events, heartbeat, run metadata, samples and JSON logs.

On-disk layout (identical file names and row shapes to the reference's
RunMonitor, monitor.py:281-700, so its dashboard and tools read our runs):

    <output_dir>/metrics.jsonl      one row per log() (step, timestamp, metrics, resources)
    <output_dir>/metrics.csv        same rows, columns grown as new keys appear
    <output_dir>/events.jsonl       {timestamp, event, step, payload}
    <output_dir>/heartbeat.json     {timestamp, pid, status, step, metrics, ranks}
    <output_dir>/run_metadata.json  start time, pid, world, resumed_from, redacted config
    <output_dir>/samples.jsonl      bounded sample history
    <output_dir>/logs/<role>[.rank-N].jsonl   structured logs

    <output_dir>/wandb_run_id.txt   the W&B run id (resumed runs continue it)

Only the global rank 0 writes.  W&B is used when importable and enabled;
otherwise the run continues with local files (offline fallback).
"""

from __future__ import annotations

import csv
import datetime as _dt
import json
import logging
import math
import os
import shutil
from pathlib import Path
from typing import Any, Iterable

SECRET_HINTS = ("api_key", "apikey", "token", "secret", "password", "env_vars")


def perf_enabled() -> bool:
    """``WAVELET_PERF_LOG=1`` turns on ``WAVELET_PERF`` timing lines on stdout."""
    return os.environ.get("WAVELET_PERF_LOG", "").lower() in {"1", "true", "yes", "on"}


def emit_perf(event: str, *, force: bool = False, **fields: object) -> None:
    """One grep-able line, ``WAVELET_PERF <event> key=value ...`` (floats to
    3 decimals), the line shape of the reference's monitor.py:263-279."""
    if not (force or perf_enabled()):
        return
    vals = " ".join(f"{k}={v:.3f}" if isinstance(v, float) else f"{k}={v}" for k, v in fields.items())
    print(f"WAVELET_PERF {event}" + (f" {vals}" if vals else ""), flush=True)


def utc_now() -> str:
    return _dt.datetime.now(_dt.timezone.utc).isoformat()


def append_jsonl(path: Path, row: dict[str, Any]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a", encoding="utf-8") as f:
        f.write(json.dumps(row, default=str) + "\n")


def read_jsonl(path: Path) -> list[dict[str, Any]]:
    if not path.exists():
        return []
    out = []
    for line in path.read_text(encoding="utf-8").splitlines():
        line = line.strip()
        if not line:
            continue
        try:
            v = json.loads(line)
        except json.JSONDecodeError:
            continue  # a torn final line from a concurrent writer
        if isinstance(v, dict):
            out.append(v)
    return out


def tail_jsonl(path: Path, limit: int) -> list[dict[str, Any]]:
    return read_jsonl(path)[-limit:] if limit > 0 else []


def _write_json_atomic(path: Path, payload: Any) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(payload, indent=2, default=str))
    os.replace(tmp, path)


def redact(value: Any) -> Any:
    """Replace values under secret-looking keys with '***'."""
    if isinstance(value, dict):
        return {k: ("***" if any(h in str(k).lower() for h in SECRET_HINTS) and v else redact(v)) for k, v in value.items()}
    if isinstance(value, list):
        return [redact(v) for v in value]
    return value


def sanitize(row: dict[str, Any]) -> tuple[dict[str, Any], set[str]]:
    bad = set()
    out = {}
    for k, v in row.items():
        if isinstance(v, float) and not math.isfinite(v):
            bad.add(k)
            out[k] = None
        else:
            out[k] = v
    return out, bad


def series_stats(values: Iterable[float]) -> dict[str, float | int | None]:
    vals = [float(v) for v in values if v is not None and math.isfinite(float(v))]
    if not vals:
        return {"count": 0, "mean": None, "min": None, "max": None}
    return {"count": len(vals), "mean": sum(vals) / len(vals), "min": min(vals), "max": max(vals)}


def _append_csv(path: Path, row: dict[str, Any]) -> None:
    """Append a row; rewrite the file with a widened header when keys grow."""
    path.parent.mkdir(parents=True, exist_ok=True)
    if path.exists():
        with path.open(newline="", encoding="utf-8") as f:
            reader = csv.DictReader(f)
            header = list(reader.fieldnames or [])
            new = [k for k in row if k not in header]
            if new:
                rows = list(reader)
                header += new
                with path.open("w", newline="", encoding="utf-8") as g:
                    w = csv.DictWriter(g, fieldnames=header)
                    w.writeheader()
                    w.writerows(rows)
    else:
        header = list(row)
        with path.open("w", newline="", encoding="utf-8") as g:
            csv.DictWriter(g, fieldnames=header).writeheader()
    with path.open("a", newline="", encoding="utf-8") as g:
        csv.DictWriter(g, fieldnames=header).writerow({k: row.get(k) for k in header})


def _rank() -> int:
    return int(os.environ.get("RANK", "0"))


class RunMonitor:
    def __init__(self, output_dir: Path | str, *, checkpoint_dir: Path | None = None, enabled: bool = True,
                 write_events: bool = True, write_metrics_jsonl: bool = True, write_metrics_csv: bool = True,
                 write_run_metadata: bool = True, write_heartbeat: bool = True, log_cuda_memory: bool = True,
                 log_disk_usage: bool = True, sample_history_size: int = 256, wandb: Any = None):
        if sample_history_size < 1:
            raise ValueError("sample_history_size must be at least 1.")
        self.output_dir = Path(output_dir)
        self.checkpoint_dir = checkpoint_dir
        self.enabled = enabled
        self.write_events = write_events
        self.write_metrics_jsonl = write_metrics_jsonl
        self.write_metrics_csv = write_metrics_csv
        self.write_run_metadata = write_run_metadata
        self.write_heartbeat = write_heartbeat
        self.log_cuda_memory = log_cuda_memory
        self.log_disk_usage = log_disk_usage
        self.sample_history_size = sample_history_size
        self.wandb_cfg = wandb
        self.metrics_file = self.output_dir / "metrics.jsonl"
        self.csv_file = self.output_dir / "metrics.csv"
        self.samples_file = self.output_dir / "samples.jsonl"
        self.events_file = self.output_dir / "events.jsonl"
        self.heartbeat_file = self.output_dir / "heartbeat.json"
        self.run_metadata_file = self.output_dir / "run_metadata.json"
        self._wandb = None
        self._warned: set[str] = set()

    @classmethod
    def from_config(cls, output_dir: Path, cfg: Any, checkpoint_dir: Path | None = None) -> "RunMonitor":
        return cls(
            output_dir, checkpoint_dir=checkpoint_dir, enabled=cfg.enabled, write_events=cfg.write_events,
            write_metrics_jsonl=cfg.write_metrics_jsonl, write_metrics_csv=cfg.write_metrics_csv,
            write_run_metadata=cfg.write_run_metadata, write_heartbeat=cfg.write_heartbeat,
            log_cuda_memory=cfg.log_cuda_memory, log_disk_usage=cfg.log_disk_usage,
            sample_history_size=cfg.samples.keep_last, wandb=cfg.wandb,
        )

    def _active(self) -> bool:
        return self.enabled and _rank() == 0

    def start_run(self, *, run_config: dict[str, Any] | None = None, world: Any = None,
                  resumed_from: str | None = None) -> None:
        if not self._active():
            return
        self.output_dir.mkdir(parents=True, exist_ok=True)
        safe = redact(run_config)
        if self.write_run_metadata:
            meta = {
                "started_at": utc_now(),
                "pid": os.getpid(),
                "output_dir": str(self.output_dir),
                "world": {
                    "rank": getattr(world, "rank", 0),
                    "local_rank": getattr(world, "local_rank", 0),
                    "world_size": getattr(world, "world_size", 1),
                    "local_world_size": getattr(world, "local_world_size", 1),
                    "device": str(getattr(world, "device", "cpu")),
                },
                "resumed_from": resumed_from,
                "config": safe,
            }
            _write_json_atomic(self.run_metadata_file, meta)
        self._init_wandb(safe, resumed_from)
        self.log_event("run_resumed" if resumed_from else "run_started", payload={"resumed_from": resumed_from})
        self._heartbeat("running", None)

    def log(self, metrics: dict[str, Any], step: int | None, *, ranks: list[dict[str, Any]] | None = None) -> None:
        if not self._active():
            return
        row = dict(metrics)
        row["step"] = step
        row["timestamp"] = utc_now()
        row.update(self._resources())
        row, bad = sanitize(row)
        for k in sorted(bad - self._warned):
            logging.getLogger("wavelet").warning("Replacing non-finite metric %r with null.", k)
        self._warned |= bad
        if self.write_metrics_jsonl:
            append_jsonl(self.metrics_file, row)
        if self.write_metrics_csv:
            _append_csv(self.csv_file, row)
        if self._wandb is not None:
            try:
                self._wandb.log({k: v for k, v in row.items() if k != "timestamp" and k not in bad})
            except Exception:
                pass
        if ranks is not None:
            self._last_ranks = ranks
        self._heartbeat("running", step, row, ranks)

    def log_event(self, name: str, *, step: int | None = None, payload: dict[str, Any] | None = None) -> None:
        if not self._active() or not self.write_events:
            return
        append_jsonl(self.events_file, {"timestamp": utc_now(), "event": name, "step": step, "payload": payload or {}})

    def log_samples(self, samples: list[dict[str, Any]], step: int) -> None:
        if not self._active() or not samples:
            return
        ts = utc_now()
        rows = tail_jsonl(self.samples_file, self.sample_history_size) + [{"timestamp": ts, "step": step, **s} for s in samples]
        rows = rows[-self.sample_history_size:]
        tmp = self.samples_file.with_suffix(".jsonl.tmp")
        tmp.write_text("".join(json.dumps(r, default=str) + "\n" for r in rows))
        os.replace(tmp, self.samples_file)

    def finish(self, *, status: str, step: int | None) -> None:
        if not self._active():
            return
        self.log_event("run_finished", step=step, payload={"status": status})
        self._heartbeat(status, step, ranks=getattr(self, "_last_ranks", None))
        if self._wandb is not None:
            try:
                self._wandb.finish()
            except Exception:
                pass
            self._wandb = None

    # ------------------------------------------------------------ internals
    def _resources(self) -> dict[str, Any]:
        out: dict[str, Any] = {}
        if self.log_cuda_memory:
            try:
                import torch

                avail = torch.cuda.is_available()
                for n in ("memory_allocated", "memory_reserved", "max_memory_allocated", "max_memory_reserved"):
                    out[f"cuda_{n}_bytes"] = getattr(torch.cuda, n)() if avail else None
            except Exception:
                pass
        if self.log_disk_usage:
            out.update(_usage("disk", self.output_dir))
            if self.checkpoint_dir is not None:
                out.update(_usage("checkpoint_disk", self.checkpoint_dir))
        return out

    def _heartbeat(self, status, step, metrics=None, ranks=None) -> None:
        if not self.write_heartbeat:
            return
        payload: dict[str, Any] = {"timestamp": utc_now(), "pid": os.getpid(), "status": status, "step": step}
        if metrics is not None:
            payload["metrics"] = metrics
        if ranks is not None:
            payload["ranks"] = ranks
        self.output_dir.mkdir(parents=True, exist_ok=True)
        _write_json_atomic(self.heartbeat_file, payload)

    def _init_wandb(self, cfg: Any, resumed_from: str | None = None) -> None:
        """Start the W&B run (ref monitor.py:555-640).

        * A resumed run continues the W&B run whose id ``wandb_run_id.txt``
          holds (``resume="allow"``); every run writes its id there.
        * Shared mode (``WANDB_SHARED_MODE=1`` and ``WANDB_RUN_ID`` from the
          process launcher, online runs only): every role of one RL run logs
          into the same W&B run, labelled by ``WANDB_SHARED_LABEL``; the primary
          (``WANDB_SHARED_PRIMARY``, default the orchestrator) owns the run
          and the launcher finishes it after every role has exited.
        * An online start that fails falls back to an offline W&B run in the
          run directory (``monitor.wandb.offline_fallback``); without the
          package the run keeps its local files only.
        """
        w = self.wandb_cfg
        if w is None or not getattr(w, "enabled", False) or getattr(w, "mode", "disabled") == "disabled":
            return
        try:
            import wandb  # type: ignore
        except ImportError:
            self.log_event("wandb_unavailable", payload={"reason": "wandb is not installed; local files only"})
            return
        timeout = float(getattr(w, "init_timeout_seconds", 30.0))
        settings_cls = getattr(wandb, "Settings", None)
        shared = shared_wandb_settings(wandb, configured_mode=w.mode, init_timeout_seconds=timeout)
        prev = self._read_wandb_run_id() if shared is None and resumed_from is not None else None
        kwargs: dict[str, Any] = {"project": w.project or "wavelet", "entity": w.entity, "name": w.name,
                                  "group": w.group, "tags": w.tags, "config": cfg, "dir": str(self.output_dir),
                                  "id": prev, "resume": "allow" if prev is not None else None}
        if shared is not None:
            kwargs.update(shared)
        elif callable(settings_cls):
            kwargs["settings"] = settings_cls(init_timeout=timeout)
        online_overview = w.mode == "online"
        try:
            self._wandb = wandb.init(**kwargs) if shared is not None else wandb.init(mode=w.mode, **kwargs)
        except Exception as e:
            if w.mode != "online" or not getattr(w, "offline_fallback", True):
                raise
            self.log_event("wandb_init_failed", payload={"error": str(e), "fallback": "offline"})
            fb = {**kwargs, "id": None, "resume": None}
            if callable(settings_cls):
                fb["settings"] = settings_cls(init_timeout=timeout)
            try:
                self._wandb = wandb.init(mode="offline", **fb)
            except Exception as e2:  # no W&B at all: local files only
                self.log_event("wandb_init_failed", payload={"error": str(e2), "fallback": "local files"})
                self._wandb = None
                return
            online_overview = False
        define = getattr(self._wandb, "define_metric", None)
        if callable(define):  # every metric is plotted against the optimizer step
            define("step")
            define("*", step_metric="step")
        run_id = os.environ.get("WANDB_RUN_ID") if shared is not None else getattr(self._wandb, "id", None)
        self._write_wandb_run_id(run_id)
        if online_overview:
            from .wandb_overview import maybe_create_overview

            maybe_create_overview(self._wandb, cfg if isinstance(cfg, dict) else None, w)

    @property
    def wandb_run_id_file(self) -> Path:
        return self.output_dir / "wandb_run_id.txt"

    def _read_wandb_run_id(self) -> str | None:
        try:
            rid = self.wandb_run_id_file.read_text(encoding="utf-8").strip()
        except OSError:
            return None
        return rid or None

    def _write_wandb_run_id(self, run_id: object) -> None:
        if isinstance(run_id, str) and run_id:
            self.output_dir.mkdir(parents=True, exist_ok=True)
            self.wandb_run_id_file.write_text(run_id, encoding="utf-8")


def shared_wandb_settings(wandb: Any, *, configured_mode: str, init_timeout_seconds: float) -> dict[str, Any] | None:
    """``wandb.init`` arguments that join the launcher's shared run, or None
    when this process is not part of one."""
    if (os.environ.get("WANDB_SHARED_MODE") != "1" or configured_mode != "online"
            or os.environ.get("WANDB_MODE") in {"disabled", "offline"}):
        return None
    run_id = os.environ.get("WANDB_RUN_ID", "").strip()
    if not run_id:
        raise ValueError("WANDB_SHARED_MODE=1 requires WANDB_RUN_ID")
    settings_cls = getattr(wandb, "Settings", None)
    if not callable(settings_cls):
        raise TypeError("the installed W&B SDK has no Settings for shared runs")
    label = os.environ.get("WANDB_SHARED_LABEL")
    primary = os.environ.get("WANDB_SHARED_PRIMARY", "orchestrator")
    finisher = os.environ.get("WANDB_SHARED_FINISHER", primary)
    return {"id": run_id, "resume": "allow",
            "settings": settings_cls(mode="shared", init_timeout=init_timeout_seconds, x_label=label,
                                     x_primary=label == primary, x_update_finish_state=label == finisher)}


def shared_wandb_environment(cfg: Any) -> dict[str, str]:
    """Environment that makes every role of a process-mode RL run log into
    one W&B run (online runs only): a fresh run id, or the persisted one when
    the run resumes from a checkpoint (ref orchestrator/runtime.py:559-585)."""
    import secrets

    w = cfg.monitor.wandb
    if not w.enabled or w.mode != "online" or os.environ.get("WANDB_MODE") in {"disabled", "offline"}:
        return {}
    out = Path(cfg.output_dir)
    id_file = out / "wandb_run_id.txt"
    run_id = os.environ.get("WANDB_RUN_ID", "").strip()
    ck = getattr(cfg, "ckpt", None)
    if not run_id and ck is not None and ck.is_resuming and id_file.exists():
        run_id = id_file.read_text(encoding="utf-8").strip()
    run_id = run_id or secrets.token_hex(4)
    out.mkdir(parents=True, exist_ok=True)
    id_file.write_text(run_id, encoding="utf-8")
    return {"WANDB_SHARED_MODE": "1", "WANDB_RUN_ID": run_id}


def finish_shared_wandb_run(cfg: Any, shared_env: dict[str, str], *, exit_code: int) -> None:
    """Close the shared run once the launcher has joined every role."""
    if not shared_env:
        return
    try:
        import wandb  # type: ignore

        run = wandb.init(id=shared_env["WANDB_RUN_ID"], project=cfg.monitor.wandb.project or "wavelet",
                         entity=cfg.monitor.wandb.entity, dir=str(cfg.output_dir),
                         settings=wandb.Settings(mode="shared", x_label="launcher", x_primary=False,
                                                 x_update_finish_state=True,
                                                 init_timeout=cfg.monitor.wandb.init_timeout_seconds))
        run.finish(exit_code=exit_code)
    except Exception as e:  # noqa: BLE001 - the roles' data is already uploaded
        logging.getLogger("wavelet").warning("could not finish the shared W&B run: %s", e)


def _usage(prefix: str, path: Path) -> dict[str, Any]:
    p = Path(path)
    while not p.exists() and p != p.parent:
        p = p.parent
    try:
        u = shutil.disk_usage(p)
    except OSError:
        return {}
    return {f"{prefix}_total_bytes": u.total, f"{prefix}_used_bytes": u.used, f"{prefix}_free_bytes": u.free}


class JsonLogFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        payload = {
            "timestamp": utc_now(),
            "level": record.levelname.lower(),
            "logger": record.name,
            "message": record.getMessage(),
            "rank": _rank(),
        }
        if record.exc_info:
            payload["exception"] = self.formatException(record.exc_info)
        return json.dumps(payload)


def setup_logger(name: str, output_dir: Path | str | None = None, level: str = "info", json_console: bool = False,
                 json_file: bool = True) -> logging.Logger:
    log = logging.getLogger("wavelet")
    log.setLevel(level.upper())
    for h in list(log.handlers):
        if getattr(h, "_wavelet_managed", False):
            log.removeHandler(h)
    ch = logging.StreamHandler()
    ch.setFormatter(JsonLogFormatter() if json_console else logging.Formatter("[%(asctime)s %(levelname)s] %(message)s"))
    ch._wavelet_managed = True  # type: ignore[attr-defined]
    log.addHandler(ch)
    if output_dir is not None and json_file:
        r = _rank()
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        safe = "".join(c if c.isalnum() or c in "-_" else "_" for c in name)
        path = Path(output_dir) / "logs" / f"{safe}{f'.rank-{r}' if ws > 1 else ''}.jsonl"
        path.parent.mkdir(parents=True, exist_ok=True)
        fh = logging.FileHandler(path)
        fh.setFormatter(JsonLogFormatter())
        fh._wavelet_managed = True  # type: ignore[attr-defined]
        log.addHandler(fh)
    log.propagate = False
    return log
