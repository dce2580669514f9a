"""Rollout and policy metadata helpers (reference
orchestrator/rollout_metadata.py, policy_metadata.py,
periodic_logger.py)."""

from __future__ import annotations

import logging
import time
from pathlib import Path
from typing import Any

log = logging.getLogger("wavelet")


def metadata_task_name(md: dict[str, Any] | None) -> str | None:
    md = md or {}
    return md.get("task") or md.get("env") or md.get("source")


def rollout_task_metadata(records) -> dict[str, float]:
    """Per-task counts, mean reward, truncation rate and completion length."""
    by: dict[str, list] = {}
    for r in records:
        by.setdefault(metadata_task_name(r.metadata) or "default", []).append(r)
    out: dict[str, float] = {}
    for task, rs in by.items():
        n = len(rs)
        out[f"task/{task}/count"] = float(n)
        out[f"task/{task}/reward_mean"] = sum(float(r.reward or 0.0) for r in rs) / n
        out[f"task/{task}/truncated_rate"] = sum(bool((r.metadata or {}).get("is_truncated")) for r in rs) / n
        out[f"task/{task}/completion_tokens"] = sum(
            float((r.metadata or {}).get("completion_token_count") or 0) for r in rs) / n
    return out


def error_metric_name(error: object) -> str:
    name = type(error).__name__ if isinstance(error, BaseException) else str(error)
    return "errors/" + "".join(c if c.isalnum() or c in "_-" else "_" for c in name)[:64]


def precision_metadata(cfg) -> dict[str, Any]:
    return {"trainer_dtype": "bfloat16", "master_dtype": "float32", "lora": cfg.lora is not None,
            "load_in_4bit": bool(getattr(cfg.model, "load_in_4bit", False))}


def policy_metadata(cfg, step: int, kind: str) -> dict[str, Any]:
    return {"step": step, "kind": kind, "model": cfg.model.name, "precision": precision_metadata(cfg)}


def adapter_artifact_metadata(adapter_dir: Path) -> dict[str, Any] | None:
    p = Path(adapter_dir)
    if not (p / "adapter_config.json").exists():
        return None
    import json

    cfg = json.loads((p / "adapter_config.json").read_text())
    return {"r": cfg.get("r"), "lora_alpha": cfg.get("lora_alpha"), "target_modules": cfg.get("target_modules"),
            "bytes": sum(f.stat().st_size for f in p.iterdir() if f.is_file())}


def pipeline_status(*, step: int, policy_step: int | None, queue_depth: int, inflight: int, limit: int) -> str:
    lag = None if policy_step is None else step - policy_step
    return f"step={step} policy={policy_step} lag={lag} queue={queue_depth} inflight={inflight}/{limit}"


class PeriodicLogger:
    """Logs ``status()`` at most every ``interval`` seconds."""

    def __init__(self, interval: float = 30.0):
        self.interval = interval
        self._last = 0.0

    def maybe_log(self, status) -> bool:
        now = time.monotonic()
        if now - self._last < self.interval:
            return False
        self._last = now
        log.info("pipeline %s", status() if callable(status) else status)
        return True
