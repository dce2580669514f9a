"""Structured trace events (JSONL) for rollouts, evals and policy updates.

One line per event under ``<output_dir>/traces/<subsystem>.jsonl`` with the
fields that ``wavelet convert-traces`` understands (reference
orchestrator/trace.py:17-60): ``format_version``, ``timestamp``,
``subsystem``, ``event`` and optional step / policy / task / rollout ids; any
other keys are kept as the event payload.
"""

from __future__ import annotations

import json
import os
import threading
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

FORMAT_VERSION = 1
TRACE_FIELDS = ("format_version", "timestamp", "subsystem", "event", "step", "queue_step", "optimizer_step",
                "policy_step", "task", "harness", "rollout_id")


class TraceWriter:
    def __init__(self, output_dir: Path | str, subsystem: str, enabled: bool = True):
        self.path = Path(output_dir) / "traces" / f"{subsystem}.jsonl"
        self.subsystem = subsystem
        self.enabled = enabled
        self._lock = threading.Lock()

    def event(self, event: str, **fields: Any) -> None:
        if not self.enabled:
            return
        row = {"format_version": FORMAT_VERSION, "timestamp": datetime.now(timezone.utc).isoformat(),
               "subsystem": self.subsystem, "event": event, **fields}
        line = json.dumps(row, default=str) + "\n"
        with self._lock:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            with self.path.open("a", encoding="utf-8") as f:
                f.write(line)
                f.flush()
                os.fsync(f.fileno())

    def rollouts(self, records, step: int, policy_step: int | None = None, task: str | None = None) -> None:
        """One ``rollout`` event per record: prompt/completion ids, reward, advantage."""
        for r in records:
            md = r.metadata or {}
            self.event("rollout", step=step, policy_step=policy_step, task=task or md.get("task"),
                       rollout_id=f"{md.get('group', step)}:{md.get('sample_index', 0)}",
                       prompt_ids=md.get("prompt_ids"), completion_ids=md.get("completion_ids"),
                       reward=r.reward, advantage=r.advantage, finish_reason=md.get("finish_reason"))
