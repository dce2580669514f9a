"""Live episode traces (reference orchestrator/live.py:108-401).

A ``LiveEpisode`` appends ``episode_started`` / ``episode_turn`` /
``episode_finished`` events for one rollout episode to
``<run>/traces/live.jsonl`` as they happen (so a dashboard can follow an
agent episode before the batch is published).  Every event carries the
writer's pid and process start time; ``episode_abandoned`` flags episodes
whose writer died without finishing them.
"""

from __future__ import annotations

import os
import time
import uuid
from pathlib import Path
from typing import Any

from .trace import TraceWriter

_START = time.time()


class LiveEpisode:
    def __init__(self, run_dir: Path, *, task: str | None = None, step: int | None = None, enabled: bool = True):
        self.id = uuid.uuid4().hex[:12]
        self.trace = TraceWriter(run_dir, "live", enabled)
        self.task, self.step = task, step
        self.turns = 0
        self.finished = False

    def _emit(self, event: str, **kw: Any) -> None:
        self.trace.event(event, rollout_id=self.id, task=self.task, step=self.step, pid=os.getpid(),
                         process_start=_START, **kw)

    def __enter__(self) -> "LiveEpisode":
        self._emit("episode_started")
        return self

    def turn(self, *, prompt_tokens: int, output_tokens: int, **extra: Any) -> None:
        self.turns += 1
        self._emit("episode_turn", turn=self.turns, prompt_tokens=prompt_tokens, output_tokens=output_tokens, **extra)

    def finish(self, *, reward: float | None = None, error: str | None = None) -> None:
        if not self.finished:
            self.finished = True
            self._emit("episode_finished", turns=self.turns, reward=reward, error=error)

    def __exit__(self, et, ev, tb) -> None:
        self.finish(error=None if ev is None else f"{et.__name__}: {ev}")


def _alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
        return True
    except OSError:
        return False


def episode_abandoned(events: list[dict[str, Any]], rollout_id: str) -> bool:
    evs = [e for e in events if e.get("rollout_id") == rollout_id]
    if not evs or any(e["event"] == "episode_finished" for e in evs):
        return False
    pid = evs[-1].get("pid")
    return pid is None or not _alive(int(pid))
