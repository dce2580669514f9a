"""Periodic pipeline status of the rollout role (reference
orchestrator/periodic_logger.py:1-70): a daemon thread that, every
``orchestrator.pipeline_status_interval_seconds``, logs one line with the
loaded policy, published / target queue steps, steps submitted, in flight
and finished-but-unpublished, and whether a policy load is under way, and
hands the same snapshot to an optional sink (the live state server)."""

from __future__ import annotations

import logging
import threading
from typing import Any, Callable

log = logging.getLogger("wavelet")


def pipeline_line(s: dict[str, Any]) -> str:
    pol = "none" if s.get("policy_step") is None else s["policy_step"]
    return (f"pipeline: policy {pol}, published {s['published']}/{s['target']}, submitted {s['submitted']}, "
            f"in flight {s['inflight']}, ready {s['ready']}, policy load {'running' if s['loading'] else 'idle'}")


class StatusReporter:
    def __init__(self, collect: Callable[[], dict[str, Any]], interval_s: float,
                 sink: Callable[[dict[str, Any]], None] | None = None):
        self.collect = collect
        self.interval_s = float(interval_s)
        self.sink = sink
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.emitted = 0

    def emit(self) -> dict[str, Any]:
        snap = self.collect()
        log.info(pipeline_line(snap))
        if self.sink is not None:
            try:
                self.sink(snap)
            except Exception as e:  # a status consumer never stops the pipeline
                log.debug("pipeline status sink failed: %s", e)
        self.emitted += 1
        return snap

    def _loop(self) -> None:
        while not self._stop.wait(self.interval_s):
            self.emit()

    def __enter__(self) -> "StatusReporter":
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="wavelet-pipeline-status", daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=min(self.interval_s, 5.0))
            self._thread = None
