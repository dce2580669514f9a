"""Deterministic Python garbage collection at step boundaries.

Automatic collection is disabled and generation-1 collections run every
``interval`` optimizer steps on every rank at the same point, so no rank
stalls in the middle of a collective waiting for another rank's collector
(reference trainer/garbage_collection.py:10-40).
"""

from __future__ import annotations

import gc
import logging
import time

log = logging.getLogger("wavelet")


class StepGarbageCollector:
    def __init__(self, interval: int):
        if interval < 1:
            raise ValueError("gc.interval must be positive")
        self.interval = interval
        self._was_enabled = gc.isenabled()
        self._closed = False
        gc.disable()
        self.collect()

    def run(self, step: int) -> None:
        if step > 0 and step % self.interval == 0:
            self.collect()

    @staticmethod
    def collect() -> float:
        t0 = time.monotonic()
        gc.collect(1)
        dt = time.monotonic() - t0
        log.debug("gc generation 1 took %.3fs", dt)
        return dt

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            if self._was_enabled:
                gc.enable()
