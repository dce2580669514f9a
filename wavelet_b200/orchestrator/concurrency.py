"""Rollout concurrency control (reference orchestrator/concurrency.py:43 and
admission.py:20).

``AdaptiveConcurrency`` resizes the in-flight rollout cap from engine load
samples (KV-cache usage, running / waiting requests, preemptions), polled
every ``poll_interval_seconds``:
* hard signal (KV usage >= ``hard_kv_cache_usage``, a preemption, or a queue
  above ``queue_ratio`` x running for ``queue_persistence_polls`` polls):
  multiply the cap by ``preemption_decrease_factor`` (or the queue factor);
* soft signal (KV usage >= ``soft_kv_cache_usage`` or a queue seen on two
  consecutive polls): trim toward the ``target_kv_cache_usage`` share,
  at most once per ``kv_trim_cooldown_polls``;
* clear and binding (in-flight >= ``binding_fraction`` x cap) with KV usage
  below ``growth_kv_cache_usage`` for ``growth_gate_polls`` polls: grow by
  ``growth_factor_per_turnover``.
The cap stays within [min_inflight, max_inflight].

``AdmissionController`` enforces the cap (and an optional token-bucket rate
of request starts) for rollout workers; it is thread-safe and has an asyncio
variant for the HTTP client.
"""

from __future__ import annotations

import asyncio
import threading
import time
from dataclasses import dataclass


@dataclass
class EngineLoad:
    kv_cache_usage: float = 0.0
    running: int = 0
    waiting: int = 0
    preemptions_delta: int = 0


class AdaptiveConcurrency:
    def __init__(self, cfg, default_initial: int = 64):
        self.cfg = cfg
        init = cfg.initial_inflight or default_initial
        self.limit = float(self._clamp(init))
        self.signal = "clear"
        self._growth_polls = 0
        self._queue_polls = 0
        self._prev_waiting = 0
        self._trim_cooldown = 0
        self.decisions = {"grow": 0, "trim": 0, "shed": 0}

    def _clamp(self, v: float) -> float:
        lo = self.cfg.min_inflight
        hi = self.cfg.max_inflight if self.cfg.max_inflight is not None else float("inf")
        return max(lo, min(hi, v))

    @property
    def cap(self) -> int:
        return int(self.limit)

    def observe(self, s: EngineLoad, inflight: int) -> int:
        c = self.cfg
        queue_over = s.running > 0 and s.waiting > c.queue_ratio * s.running
        self._queue_polls = self._queue_polls + 1 if queue_over else 0
        persistent_queue = s.waiting > 0 and self._prev_waiting > 0
        self._prev_waiting = s.waiting
        self._trim_cooldown = max(0, self._trim_cooldown - 1)
        if s.preemptions_delta > 0 or s.kv_cache_usage >= c.hard_kv_cache_usage:
            self.signal = "hard"
            self.limit = self._clamp(self.limit * c.preemption_decrease_factor)
            self.decisions["shed"] += 1
            self._growth_polls = 0
        elif self._queue_polls >= c.queue_persistence_polls:
            self.signal = "hard"
            self.limit = self._clamp(self.limit * c.queue_decrease_factor)
            self.decisions["shed"] += 1
            self._growth_polls = 0
        elif s.kv_cache_usage >= c.soft_kv_cache_usage or persistent_queue:
            self.signal = "soft"
            self._growth_polls = 0
            if self._trim_cooldown == 0 and s.kv_cache_usage > 0:
                self.limit = self._clamp(min(self.limit, inflight * c.target_kv_cache_usage / s.kv_cache_usage))
                self._trim_cooldown = c.kv_trim_cooldown_polls
                self.decisions["trim"] += 1
        else:
            self.signal = "clear"
            binding = inflight >= c.binding_fraction * self.limit
            if binding and s.kv_cache_usage < c.growth_kv_cache_usage:
                self._growth_polls += 1
                if self._growth_polls >= c.growth_gate_polls:
                    self.limit = self._clamp(self.limit * c.growth_factor_per_turnover)
                    self.decisions["grow"] += 1
                    self._growth_polls = 0
            else:
                self._growth_polls = 0
        return self.cap

    def metrics(self) -> dict[str, float]:
        return {"concurrency/limit": float(self.cap), **{f"concurrency/{k}": float(v) for k, v in self.decisions.items()}}


class AdmissionController:
    """In-flight cap plus an optional token-bucket start rate (requests/s)."""

    def __init__(self, limit: int, rate: float | None = None, burst: int | None = None):
        self.limit = limit
        self.rate = rate
        self.burst = float(burst or max(1, limit))
        self.tokens = self.burst
        self.inflight = 0
        self._last = time.monotonic()
        self._cv = threading.Condition()

    def set_limit(self, limit: int) -> None:
        with self._cv:
            self.limit = max(1, int(limit))
            self._cv.notify_all()

    def _refill(self) -> None:
        if self.rate is None:
            return
        now = time.monotonic()
        self.tokens = min(self.burst, self.tokens + (now - self._last) * self.rate)
        self._last = now

    def acquire(self, cost: int = 1, timeout: float | None = None) -> bool:
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._cv:
            while True:
                self._refill()
                # a request larger than the cap (a jointly scored group) runs when nothing else does
                fits = self.inflight + cost <= self.limit or self.inflight == 0
                if fits and (self.rate is None or self.tokens >= 1.0):
                    self.inflight += cost
                    if self.rate is not None:
                        self.tokens -= 1.0
                    return True
                wait = 0.05 if self.rate is not None else None
                if deadline is not None:
                    left = deadline - time.monotonic()
                    if left <= 0:
                        return False
                    wait = left if wait is None else min(wait, left)
                self._cv.wait(wait)

    def release(self, cost: int = 1) -> None:
        with self._cv:
            self.inflight = max(0, self.inflight - cost)
            self._cv.notify_all()

    async def aacquire(self, cost: int = 1) -> None:
        while not self.acquire(cost, timeout=0):
            await asyncio.sleep(0.01)
