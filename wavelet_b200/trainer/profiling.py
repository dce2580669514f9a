"""Step-range profiling.

* ``StepProfiler`` — a ``torch.profiler`` Chrome trace (CPU + CUPTI kernel
  activity, so the sm_100a kernels of this package appear by name) over an
  inclusive optimizer-step range (reference trainer/profiling.py:53-97).
* ``CudaMemoryProfiler`` — caching-allocator history with a rank-local
  snapshot every ``interval`` steps (reference trainer/profiling.py:12-50).
  Buffers allocated outside the caching allocator (the peer fabric) are not
  in these snapshots; ``fabric_bytes`` in the step metrics covers them.
* ``PhaseTimer`` — CUDA-event timing of named phases (forward/backward,
  optimizer) on the launching stream, read once per step.
"""

from __future__ import annotations

import logging
import pickle
from pathlib import Path

import torch

log = logging.getLogger("wavelet")


class StepProfiler:
    def __init__(self, trace_path: Path, *, start_step: int, end_step: int, record_shapes: bool = True,
                 profile_memory: bool = True):
        self.trace_path = Path(trace_path)
        self.start_step, self.end_step = start_step, end_step
        self.record_shapes, self.profile_memory = record_shapes, profile_memory
        self._prof = None
        self._done = False

    def before_step(self, step: int) -> None:
        if self._done or self._prof is not None or not (self.start_step <= step <= self.end_step):
            return
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self.trace_path.parent.mkdir(parents=True, exist_ok=True)
        self._prof = torch.profiler.profile(activities=acts, record_shapes=self.record_shapes,
                                            profile_memory=self.profile_memory)
        self._prof.__enter__()

    def after_step(self, step: int) -> None:
        if self._prof is not None and step >= self.end_step:
            self.close()

    def close(self) -> None:
        if self._done:
            return
        self._done = True
        if self._prof is not None:
            self._prof.__exit__(None, None, None)
            self._prof.export_chrome_trace(str(self.trace_path))
            log.info("wrote profiler trace %s", self.trace_path)
            self._prof = None


class CudaMemoryProfiler:
    def __init__(self, output_dir: Path, *, rank: int, interval: int, max_entries: int):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA memory profiling needs a CUDA device")
        self.output_dir = Path(output_dir)
        self.rank, self.interval = rank, interval
        self._closed = False
        torch.cuda.memory._record_memory_history(max_entries=max_entries)

    def step(self, step: int) -> Path | None:
        if self._closed or step <= 0 or step % self.interval:
            return None
        d = self.output_dir / f"step-{step}"
        d.mkdir(parents=True, exist_ok=True)
        path = d / f"rank-{self.rank}.pickle"
        with path.open("wb") as f:
            pickle.dump(torch.cuda.memory._snapshot(), f)
        return path

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            torch.cuda.memory._record_memory_history(enabled=None)


class PhaseTimer:
    """Accumulates CUDA-event time of named phases; ``read()`` syncs once."""

    def __init__(self, enabled: bool):
        self.enabled = enabled and torch.cuda.is_available()
        self._open: dict[str, torch.cuda.Event] = {}
        self._pairs: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def start(self, name: str) -> None:
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open[name] = e

    def stop(self, name: str) -> None:
        if self.enabled and name in self._open:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._pairs.append((name, self._open.pop(name), e))

    def read(self) -> dict[str, float]:
        if not self._pairs:
            return {}
        self._pairs[-1][2].synchronize()
        out: dict[str, float] = {}
        for name, a, b in self._pairs:
            out[f"time/{name}_ms"] = out.get(f"time/{name}_ms", 0.0) + a.elapsed_time(b)
        self._pairs.clear()
        return out
