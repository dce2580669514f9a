"""Incremental columnar reader of a run's JSONL metric files.

Each file is tailed from its last byte offset (a live run only appends), rows
are split into numeric columns (NaN where a row lacks the key) plus step and
timestamp columns.  ``series`` returns a step window of chosen keys, reduced
to at most ``points`` points by per-bucket min/max (both extremes of every
bucket are kept so spikes survive downsampling).
"""

from __future__ import annotations

import json
import math
import os
from pathlib import Path
from typing import Any

import numpy as np


class MetricTable:
    def __init__(self, path: Path):
        self.path = Path(path)
        self.offset = 0
        self.steps: list[float] = []
        self.times: list[str | None] = []
        self.cols: dict[str, list[float]] = {}
        self.last: dict[str, Any] | None = None
        self.errors = 0

    def refresh(self) -> None:
        try:
            size = os.path.getsize(self.path)
        except OSError:
            return
        if size < self.offset:  # truncated / replaced: start over
            self.__init__(self.path)
        if size == self.offset:
            return
        with self.path.open("rb") as f:
            f.seek(self.offset)
            data = f.read()
        end = data.rfind(b"\n") + 1  # only whole lines
        self.offset += end
        for line in data[:end].splitlines():
            if not line.strip():
                continue
            try:
                row = json.loads(line)
            except json.JSONDecodeError:
                self.errors += 1
                continue
            self._append(row)

    def _append(self, row: dict[str, Any]) -> None:
        i = len(self.steps)
        s = row.get("step")
        self.steps.append(float(s) if isinstance(s, (int, float)) and not isinstance(s, bool) else math.nan)
        self.times.append(row.get("timestamp"))
        for k, v in row.items():
            if k in ("step", "timestamp") or isinstance(v, bool) or not isinstance(v, (int, float)):
                continue
            col = self.cols.get(k)
            if col is None:
                col = self.cols[k] = [math.nan] * i
            col.append(float(v))
        for col in self.cols.values():
            if len(col) < i + 1:
                col.append(math.nan)
        self.last = row

    def keys(self) -> list[str]:
        self.refresh()
        return sorted(self.cols)

    def series(self, keys: list[str], start: float | None = None, end: float | None = None,
               after: float | None = None, limit: int = 0, points: int = 0) -> dict[str, Any]:
        self.refresh()
        missing = [k for k in keys if k not in self.cols]
        if missing:
            raise KeyError(f"unknown metric keys: {missing}")
        steps = np.asarray(self.steps, dtype=np.float64)
        sel = np.ones(len(steps), dtype=bool)
        if start is not None:
            sel &= steps >= start
        if end is not None:
            sel &= steps <= end
        if after is not None:
            sel &= steps > after
        idx = np.nonzero(sel)[0]
        if limit:
            idx = idx[-limit:]
        if points and len(idx) > points:
            idx = _minmax_indices(idx, [np.asarray(self.cols[k]) for k in keys], points)
        out = {"steps": [None if math.isnan(x) else x for x in steps[idx].tolist()],
               "times": [self.times[i] for i in idx.tolist()], "series": {}}
        for k in keys:
            v = np.asarray(self.cols[k])[idx]
            out["series"][k] = [None if math.isnan(x) else x for x in v.tolist()]
        return out


def _minmax_indices(idx: np.ndarray, cols: list[np.ndarray], points: int) -> np.ndarray:
    buckets = max(1, points // 2)
    keep = set()
    for chunk in np.array_split(idx, buckets):
        if len(chunk) == 0:
            continue
        keep.add(int(chunk[0]))
        for c in cols:
            v = c[chunk]
            if np.all(np.isnan(v)):
                continue
            keep.add(int(chunk[int(np.nanargmin(v))]))
            keep.add(int(chunk[int(np.nanargmax(v))]))
    keep.add(int(idx[-1]))
    return np.asarray(sorted(keep), dtype=np.int64)


def read_jsonl(path: Path, limit: int = 0) -> list[dict[str, Any]]:
    if not Path(path).exists():
        return []
    rows = []
    for line in Path(path).read_text(encoding="utf-8", errors="replace").splitlines():
        if line.strip():
            try:
                rows.append(json.loads(line))
            except json.JSONDecodeError:
                continue
    return rows[-limit:] if limit else rows
