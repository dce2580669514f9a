"""Resumable evaluation results (``eval.resume``; ref orchestrator/eval_utils.py:39-200).

An evaluation of one environment at one policy step keeps a journal
directory next to its rollout file:

    manifest.json          {"format_version": 1, "signature": <sha256 of the settings>}
    episode-<sha256>.json  one committed result per episode key
    timing.json            seconds spent so far, summed over attempts
    writer.lock            an exclusive lock held by the one writer

Every file is written to a temporary name, flushed to disk and renamed, so a
killed run leaves either a whole record or none.  A rerun with
``eval.resume: true`` and the same settings (environment, arguments, model,
sampling plan, policy step) reuses every committed episode that has a reward
and reruns the rest; different settings are an error, and so is an existing
journal with ``eval.resume: false``.  Episode keys identify an example by the
hash of its content, so duplicates stay distinct by occurrence.
"""

from __future__ import annotations

import fcntl
import hashlib
import json
import math
import os
import time
from pathlib import Path
from typing import Any


def _default(v: Any) -> Any:
    dump = getattr(v, "model_dump", None)
    if callable(dump):
        return dump(mode="json", exclude_none=True)
    if isinstance(v, (Path, BaseException)):
        return str(v)
    tolist = getattr(v, "tolist", None)
    if callable(tolist):
        return tolist()
    raise TypeError(f"cannot store {type(v).__name__} in an evaluation journal")


def canonical(value: Any) -> str:
    return json.dumps(value, sort_keys=True, default=_default, allow_nan=False, separators=(",", ":"))


def signature(**settings: Any) -> str:
    """Hash of everything that decides an evaluation's results."""
    return hashlib.sha256(canonical(settings).encode()).hexdigest()


def _write_atomic(path: Path, value: Any) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    with tmp.open("w", encoding="utf-8") as f:
        f.write(canonical(value))
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)
    fd = os.open(path.parent, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def episode_keys(examples: list[dict[str, Any]], samples: int) -> list[str]:
    """One key per (example, sample): the example's content hash, its
    occurrence among identical examples, and the sample index."""
    seen: dict[str, int] = {}
    keys = []
    for i, ex in enumerate(examples):
        ident = dict(ex)
        ident.setdefault("example_id", ident.get("id", i))
        h = signature(example=ident)
        occ = seen.get(h, 0)
        seen[h] = occ + 1
        keys += [f"{h}:{occ}:{k}" for k in range(samples)]
    return keys


class EvalJournal:
    FORMAT = 1

    def __init__(self, path: Path, *, sig: str, resume: bool):
        self.path = Path(path)
        self.sig = sig
        self.resume = resume
        self.rows: dict[str, dict[str, Any]] = {}
        self._lock = None
        self._t0 = 0.0
        self._before = 0.0
        self.elapsed_seconds = 0.0

    @staticmethod
    def _name(key: str) -> str:
        return "episode-" + hashlib.sha256(key.encode()).hexdigest() + ".json"

    def __enter__(self) -> "EvalJournal":
        self.path.mkdir(parents=True, exist_ok=True)
        self._lock = (self.path / "writer.lock").open("a")
        try:
            fcntl.flock(self._lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
            man = self.path / "manifest.json"
            want = {"format_version": self.FORMAT, "signature": self.sig}
            if man.exists():
                if not self.resume:
                    raise FileExistsError(f"an evaluation journal exists at {self.path}; set eval.resume: true "
                                          "to continue it or use a new output directory")
                if json.loads(man.read_text()) != want:
                    raise ValueError(f"the evaluation settings differ from the journal at {self.path}")
            else:
                _write_atomic(man, want)
            timing = self.path / "timing.json"
            if timing.exists():
                self._before = float(json.loads(timing.read_text())["seconds"])
                if not math.isfinite(self._before) or self._before < 0:
                    raise ValueError(f"invalid timing in the evaluation journal at {self.path}")
            for f in self.path.glob("episode-*.json"):
                rec = json.loads(f.read_text(encoding="utf-8"))
                if not isinstance(rec, dict) or not isinstance(rec.get("key"), str) \
                        or not isinstance(rec.get("output"), dict):
                    raise ValueError(f"malformed evaluation journal record {f}")
                if f.name != self._name(rec["key"]):
                    raise ValueError(f"evaluation journal record {f} does not match its key")
                self.rows[rec["key"]] = rec["output"]
            self._t0 = time.monotonic()
        except BaseException:
            self._lock.close()
            self._lock = None
            raise
        return self

    def __exit__(self, *exc) -> None:
        if self._lock is not None:
            try:
                self._save_timing()
            finally:
                self._lock.close()
                self._lock = None

    def completed(self, key: str) -> dict[str, Any] | None:
        """A committed result that has a reward (failed episodes are rerun)."""
        row = self.rows.get(key)
        if row is None or row.get("error") is not None or "reward" not in row:
            return None
        return dict(row)

    def record(self, key: str, output: dict[str, Any]) -> dict[str, Any]:
        if self._lock is None:
            raise RuntimeError("open the evaluation journal with `with` before recording")
        out = json.loads(canonical(output))
        _write_atomic(self.path / self._name(key), {"key": key, "output": out})
        self.rows[key] = out
        self._save_timing()
        return dict(out)

    def _save_timing(self) -> None:
        self.elapsed_seconds = self._before + time.monotonic() - self._t0
        _write_atomic(self.path / "timing.json", {"seconds": self.elapsed_seconds})
