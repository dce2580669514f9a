"""Durable filesystem rollout and policy queues.

Layout (same names as the reference, transport/queue.py:24-31):

    <queue_dir>/step-XXXXXX/rollouts.jsonl                human-readable rows
    <queue_dir>/step-XXXXXX/rollouts.jsonl.train.msgpack  trainer payload (array of records)
    <queue_dir>/step-XXXXXX/manifest.json                 producer metadata
    <queue_dir>/step-XXXXXX/claim.json                    written when a trainer claims it
    <queue_dir>/step-XXXXXX/consumed.json                 written after the optimizer step
    <queue_dir>/step-XXXXXX/STABLE                        publication is complete
    <output_dir>/events/queue.jsonl                       lifecycle events
    <policy_dir>/step-XXXXXX/{policy.json, STABLE, ...}   policy snapshots

Writers stage files under ``*.tmp`` names and rename; ``STABLE`` is touched
last, so readers only ever see complete batches.  Receivers poll with an
optional idle timeout.
"""

from __future__ import annotations

import json
import os
import shutil
import socket
import time
from dataclasses import asdict, dataclass, field
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, Callable, Iterable

import msgpack

STEP_PREFIX = "step-"
STABLE = "STABLE"
MANIFEST = "manifest.json"
CLAIM = "claim.json"
CONSUMED = "consumed.json"
POLICY_META = "policy.json"
EVENTS_FILE = "queue.jsonl"
TRAIN_SUFFIX = ".train.msgpack"


def utc_now() -> str:
    return datetime.now(timezone.utc).isoformat()


def process_identity(role: str) -> str:
    return f"{role}@{socket.gethostname()}:{os.getpid()}"


def step_dir(root: Path, step: int) -> Path:
    return Path(root) / f"{STEP_PREFIX}{step:06d}"


def parse_step(p: Path) -> int | None:
    if not p.is_dir() or not p.name.startswith(STEP_PREFIX):
        return None
    try:
        return int(p.name[len(STEP_PREFIX):])
    except ValueError:
        return None


def stable_steps(root: Path) -> list[int]:
    root = Path(root)
    if not root.exists():
        return []
    return sorted(s for p in root.iterdir() if (s := parse_step(p)) is not None and (p / STABLE).exists())


def resolve_queue_dir(output_dir: Path, cfg) -> Path:
    return Path(cfg.queue_dir) if cfg.queue_dir is not None else Path(output_dir) / "rollouts"


def resolve_policy_dir(output_dir: Path, cfg) -> Path:
    return Path(cfg.policy_dir) if cfg.policy_dir is not None else Path(output_dir) / "policies"


def _write_json(path: Path, obj: Any) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(obj, indent=2, default=str))
    os.replace(tmp, path)


def _read_json(path: Path) -> dict | None:
    try:
        return json.loads(path.read_text())
    except (FileNotFoundError, json.JSONDecodeError):
        return None


def append_event(events_dir: Path, kind: str, **fields) -> None:
    try:
        events_dir.mkdir(parents=True, exist_ok=True)
        with (events_dir / EVENTS_FILE).open("a") as f:
            f.write(json.dumps({"time": utc_now(), "kind": kind, **{k: v for k, v in fields.items() if v is not None}}) + "\n")
    except OSError:
        pass


def _poll(find: Callable[[], Any], interval: float, timeout: float | None, what: str):
    t0 = time.monotonic()
    while (item := find()) is None:
        if timeout is not None and time.monotonic() - t0 >= timeout:
            raise TimeoutError(f"timed out after {timeout}s waiting for {what}")
        time.sleep(interval)
    return item, time.monotonic() - t0


# --------------------------------------------------------------- records
@dataclass
class RolloutManifest:
    format_version: int
    queue_step: int
    optimizer_step: int | None = None
    chunk_index: int | None = None
    policy_step: int | None = None
    rows: int | None = None
    tokens: int | None = None
    reward_mean: float | None = None
    producer_id: str | None = None
    created_at: str = ""
    payload_bytes: int | None = None
    transfer_seconds: float | None = None
    environment_record_cursors: dict[str, list[int]] | None = None
    environment_next_record_cursors: dict[str, int] | None = None
    environment_selection_cursor: int | None = None
    curriculum_state: dict[str, dict[str, Any]] | None = None
    prompt_source_state: dict[str, Any] | None = None  # prompt source right after this step's draw (resume)


@dataclass
class RolloutBatch:
    step: int
    path: Path
    step_dir: Path

    @property
    def training_path(self) -> Path:
        b = self.path.with_name(self.path.name + TRAIN_SUFFIX)
        return b if b.is_file() else self.path

    @property
    def manifest(self) -> RolloutManifest | None:
        d = _read_json(self.step_dir / MANIFEST)
        return RolloutManifest(**d) if d else None


def read_training_records(path: Path) -> list[dict[str, Any]]:
    if path.name.endswith(TRAIN_SUFFIX):
        with path.open("rb") as f:
            return msgpack.unpackb(f.read(), raw=False, strict_map_key=False)
    return [json.loads(l) for l in path.read_text().splitlines() if l.strip()]


# ----------------------------------------------------------------- sender
class FileSystemRolloutSender:
    def __init__(self, output_dir: Path, cfg):
        self.cfg = cfg
        self.output_dir = Path(output_dir)
        self.queue_dir = resolve_queue_dir(output_dir, cfg)

    def stable_batch(self, step: int) -> RolloutBatch | None:
        d = step_dir(self.queue_dir, step)
        p = d / self.cfg.rollout_filename
        return RolloutBatch(step, p, d) if (d / STABLE).exists() and p.is_file() else None

    def publish(self, rows: list[dict[str, Any]], *, step: int, training_records: list[dict[str, Any]] | None = None,
                optimizer_step: int | None = None, chunk_index: int | None = None, policy_step: int | None = None,
                tokens: int | None = None, reward_mean: float | None = None, producer_id: str | None = None,
                **cursor_fields) -> RolloutBatch:
        if self.stable_batch(step) is not None:
            raise FileExistsError(f"rollout queue step {step} is already stable and cannot be overwritten")
        d = step_dir(self.queue_dir, step)
        d.mkdir(parents=True, exist_ok=True)
        t0 = time.perf_counter()
        target = d / self.cfg.rollout_filename
        tmp = d / (self.cfg.rollout_filename + ".tmp")
        with tmp.open("w") as f:
            for r in rows:
                f.write(json.dumps(r, default=str) + "\n")
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, target)
        nbytes = target.stat().st_size
        train_path = target.with_name(target.name + TRAIN_SUFFIX)
        if training_records is not None:
            ttmp = train_path.with_suffix(".tmp")
            try:
                with ttmp.open("wb") as f:
                    packer = msgpack.Packer(use_bin_type=True)
                    f.write(packer.pack_array_header(len(training_records)))
                    for rec in training_records:
                        f.write(packer.pack(rec))
                os.replace(ttmp, train_path)
            except OverflowError:
                ttmp.unlink(missing_ok=True)
                train_path.unlink(missing_ok=True)
        else:
            train_path.unlink(missing_ok=True)
        pid = producer_id or process_identity("rl-inference")
        man = RolloutManifest(format_version=1, queue_step=step, optimizer_step=optimizer_step, chunk_index=chunk_index,
                              policy_step=policy_step, rows=len(rows), tokens=tokens, reward_mean=reward_mean,
                              producer_id=pid, created_at=utc_now(), payload_bytes=nbytes,
                              transfer_seconds=time.perf_counter() - t0, **cursor_fields)
        _write_json(d / MANIFEST, asdict(man))
        append_event(self.output_dir / "events", "rollout_published", queue_step=step, optimizer_step=optimizer_step,
                     policy_step=policy_step, producer_id=pid, details={"payload_bytes": nbytes})
        (d / STABLE).touch()
        return RolloutBatch(step, target, d)


# --------------------------------------------------------------- receiver
class FileSystemRolloutReceiver:
    def __init__(self, output_dir: Path, cfg, *, start_step: int = 0, consumer_id: str | None = None):
        self.cfg = cfg
        self.output_dir = Path(output_dir)
        self.queue_dir = resolve_queue_dir(output_dir, cfg)
        self.next_step = start_step
        self.consumer_id = consumer_id or process_identity("rl-trainer")
        self._floor = start_step  # batches below the resume point are never taken
        self._received: set[int] = set()

    def _batch(self, step: int) -> RolloutBatch | None:
        d = step_dir(self.queue_dir, step)
        p = d / self.cfg.rollout_filename
        return RolloutBatch(step, p, d) if (d / STABLE).exists() and p.is_file() else None

    def wait(self) -> RolloutBatch:
        """Block until the batch for ``next_step`` is stable."""
        b, waited = _poll(lambda: self._batch(self.next_step), self.cfg.poll_interval_seconds,
                          self.cfg.idle_timeout_seconds, f"rollout step {self.next_step}")
        append_event(self.output_dir / "events", "rollout_received", queue_step=b.step, consumer_id=self.consumer_id,
                     details={"wait_seconds": waited, "mode": "exact"})
        self._received.add(b.step)
        self.next_step += 1
        return b

    def wait_available(self) -> RolloutBatch:
        """Block until a stable batch this receiver has not taken (and nobody
        consumed) exists, then take the oldest: a step published late, below
        ``next_step``, is still picked up; ``next_step`` never moves back."""
        def find():
            for s in stable_steps(self.queue_dir):
                if (s >= self._floor and s not in self._received
                        and not (step_dir(self.queue_dir, s) / CONSUMED).exists()):
                    return self._batch(s)
            return None

        b, waited = _poll(find, self.cfg.poll_interval_seconds, self.cfg.idle_timeout_seconds, "any rollout batch")
        append_event(self.output_dir / "events", "rollout_received", queue_step=b.step, consumer_id=self.consumer_id,
                     details={"wait_seconds": waited, "mode": "available"})
        self._received.add(b.step)
        self.next_step = max(self.next_step, b.step + 1)
        return b

    def claim(self, b: RolloutBatch, trainer_step: int) -> None:
        _write_json(b.step_dir / CLAIM, {"format_version": 1, "queue_step": b.step, "consumer_id": self.consumer_id,
                                         "trainer_step_before": trainer_step, "claimed_at": utc_now()})
        append_event(self.output_dir / "events", "rollout_claimed", queue_step=b.step, consumer_id=self.consumer_id)

    def consumed(self, b: RolloutBatch, before: int, after: int, stepped: bool = True) -> None:
        _write_json(b.step_dir / CONSUMED, {"format_version": 1, "queue_step": b.step, "consumer_id": self.consumer_id,
                                            "trainer_step_before": before, "trainer_step_after": after,
                                            "optimizer_step_completed": stepped, "consumed_at": utc_now()})
        append_event(self.output_dir / "events", "rollout_consumed", queue_step=b.step, consumer_id=self.consumer_id,
                     optimizer_step=after)
        if self.cfg.cleanup_consumed:
            prune_consumed(self.queue_dir, keep_last=self.cfg.keep_last_consumed)


def prune_consumed(queue_dir: Path, keep_last: int) -> list[int]:
    done = [s for s in stable_steps(queue_dir) if (step_dir(queue_dir, s) / CONSUMED).exists()]
    removed = done[:-keep_last] if keep_last > 0 else done
    for s in removed:
        shutil.rmtree(step_dir(queue_dir, s), ignore_errors=True)
    return removed


def prune_from(queue_dir: Path, first_step: int) -> list[int]:
    """Drop every batch >= first_step (resume discards batches past a checkpoint)."""
    root = Path(queue_dir)
    removed = []
    if root.exists():
        for p in root.iterdir():
            s = parse_step(p)
            if s is not None and s >= first_step:
                shutil.rmtree(p, ignore_errors=True)
                removed.append(s)
    return sorted(removed)


# ----------------------------------------------------------------- policies
@dataclass
class PolicySnapshot:
    step: int
    step_dir: Path

    @property
    def meta(self) -> dict[str, Any]:
        return _read_json(self.step_dir / POLICY_META) or {}


class FileSystemPolicyReceiver:
    def __init__(self, output_dir: Path, cfg, *, start_step: int = 0):
        self.cfg = cfg
        self.output_dir = Path(output_dir)
        self.policy_dir = resolve_policy_dir(output_dir, cfg)
        self.next_step = start_step

    def _snap(self, step: int) -> PolicySnapshot | None:
        d = step_dir(self.policy_dir, step)
        return PolicySnapshot(step, d) if (d / STABLE).exists() else None

    def latest(self) -> PolicySnapshot | None:
        s = stable_steps(self.policy_dir)
        return self._snap(s[-1]) if s else None

    def wait_for_step(self, step: int) -> PolicySnapshot:
        snap, _ = _poll(lambda: self._snap(step) or (self.latest() if (self.latest() and self.latest().step >= step) else None),
                        self.cfg.poll_interval_seconds, self.cfg.idle_timeout_seconds, f"policy step {step}")
        self.next_step = snap.step + 1
        return snap

    def wait(self) -> PolicySnapshot:
        return self.wait_for_step(self.next_step)


def policy_lag(trainer_step: int, policy_step: int | None) -> int | None:
    return None if policy_step is None else trainer_step - policy_step


def scan_queue(queue_dir: Path) -> dict[str, Any]:
    """Status of every queue item (for debug/dashboards)."""
    root = Path(queue_dir)
    items = []
    if root.exists():
        for p in sorted(root.iterdir()):
            s = parse_step(p)
            if s is None:
                continue
            status = "consumed" if (p / CONSUMED).exists() else "claimed" if (p / CLAIM).exists() else "stable" if (p / STABLE).exists() else "writing"
            items.append({"queue_step": s, "status": status, "manifest": _read_json(p / MANIFEST)})
    counts: dict[str, int] = {}
    for it in items:
        counts[it["status"]] = counts.get(it["status"], 0) + 1
    return {"queue_dir": str(root), "items": items, "counts": counts}
