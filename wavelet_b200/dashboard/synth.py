"""``wavelet synth-run``: write a synthetic run directory (trainer and
orchestrator metrics, heartbeat with a rank table, events, rollout queue
batches, policy snapshots, evals, logs) for dashboard development and tests
(reference dashboard/synth.py:54-836).  Deterministic for a given seed."""

from __future__ import annotations

import argparse
import json
import math
import random
import sys
from datetime import datetime, timedelta, timezone
from pathlib import Path


def _ts(t0: datetime, s: float) -> str:
    return (t0 + timedelta(seconds=s)).isoformat()


def _jsonl(path: Path, rows: list[dict]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")


def write_synthetic_run(out: Path, steps: int = 50, ranks: int = 8, seed: int = 0) -> Path:
    rng = random.Random(seed)
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    t0 = datetime(2026, 1, 1, tzinfo=timezone.utc)
    (out / "run_metadata.json").write_text(json.dumps({"command": "rl", "started_at": t0.isoformat(),
                                                       "world_size": ranks, "synthetic": True}))
    cfg = out / "configs" / "attempt_1" / "resolved"
    cfg.mkdir(parents=True, exist_ok=True)
    (cfg / "rl.yaml").write_text("model:\n  name: synthetic\nmax_steps: %d\n" % steps)
    latest = out / "configs" / "latest"
    if not latest.exists():
        latest.symlink_to("attempt_1", target_is_directory=True)
    events = [{"timestamp": _ts(t0, 0), "event": "run_started", "step": 0, "payload": {}}]
    for s in range(1, steps + 1):
        t = 10.0 * s
        loss = 2.5 * math.exp(-s / 30) + 0.3 + 0.05 * rng.random()
        reward = 1 - math.exp(-s / 25) + 0.05 * rng.random()
        _jsonl(out / "metrics.jsonl", [{"step": s, "timestamp": _ts(t0, t), "loss": loss,
                                        "optim/grad_norm": 0.5 + rng.random(), "optim/lr": 1e-5,
                                        "perf/tokens_per_second": 2.0e5 * (0.95 + 0.1 * rng.random()),
                                        "perf/mfu": 40.0 + 2.0 * rng.random(),
                                        "node/synthetic/tokens_per_second": 2.0e5}])
        _jsonl(out / "orchestrator_metrics.jsonl", [{"step": s - 1, "timestamp": _ts(t0, t - 5), "reward/mean": reward,
                                                     "rollout/tokens_per_second": 5e4 * (0.9 + 0.2 * rng.random()),
                                                     "policy_lag": 1}])
        q = out / "rollouts" / f"step-{s - 1:06d}"
        q.mkdir(parents=True, exist_ok=True)
        rows = [{"prompt": [{"role": "user", "content": f"task {s}-{i}"}],
                 "completion": [{"role": "assistant", "content": "answer"}], "reward": reward, "advantage": 0.0}
                for i in range(4)]
        _jsonl(q / "rollouts.jsonl", rows)
        (q / "manifest.json").write_text(json.dumps({"step": s - 1, "rows": len(rows)}))
        (q / "STABLE").touch()
        (q / "consumed.json").write_text(json.dumps({"step": s - 1}))
        if s % 5 == 0:
            p = out / "policies" / f"step-{s:06d}"
            p.mkdir(parents=True, exist_ok=True)
            (p / "policy.json").write_text(json.dumps({"step": s, "kind": "model"}))
            (p / "STABLE").touch()
            events.append({"timestamp": _ts(t0, t), "event": "policy_exported", "step": s, "payload": {}})
        if s % 10 == 0:
            _jsonl(out / "eval_metrics.jsonl", [{"step": s, "timestamp": _ts(t0, t), "eval/reverse/pass@1": reward}])
    events.append({"timestamp": _ts(t0, 10.0 * steps), "event": "run_finished", "step": steps,
                   "payload": {"status": "completed"}})
    _jsonl(out / "events.jsonl", events)
    (out / "heartbeat.json").write_text(json.dumps({
        "timestamp": _ts(t0, 10.0 * steps), "status": "completed", "step": steps,
        "ranks": [{"rank": r, "local_rank": r, "node": "synthetic", "device": f"cuda:{r}", "tokens": 1.0e6,
                   "seconds": 10.0, "tokens_per_second": 1.0e5, "memory_allocated_gib": 60.0,
                   "peak_memory_gib": 80.0} for r in range(ranks)]}))
    logs = out / "logs" / "attempt_1"
    logs.mkdir(parents=True, exist_ok=True)
    (logs / "trainer.log").write_text("".join(f"step {s} loss ok\n" for s in range(1, steps + 1)))
    if not (out / "logs" / "latest").exists():
        (out / "logs" / "latest").symlink_to("attempt_1", target_is_directory=True)
    return out


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="wavelet synth-run", description=__doc__)
    p.add_argument("output_dir", type=Path)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--ranks", type=int, default=8)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(sys.argv[1:] if argv is None else argv)
    print(write_synthetic_run(a.output_dir, a.steps, a.ranks, a.seed))
    return 0


if __name__ == "__main__":
    sys.exit(main())
