"""``wavelet benchmark``: run a training command and aggregate its throughput,
or compare two results (reference tools/benchmark.py:41-300).

``run {sft,rl} CONFIG RUN_DIR OUTPUT``: runs ``wavelet <cmd> @ CONFIG`` with
``output_dir=RUN_DIR``, then reads ``metrics.jsonl``: the first
``--warmup-steps`` steps are dropped and the rest give the median / mean
tokens-per-second, step time and MFU.  With ``--baseline`` the result is
compared and the exit code is 2 on a regression beyond the threshold.
``compare CURRENT BASELINE`` prints the same comparison for two result files.
"""

from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import sys
import time
from pathlib import Path
from typing import Any

KEYS = {"tokens_per_second": ("perf/tokens_per_second", "higher"),
        "step_seconds": ("perf/step_seconds", "lower"),
        "mfu": ("perf/mfu", "higher")}


def aggregate(run_dir: Path, warmup_steps: int) -> dict[str, Any]:
    rows = [json.loads(l) for l in (Path(run_dir) / "metrics.jsonl").read_text().splitlines() if l.strip()]
    rows = [r for r in rows if r.get("step") is not None and r["step"] > warmup_steps and "loss" in r]
    if not rows:
        raise ValueError(f"no measured steps after {warmup_steps} warm-up steps in {run_dir}")
    out: dict[str, Any] = {"steps": len(rows), "warmup_steps": warmup_steps}
    for name, (key, _) in KEYS.items():
        vals = [float(r[key]) for r in rows if r.get(key) is not None]
        if vals:
            out[name] = {"median": statistics.median(vals), "mean": statistics.fmean(vals), "min": min(vals),
                         "max": max(vals)}
    out["final_loss"] = rows[-1].get("loss")
    return out


def compare(cur: dict, base: dict, threshold: float) -> tuple[list[str], bool]:
    lines, regressed = [], False
    for name, (_, better) in KEYS.items():
        if name not in cur or name not in base:
            continue
        c, b = cur[name]["median"], base[name]["median"]
        delta = (c - b) / b if b else 0.0
        bad = (delta < -threshold) if better == "higher" else (delta > threshold)
        regressed |= bad
        lines.append(f"{name:18s} current {c:12.4g}  baseline {b:12.4g}  {delta:+7.2%}{'  REGRESSION' if bad else ''}")
    return lines, regressed


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="wavelet benchmark", description=__doc__)
    sub = p.add_subparsers(dest="action", required=True)
    r = sub.add_parser("run")
    r.add_argument("command", choices=("sft", "rl"))
    r.add_argument("config", type=Path)
    r.add_argument("run_dir", type=Path)
    r.add_argument("output", type=Path)
    r.add_argument("--warmup-steps", type=int, default=1)
    r.add_argument("--timeout-seconds", type=float, default=3600)
    r.add_argument("--baseline", type=Path)
    r.add_argument("--regression-threshold", type=float, default=0.05)
    c = sub.add_parser("compare")
    c.add_argument("current", type=Path)
    c.add_argument("baseline", type=Path)
    c.add_argument("--regression-threshold", type=float, default=0.05)
    a = p.parse_args(sys.argv[1:] if argv is None else argv)
    if a.action == "compare":
        lines, bad = compare(json.loads(a.current.read_text()), json.loads(a.baseline.read_text()),
                             a.regression_threshold)
        print("\n".join(lines))
        return 2 if bad else 0
    t0 = time.time()
    cmd = [sys.executable, "-m", "wavelet_b200", a.command, "@", str(a.config), "--output-dir", str(a.run_dir),
           "--clean-output-dir"]
    proc = subprocess.run(cmd, timeout=a.timeout_seconds)
    if proc.returncode != 0:
        print(f"benchmark command failed with exit code {proc.returncode}", file=sys.stderr)
        return proc.returncode
    res = {"command": a.command, "config": str(a.config), "wall_seconds": time.time() - t0,
           **aggregate(a.run_dir, a.warmup_steps)}
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(res, indent=2))
    print(json.dumps(res, indent=2))
    if a.baseline:
        lines, bad = compare(res, json.loads(a.baseline.read_text()), a.regression_threshold)
        print("\n".join(lines))
        return 2 if bad else 0
    return 0


if __name__ == "__main__":
    sys.exit(main())
