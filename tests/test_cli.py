"""CLI dispatch and the end-to-end CPU SFT run with checkpoint resume."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

from wavelet_b200.cli import COMMANDS, PUBLIC_COMMANDS, main

ROOT = Path(__file__).resolve().parents[1]


def test_commands_match_reference_surface():
    for c in ["rl", "sft", "debug", "evals", "convert-checkpoint", "convert-traces", "benchmark", "dashboard",
              "rl-trainer", "rl-orchestrator", "rl-inference", "inference-server"]:
        assert c in PUBLIC_COMMANDS
    for c in ["slurm-worker", "synth-run", "native-inference-server"]:
        assert c in COMMANDS


def test_unknown_command():
    assert main(["nope"]) == 1


@pytest.mark.integration
def test_sft_cpu_end_to_end_and_resume(tmp_path):
    cfg = tmp_path / "sft.yaml"
    out = tmp_path / "out"
    cfg.write_text(
        (ROOT / "examples" / "tiny_cpu" / "sft.yaml").read_text().replace("outputs/tiny_cpu_sft", str(out))
        + "ckpt:\n  mode: async\n  interval: 5\n"
    )
    env = {"WAVELET_FORCE_CPU": "1", "PATH": "/usr/bin:/bin"}
    import os

    env = {**os.environ, **env}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    rows = [json.loads(l) for l in (out / "metrics.jsonl").read_text().splitlines()]
    assert [r["step"] for r in rows] == list(range(1, 11))
    assert rows[-1]["loss"] < rows[0]["loss"]
    assert (out / "checkpoint-10" / "STABLE").exists()
    assert (out / "configs" / "latest" / "resolved" / "sft.yaml").exists()
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg), "--max-steps", "12",
                        "--ckpt.resume-step", "-1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    rows = [json.loads(l) for l in (out / "metrics.jsonl").read_text().splitlines()]
    assert [r["step"] for r in rows][-2:] == [11, 12]
    events = [json.loads(l)["event"] for l in (out / "events.jsonl").read_text().splitlines()]
    assert "run_resumed" in events


@pytest.mark.integration
def test_sft_cpu_validation_telemetry_profiler_lora(tmp_path):
    import os

    out = tmp_path / "out"
    base = (ROOT / "examples" / "tiny_cpu" / "sft.yaml").read_text().replace("outputs/tiny_cpu_sft", str(out))
    base = base.replace("lora: null\n", "").replace("max_steps: 10\n", "")
    cfg = tmp_path / "sft.yaml"
    cfg.write_text(base + """lora:
  rank: 4
  alpha: 8
val:
  interval: 2
  eval_on_start: true
  data:
    source: fake
    seq_len: 64
    batch_size: 4
    micro_batch_size: 2
    fake_vocab_size: 1024
    max_examples: 8
profiler:
  start_step: 2
  end_step: 3
gc:
  interval: 2
max_steps: 4
""")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(l) for l in (out / "metrics.jsonl").read_text().splitlines()]
    vals = [x for x in rows if "val/loss" in x]
    assert len(vals) >= 3 and all(v["val/loss"] > 0 for v in vals)  # start, step 2, step 4
    train = [x for x in rows if "loss" in x]
    assert any(k.startswith("node/") for k in train[-1])
    hb = json.loads((out / "heartbeat.json").read_text())
    assert hb.get("ranks") and hb["ranks"][0]["rank"] == 0
    assert (out / "traces" / "rank0.json").exists()
