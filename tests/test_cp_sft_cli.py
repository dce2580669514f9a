"""`wavelet sft` with context parallelism on 2 gloo CPU ranks (one data-
parallel replica split over cp = 2) against the same run on one process: the
per-step losses agree (the CP run computes the same token-mean loss from its
two sequence shards)."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _cfg(tmp: Path, name: str, cp: int) -> Path:
    out = tmp / name
    text = (ROOT / "examples" / "tiny_cpu" / "sft.yaml").read_text().replace("outputs/tiny_cpu_sft", str(out))
    text = text.replace("max_steps: 10", "max_steps: 3").replace("micro_batch_size: 4", "micro_batch_size: 8")
    text = text.replace("model:\n  name: tiny\n", "model:\n  name: tiny\n  attn_implementation: sdpa\n")
    text = text.replace("fsdp:\n  backend: gloo\n", f"fsdp:\n  backend: gloo\n  enabled: true\n  impl: fsdp2\n  cp: {cp}\n")
    p = tmp / f"{name}.yaml"
    p.write_text(text)
    return p


def _losses(out: Path) -> list[float]:
    return [json.loads(line)["loss"] for line in (out / "metrics.jsonl").read_text().splitlines()]


def _tokens(out: Path) -> list[float]:
    return [json.loads(line)["train/loss_tokens"] for line in (out / "metrics.jsonl").read_text().splitlines()]


@pytest.mark.integration
def test_cp2_sft_matches_single_process(tmp_path):
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    single = _cfg(tmp_path, "single", 1)
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(single)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cp = _cfg(tmp_path, "cp", 2)
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "wavelet_b200", "sft", "@",
                        str(cp)], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    a, b = _losses(tmp_path / "single"), _losses(tmp_path / "cp")
    assert len(a) == len(b) == 3
    for x, y in zip(a, b):
        assert abs(x - y) <= 1e-3 * abs(x), (a, b)
    # the CP ranks each count half of every sequence's loss tokens (not all of them twice)
    assert _tokens(tmp_path / "cp") == _tokens(tmp_path / "single")
