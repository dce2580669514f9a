"""`wavelet sft` with tensor parallelism on 2 gloo CPU ranks against the same
run on one process: per-step losses agree."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _cfg(tmp: Path, name: str, tp: int) -> Path:
    out = tmp / name
    text = (ROOT / "examples" / "tiny_cpu" / "sft.yaml").read_text().replace("outputs/tiny_cpu_sft", str(out))
    text = text.replace("max_steps: 10", "max_steps: 3").replace("micro_batch_size: 4", "micro_batch_size: 8")
    text = text.replace("fsdp:\n  backend: gloo\n", f"fsdp:\n  backend: gloo\n  tp: {tp}\n")
    p = tmp / f"{name}.yaml"
    p.write_text(text)
    return p


def _losses(out: Path) -> list[float]:
    return [json.loads(line)["loss"] for line in (out / "metrics.jsonl").read_text().splitlines()]


@pytest.mark.integration
def test_tp2_sft_matches_single_process(tmp_path):
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(_cfg(tmp_path, "single", 1))], cwd=ROOT,
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "wavelet_b200", "sft", "@",
                        str(_cfg(tmp_path, "tp", 2))], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    a, b = _losses(tmp_path / "single"), _losses(tmp_path / "tp")
    assert len(a) == len(b) == 3
    for x, y in zip(a, b):
        assert abs(x - y) <= 1e-3 * abs(x), (a, b)
