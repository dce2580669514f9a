"""The split RL placement on 2 B200s: the rl-trainer on GPU 0 and one
inference server on GPU 1 (launcher.mode process), with device policy
transfer: each update is pushed into the server's receive slots over peer
memory (update protocol peer_v1) and loaded between generation batches."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_split_placement_with_peer_policy_push(tmp_path):
    cfg = tmp_path / "rl.yaml"
    cfg.write_text(f"""model:
  name: tiny-gpu
  random_init: true
data:
  source: fake
  seq_len: 256
  fake_vocab_size: 64
  fake_prompt_len: 8
algo:
  type: grpo
reward:
  mode: reverse_match
orchestrator:
  examples_per_step: 4
  rollouts_per_example: 4
inference:
  sampling:
    max_completion_tokens: 16
  http:
    port: {_free()}
    startup_timeout_seconds: 300
transport:
  poll_interval_seconds: 0.2
  idle_timeout_seconds: 300
policy_transfer:
  type: nccl
  nccl_port: {_free()}
  nccl_timeout_seconds: 300
  poll_interval_seconds: 0.2
  idle_timeout_seconds: 300
launcher:
  mode: process
  poll_interval_seconds: 0.5
  trainer_cuda_visible_devices: "0"
  inference_cuda_visible_devices: "1"
lora: null
max_steps: 3
output_dir: {tmp_path / 'out'}
""")
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "rl", "@", str(cfg)], cwd=root, env=dict(os.environ),
                       capture_output=True, text=True, timeout=900)
    logs = ""
    for p in (tmp_path / "out" / "logs").rglob("*.log"):
        logs += p.name + ":\n" + p.read_text()[-1500:]
    assert r.returncode == 0, (r.stderr[-2000:], logs)
    rows = [json.loads(line) for line in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2, 3]
    info = json.loads((tmp_path / "out" / "policies" / "step-000003" / "update_info.json").read_text())
    assert info["protocol"] == "peer_v1" and info["receivers"] == 1
