"""`wavelet sft` with sharded parameters (fsdp.shard_params, ZeRO-3) on 2
gloo CPU ranks against the same data-parallel run with replicated weights:
per-step losses agree, and a checkpoint is written from the shards."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _cfg(tmp: Path, name: str, shard: bool) -> Path:
    out = tmp / name
    text = (ROOT / "examples" / "tiny_cpu" / "sft.yaml").read_text().replace("outputs/tiny_cpu_sft", str(out))
    text = text.replace("max_steps: 10", "max_steps: 3")
    text = text.replace("fsdp:\n  backend: gloo\n", f"fsdp:\n  backend: gloo\n  shard_params: {str(shard).lower()}\n")
    text += "ckpt:\n  mode: async\n  interval: 3\n"
    p = tmp / f"{name}.yaml"
    p.write_text(text)
    return p


def _run(cfg: Path) -> None:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "wavelet_b200", "sft", "@",
                        str(cfg)], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]


def _losses(out: Path) -> list[float]:
    return [json.loads(line)["loss"] for line in (out / "metrics.jsonl").read_text().splitlines()]


@pytest.mark.integration
def test_zero3_sft_matches_replicated_weights(tmp_path):
    _run(_cfg(tmp_path, "rep", False))
    _run(_cfg(tmp_path, "z3", True))
    a, b = _losses(tmp_path / "rep"), _losses(tmp_path / "z3")
    assert len(a) == len(b) == 3
    for x, y in zip(a, b):
        assert abs(x - y) <= 1e-4 * abs(x), (a, b)
    assert (tmp_path / "z3" / "checkpoint-3" / "trainer" / "model.safetensors").exists()


def _run4(cfg: Path) -> None:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "4",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "wavelet_b200", "sft", "@",
                        str(cfg)], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]


@pytest.mark.integration
def test_hybrid_sharding_matches_replicated_weights(tmp_path):
    """HSDP: 4 ranks = 2 replicas x 2 shards (fsdp.dp_replicate 2 with
    sharded parameters): the losses of 4-way data parallelism with
    replicated weights."""
    def four(p):  # the global batch divisible by 4 ranks x micro-batch
        p.write_text(p.read_text().replace("micro_batch_size: 4", "micro_batch_size: 2"))
        return p

    _run4(four(_cfg(tmp_path, "rep4", False)))
    p = four(_cfg(tmp_path, "hsdp", True))
    p.write_text(p.read_text().replace("  shard_params: true\n", "  shard_params: true\n  dp_replicate: 2\n"))
    _run4(p)
    a, b = _losses(tmp_path / "rep4"), _losses(tmp_path / "hsdp")
    assert len(a) == len(b) == 3
    for x, y in zip(a, b):
        assert abs(x - y) <= 1e-4 * abs(x), (a, b)
    assert (tmp_path / "hsdp" / "checkpoint-3" / "trainer" / "model.safetensors").exists()


@pytest.mark.integration
def test_integrated_rl_with_sharded_parameters(tmp_path):
    """`wavelet rl` on 2 gloo ranks with fsdp.shard_params: the sharded
    trainer trains and its full generator replica is refreshed every step."""
    cfg = tmp_path / "rl.yaml"
    cfg.write_text(f"""model:
  name: tiny
  random_init: true
data:
  source: fake
  seq_len: 128
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
    max_completion_tokens: 8
fsdp:
  backend: gloo
  shard_params: true
lora: null
max_steps: 2
output_dir: {tmp_path / 'out'}
""")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "wavelet_b200", "rl", "@",
                        str(cfg)], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(line) for line in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2]
