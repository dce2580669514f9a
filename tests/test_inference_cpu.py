"""Inference server routes, HTTP client engine and rollout scheduler on CPU."""

import json
import os
import threading
import time

import pytest
import torch

from wavelet_b200.configs.config import RLConfig
from wavelet_b200.data.rl import RLExample, example_to_payload


def _cfg(tmp_path, **extra):
    d = {
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64, "fake_prompt_len": 6},
        "inference": {"sampling": {"max_completion_tokens": 5}, "vllm": {"server_backend": "offline", "max_num_seqs": 32}},
        "orchestrator": {"examples_per_step": 2, "rollouts_per_example": 2},
        "algo": {"type": "grpo"},
        "reward": {"mode": "reverse_match"},
        "lora": None,
        "output_dir": str(tmp_path / "out"),
        "max_steps": 2,
    }
    d.update(extra)
    return RLConfig.model_validate(d)


@pytest.fixture
def cpu_env(monkeypatch):
    monkeypatch.setenv("WAVELET_FORCE_CPU", "1")


def test_server_routes(tmp_path, cpu_env, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    from fastapi.testclient import TestClient

    from wavelet_b200.inference.server import build_app

    cfg = _cfg(tmp_path)
    app = build_app(cfg)
    c = TestClient(app)
    assert c.get("/health").json()["status"] == "ok"
    assert c.get("/v1/models").json()["data"][0]["id"] == "tiny"
    rec = RLExample(prompt=[], completion=[], advantage=None, reward=None, metadata={"prompt_ids": [5, 6, 7]})
    r = c.post("/annotate", json={"records": [example_to_payload(rec)]}).json()
    out = r["records"][0]
    assert out["input_ids"][:3] == [5, 6, 7] and len(out["inference_logprobs"]) == 5
    assert sum(out["loss_mask"]) == 5
    assert c.post("/pause").json()["status"] == "paused"
    assert c.post("/load_policy", json={"policy_dir": None, "step": 3}).json()["policy_step"] == 3
    assert c.post("/resume").json()["status"] == "resumed"
    comp = c.post("/v1/completions", json={"prompt_token_ids": [[1, 2, 3]], "max_tokens": 4, "n": 2}).json()
    assert len(comp["choices"]) == 2 and len(comp["choices"][0]["token_ids"]) == 4
    tok = c.post("/tokenize", json={"prompt": "abc"}).json()
    assert tok["count"] == 3
    sc = c.post("/score", json={"sequences": [[1, 2, 3, 4]], "prompt_lens": [2]}).json()
    assert len(sc["logprobs"][0]) == 2
    st = c.get("/debug/state").json()
    assert st["policy_step"] == 3


def test_scheduler_publishes_with_policy_lag(tmp_path, cpu_env, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    from wavelet_b200.inference.policy import NativePolicyInferenceEngine
    from wavelet_b200.orchestrator.scheduler import RolloutScheduler
    from wavelet_b200.transport.queue import STABLE, read_training_records, stable_steps, step_dir

    cfg = _cfg(tmp_path, orchestrator={"examples_per_step": 2, "rollouts_per_example": 2, "max_async_level": 1,
                                       "filter_zero_advantage": False})
    out = tmp_path / "out"
    eng = NativePolicyInferenceEngine(cfg)
    eng.setup()
    # the policy snapshot of step 0: the generator's own weights, exported through the filesystem
    from wavelet_b200.transport.policy import PolicyExporter

    PolicyExporter(out, cfg.policy_transfer).export(eng.model, 0)
    assert (step_dir(out / "policies", 0) / STABLE).exists()
    sch = RolloutScheduler(cfg, engine=eng)
    assert sch.run() == 0
    steps = stable_steps(out / "rollouts")
    assert steps == [0, 1]  # step 1 allowed with policy 0 under max_async_level=1
    rows = read_training_records(step_dir(out / "rollouts", 1) / "rollouts.jsonl.train.msgpack")
    assert len(rows) == 4 and all(r["advantage"] is not None for r in rows)
    m = [json.loads(l) for l in (out / "orchestrator_metrics.jsonl").read_text().splitlines()]
    assert m[1]["policy_lag"] == 1


def test_placement_split():
    from wavelet_b200.orchestrator.placement import plan

    cfg = RLConfig.model_validate({"launcher": {"mode": "process", "trainer_num_processes": 4, "inference_num_replicas": 2}})
    p = plan(cfg, available=[str(i) for i in range(8)])
    assert p.trainer_devices == ["0", "1", "2", "3"]
    assert p.inference_devices == [["4", "5"], ["6", "7"]]
    assert p.ports == [8000, 8001]
    with pytest.raises(ValueError):
        plan(RLConfig.model_validate({"launcher": {"mode": "process", "trainer_num_processes": 8}}), available=["0", "1"])


@pytest.mark.integration
@pytest.mark.parametrize("transfer", ["filesystem", "nccl"])
def test_process_mode_end_to_end(tmp_path, transfer):
    """launcher.mode=process on CPU: inference server + rl-trainer + rl-inference
    processes cooperating through HTTP and the filesystem queues.  With
    policy_transfer.type nccl the weights move as device updates (on the CPU
    the peer slots cannot cross processes, so the trainer broadcasts over its
    own gloo group and the rollout role loads every update in order)."""
    import socket
    import subprocess
    import sys
    from pathlib import Path

    def free():
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        p = s.getsockname()[1]
        s.close()
        return p

    port = free()
    extra = f"  type: nccl\n  nccl_port: {free()}\n  nccl_timeout_seconds: 120\n" if transfer == "nccl" else ""
    cfg = tmp_path / "rl.yaml"
    cfg.write_text(f"""model:
  name: tiny
  random_init: true
data:
  source: fake
  seq_len: 128
  fake_vocab_size: 64
  fake_prompt_len: 6
algo:
  type: grpo
reward:
  mode: reverse_match
orchestrator:
  examples_per_step: 2
  rollouts_per_example: 2
inference:
  sampling:
    max_completion_tokens: 5
  http:
    port: {port}
    startup_timeout_seconds: 120
transport:
  poll_interval_seconds: 0.2
  idle_timeout_seconds: 120
policy_transfer:
  poll_interval_seconds: 0.2
  idle_timeout_seconds: 120
{extra}launcher:
  mode: process
  poll_interval_seconds: 0.5
lora: null
max_steps: 2
output_dir: {tmp_path / 'out'}
""")
    root = Path(__file__).resolve().parents[1]
    env = {**os.environ, "WAVELET_FORCE_CPU": "1", "CUDA_VISIBLE_DEVICES": ""}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "rl", "@", str(cfg)], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    logs = ""
    for p in (tmp_path / "out" / "logs").rglob("*.log"):
        logs += p.name + ":\n" + p.read_text()[-1500:]
    assert r.returncode == 0, (r.stderr[-2000:], logs)
    rows = [json.loads(l) for l in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2]
    assert (tmp_path / "out" / "orchestrator_metrics.jsonl").exists()
    if transfer == "nccl":
        info = json.loads((tmp_path / "out" / "policies" / "step-000002" / "update_info.json").read_text())
        assert info["protocol"] == "flat_v1"
