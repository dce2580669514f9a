"""``wavelet debug`` probes on CPU: continuous-batch load against (fake)
HTTP replicas, orchestrator benchmark / materialize with the in-process
engine, inference benchmark, trainer parity from a stored column and from
log-probs the trainer computes, and the token dump."""

import json
import os

import pytest
import torch

from wavelet_b200.configs.config import RLConfig


@pytest.fixture
def cpu(monkeypatch):
    monkeypatch.setenv("WAVELET_FORCE_CPU", "1")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)


def _cfg(tmp_path, **extra):
    d = {"model": {"name": "tiny", "random_init": True},
         "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64, "fake_prompt_len": 6},
         "inference": {"sampling": {"max_completion_tokens": 5},
                       "vllm": {"server_backend": "offline", "max_num_seqs": 32},
                       "http": {"ports": [8100, 8101]}},
         "orchestrator": {"examples_per_step": 2, "rollouts_per_example": 2, "filter_zero_advantage": False},
         "algo": {"type": "grpo"}, "reward": {"mode": "reverse_match"}, "lora": None,
         "output_dir": str(tmp_path / "out"), "max_steps": 1}
    d.update(extra)
    return RLConfig.model_validate(d)


def test_continuous_batch_probe_with_fake_servers(tmp_path):
    from wavelet_b200.debug import continuous_batch_probe

    seen = []

    def post(url, payload):
        seen.append(url)
        if len(seen) == 3:
            raise ConnectionError("replica down")
        return {"choices": [{"token_ids": list(range(payload["max_tokens"]))}]}

    rep = continuous_batch_probe(_cfg(tmp_path), count=6, concurrency=3, max_completion_tokens=4, post=post)
    m = rep["metrics"]
    assert m["requests"] == 6 and m["errors"] == 1 and m["tokens"] == 20
    assert m["latency_p50"] is not None and m["tokens_per_second"] > 0
    assert len({u for u in seen}) == 2  # round robin over both replicas
    assert rep["errors"][0]["error"] == "replica down"


def test_orchestrator_benchmark_materialize_and_trainer_parity(tmp_path, cpu, capsys):
    from wavelet_b200.debug import (inference_benchmark, main, probe_orchestrator, runtime_parity_report,
                                    trainer_logprobs_of_rows)
    from wavelet_b200.inference.policy import NativePolicyInferenceEngine
    from wavelet_b200.transport.queue import read_training_records, stable_steps

    cfg = _cfg(tmp_path)
    eng = NativePolicyInferenceEngine(cfg)
    eng.setup()
    bench = inference_benchmark(cfg, count=2, warmup=1, repeats=2, engine=eng)
    assert len(bench["rounds"]) == 2 and bench["tokens_per_second"]["mean"] > 0
    rep = probe_orchestrator(cfg, step=0, engine=eng, write=False)
    assert rep["records_trainable"] == 4 and rep["output_path"] is None and rep["timings"]["materialize"] > 0
    rep = probe_orchestrator(cfg, step=3, engine=eng, write=True)
    assert stable_steps(tmp_path / "out" / "rollouts") == [3]
    path = tmp_path / "out" / "rollouts" / "step-000003" / "rollouts.jsonl.train.msgpack"
    rows = read_training_records(path)
    # the generator's log-probs against the trainer's, same weights: equal up to kernel rounding
    computed = trainer_logprobs_of_rows(cfg, rows, model=eng.generator.m)
    par = runtime_parity_report(path, threshold=1e-3, computed=computed)
    assert par["token_count"] == sum(sum(r["loss_mask"]) for r in rows)
    assert par["passed"], par
    # a stored column that disagrees fails the check
    for r in rows:
        r["trainer_logprobs"] = [x + 0.5 for x in r["inference_logprobs"]]
    p2 = tmp_path / "bad.jsonl"
    p2.write_text("".join(json.dumps(r) + "\n" for r in rows))
    bad = runtime_parity_report(p2, threshold=1e-3)
    assert not bad["passed"] and abs(bad["max_abs_diff"] - 0.5) < 1e-6
    assert main(["trainer", "parity", str(p2), "--json"]) == 1
    out = tmp_path / "tok.jsonl"
    assert main(["trainer", "tokens", str(p2), "--write-tokens", str(out)]) == 0
    first = json.loads(out.read_text().splitlines()[0])
    assert sum(t["trainable"] for t in first) == sum(rows[0]["loss_mask"])
    capsys.readouterr()


def test_preflight_lists_commands_paths_and_environments(tmp_path, monkeypatch):
    import sys

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.debug import build_preflight_report

    monkeypatch.setitem(sys.modules, "verifiers", None)  # the package is absent
    cfg = RLConfig.model_validate({
        "launcher": {"mode": "process", "env_vars": {"common": {"HF_TOKEN": "secret"}}},
        "output_dir": str(tmp_path / "o"), "model": {"name": "tiny", "random_init": True}, "lora": None,
        "data": {"source": "fake"},
        "orchestrator": {"verifier_env_id": "someone/hub-env"},
        "eval": {"env": [{"id": "equation_builder"}, {"id": "reverse"}]}})
    r = build_preflight_report(cfg)
    roles = [c["role"] for c in r["commands"]]
    assert roles == ["inference-server-0", "rl-trainer", "rl-inference"]
    assert all(c["env"].get("HF_TOKEN") in (None, "<redacted>") for c in r["commands"])
    assert r["paths"]["rollouts"].endswith("rollouts") and r["paths"]["policies"].endswith("policies")
    checks = {c["name"]: c for c in r["checks"]}
    assert checks["env:equation_builder"]["status"] == "ok"
    assert checks["env:someone/hub-env"]["status"] == "error" and not r["ok"]
    assert "env:reverse" not in checks
    assert r["summary"]["policy_freshness"]["effective_max_policy_lag"] == 0
