"""Token-sized rollout steps (orchestrator.token_batch_size): groups are drawn
in rounds sized from the running tokens-per-group estimate until the kept rows
hold the target (ref orchestrator/scheduler.py:553-560)."""

from __future__ import annotations

from dataclasses import dataclass

import pytest

from wavelet_b200.configs.config import RLConfig


@dataclass
class _Comp:
    prompt_index: int
    sample_index: int
    token_ids: list
    logprobs: list
    finish_reason: str = "stop"
    sampling_mask: list | None = None


class _Engine:
    def __init__(self, comp_len=5):
        self.comp_len = comp_len
        self.calls = []

    def generate(self, prompts, params):
        self.calls.append(len(prompts))
        return [_Comp(i, k, [3] * self.comp_len, [-0.5] * self.comp_len)
                for i in range(len(prompts)) for k in range(params.n)]


def _cfg(tmp_path, **orch):
    return RLConfig.model_validate({
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 64, "fake_vocab_size": 64, "fake_prompt_len": 6},
        "orchestrator": {"examples_per_step": None, "rollouts_per_example": 2, "filter_zero_advantage": False,
                         **orch},
        "reward": {"mode": "reverse_match"}, "algo": {"type": "grpo"},
        "lora": None, "output_dir": str(tmp_path / "out")})


def test_token_batches_fill_to_the_target(tmp_path):
    from wavelet_b200.orchestrator.rollouts import RLOrchestrator
    from wavelet_b200.orchestrator.runtime import build_prompt_source

    cfg = _cfg(tmp_path, token_batch_size=100)
    eng = _Engine()
    orch = RLOrchestrator(cfg, eng, None, build_prompt_source(cfg, 64))
    recs = orch.materialize(0)
    # one group first (2 rollouts x 11 tokens = 22), then ceil(78 / 22) = 4 more groups
    assert eng.calls == [1, 4]
    assert sum(len(r.input_ids) for r in recs) == 110 and len(recs) == 10
    assert orch.last_stats["rollout/token_batch_tokens"] == 110.0
    assert orch.last_stats["rollout/token_batch_rounds"] == 2.0
    # the next step starts from the estimate: one round of ceil(100 / 22) = 5 groups
    orch.materialize(1)
    assert eng.calls[-1] == 5


def test_token_batch_rules():
    with pytest.raises(ValueError, match="only one of"):
        RLConfig.model_validate({"orchestrator": {"examples_per_step": 2, "token_batch_size": 64}})
    with pytest.raises(ValueError, match="rollout_chunk_examples cannot be combined"):
        RLConfig.model_validate({"orchestrator": {"examples_per_step": None, "token_batch_size": 64,
                                                  "rollout_chunk_examples": 1}})


def test_oversampling_keeps_the_first_usable_groups(tmp_path):
    from wavelet_b200.orchestrator.rollouts import RLOrchestrator
    from wavelet_b200.orchestrator.runtime import build_prompt_source

    cfg = _cfg(tmp_path, examples_per_step=2, oversampling_factor=2.0)
    eng = _Engine()
    orch = RLOrchestrator(cfg, eng, None, build_prompt_source(cfg, 64))
    recs = orch.materialize(0)
    assert eng.calls == [4]  # ceil(2 x 2.0) groups generated
    assert len({r.metadata["group"] for r in recs}) == 2 and len(recs) == 4


def test_eval_rollout_sets_are_pruned(tmp_path):
    from wavelet_b200.orchestrator.evals import prune_eval_sets

    d = tmp_path / "evals" / "env"
    d.mkdir(parents=True)
    for s in (0, 5, 10, 20):
        (d / f"step-{s}.jsonl").write_text("{}\n")
    (d / "notes.txt").write_text("x")
    removed = prune_eval_sets(d, 2)
    assert sorted(p.name for p in removed) == ["step-0.jsonl", "step-5.jsonl"]
    assert sorted(p.name for p in d.iterdir()) == ["notes.txt", "step-10.jsonl", "step-20.jsonl"]


def test_publish_reuses_a_stable_batch_and_writes_the_materialized_file(tmp_path):
    import json

    from wavelet_b200.orchestrator.rollouts import RLOrchestrator
    from wavelet_b200.orchestrator.runtime import build_prompt_source
    from wavelet_b200.transport.queue import FileSystemRolloutSender

    mpath = tmp_path / "m" / "rollouts.jsonl"
    cfg = _cfg(tmp_path, examples_per_step=2, materialize_path=str(mpath), overwrite=False)
    eng = _Engine()
    sender = FileSystemRolloutSender(tmp_path / "out", cfg.transport)
    orch = RLOrchestrator(cfg, eng, sender, build_prompt_source(cfg, 64))
    b = orch.publish(0, policy_step=0)
    assert eng.calls == [2] and len(mpath.read_text().splitlines()) == 4
    assert json.loads(mpath.read_text().splitlines()[0])["input_ids"]
    # the same step again: the stable batch is reused, nothing is generated
    again = orch.publish(0, policy_step=0)
    assert again.path == b.path and eng.calls == [2]
    events = (tmp_path / "out" / "events").rglob("*.jsonl")
    assert any("rollout_reused" in p.read_text() for p in events)
    # a new step would overwrite the materialized file: refused with overwrite off
    with pytest.raises(FileExistsError, match="overwrite is disabled"):
        orch.publish(1, policy_step=1)
