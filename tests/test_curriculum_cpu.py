"""Curriculum samplers, gates and their composition against the behaviour
the reference's curriculum tests pin (tests/test_curriculum.py of the
reference), plus the orchestrator wiring: prompts come from the sampler and
rejected groups never reach the queue."""

import json

import pytest

from wavelet_b200.configs.config import (RLAdvRangeGateConfig, RLConfig, RLCurriculumConfig, RLDifficultyPoolConfig,
                                         RLDifficultyPoolSamplerConfig)
from wavelet_b200.data.rl import RLExample
from wavelet_b200.orchestrator.curriculum import AdvRangeGate, Curriculum, DifficultyPoolSampler, StandardSampler


def _out(reward, advantage):
    return {"reward": reward, "advantage": advantage}


def test_advantage_range_gate_rejects_only_groups_inside_interval():
    gate = AdvRangeGate(RLAdvRangeGateConfig(reject_min=-0.1, reject_max=0.1))
    assert gate.admit([_out(1.0, [0.0, 0.05])]) is False
    assert gate.admit([_out(1.0, [-0.2, 0.0])]) is True
    assert gate.admit([{"reward": 1.0}]) is True
    assert gate.metrics() == {"admitted": 2.0, "rejected": 1.0, "admission_rate": pytest.approx(2 / 3)}


def test_difficulty_pool_sampler_tracks_reward_ema_and_pool_weights():
    cfg = RLDifficultyPoolSamplerConfig(seed=7, ema_alpha=0.5, pools={
        "hard": RLDifficultyPoolConfig(threshold=0.25, weight=0.0),
        "normal": RLDifficultyPoolConfig(threshold=0.75, weight=1.0),
        "easy": RLDifficultyPoolConfig(threshold=1.0, weight=0.0)})
    s = DifficultyPoolSampler(cfg, task_count=3)
    s.observe("record:0", [_out(0.0, 0.0)])
    s.observe("record:0", [_out(1.0, 1.0)])
    s.observe("record:1", [_out(0.5, 0.5)])
    s.observe("record:2", [_out(1.0, 1.0)])
    assert s.task_rewards["record:0"] == pytest.approx(0.5)
    assert (s.task_pool("record:0"), s.task_pool("record:1"), s.task_pool("record:2")) == ("normal", "normal", "easy")
    assert {s.next_index() for _ in range(20)} <= {0, 1}
    assert s.metrics()["pool/normal"] == 2.0


def test_difficulty_pool_state_restores_exact_rng_sequence():
    cfg = RLDifficultyPoolSamplerConfig(seed=11, ema_alpha=1.0)
    a = DifficultyPoolSampler(cfg, task_count=4)
    for i, r in enumerate((0.1, 0.5, 0.9)):
        a.observe(f"record:{i}", [_out(r, 0.0)])
    a.next_index()
    b = DifficultyPoolSampler(cfg, task_count=4)
    b.load_state_dict(json.loads(json.dumps(a.state_dict())))
    assert [a.next_index() for _ in range(20)] == [b.next_index() for _ in range(20)]
    assert b.task_rewards == a.task_rewards


def test_standard_sampler_resumes_epoch_shuffle():
    a = StandardSampler(5, seed=3, shuffle=True)
    assert len([a.next_index() for _ in range(7)]) == 7
    b = StandardSampler(5, seed=3, shuffle=True)
    b.load_state_dict(a.state_dict())
    assert [a.next_index() for _ in range(10)] == [b.next_index() for _ in range(10)]


def test_curriculum_composes_sampler_gate_and_state():
    cfg = RLCurriculumConfig(sampler={"type": "difficulty_pool", "seed": 5, "ema_alpha": 1.0},
                             gates={"zero_signal": {"type": "advantage_range"}})
    cur = Curriculum(cfg, task_count=2, data_seed=0, shuffle=False)
    _, key = cur.next_record_index()
    assert cur.on_result(key, [_out(0.5, 0.0)]) is False
    again = Curriculum(cfg, task_count=2, data_seed=0, shuffle=False)
    again.load_state_dict(json.loads(json.dumps(cur.state_dict())))
    assert again.state_dict()["sampler"]["task_rewards"] == {key: 0.5}
    assert again.metrics()["gate/zero_signal/rejected"] == 1.0


def test_orchestrator_samples_from_and_reports_to_the_curriculum(tmp_path):
    from wavelet_b200.orchestrator.rollouts import RLOrchestrator
    from wavelet_b200.orchestrator.sources import FilePromptSource

    rows = tmp_path / "prompts.jsonl"
    rows.write_text("".join(json.dumps({"prompt_ids": [1, 2, i + 3], "answer": str(i)}) + "\n" for i in range(4)))
    cfg = RLConfig.model_validate({
        "data": {"path": str(rows)}, "output_dir": str(tmp_path / "out"),
        "orchestrator": {"examples_per_step": 2, "rollouts_per_example": 2,
                         "curriculum": {"sampler": {"type": "difficulty_pool", "seed": 1},
                                        "gates": {"zero_signal": {"type": "advantage_range"}}}}})
    src = FilePromptSource(cfg)
    prompts = src.take(2)
    assert all(p.metadata["task_key"].startswith("record:") for p in prompts)
    orch = RLOrchestrator(cfg, engine=None, sender=None, prompts=src)

    def rec(p, g, reward, adv):
        return RLExample(prompt=[], completion=[], advantage=adv, reward=reward,
                         metadata={"group": g, "task_key": p.metadata["task_key"]})

    recs = [rec(prompts[0], "a", 1.0, 0.5), rec(prompts[0], "a", 0.0, -0.5),
            rec(prompts[1], "b", 1.0, 0.0), rec(prompts[1], "b", 1.0, 0.0)]
    kept, rejected = orch._curriculum_gate(recs)
    assert [r.metadata["group"] for r in kept] == ["a", "a"] and rejected == 2
    assert orch.last_stats["curriculum/gate/zero_signal/rejected"] == 1.0
    assert src.curriculum.sampler.task_rewards[prompts[1].metadata["task_key"]] == pytest.approx(1.0)
    sd = json.loads(json.dumps(src.state_dict()))
    src2 = FilePromptSource(cfg)
    src2.load_state_dict(sd)
    assert [p.metadata["task_key"] for p in src2.take(5)] == [p.metadata["task_key"] for p in src.take(5)]
