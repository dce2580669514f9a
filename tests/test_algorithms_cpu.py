"""Advantage algorithms and custom-algorithm loading against the behaviour
the reference's tests pin (tests/test_algorithms.py of the reference): GRPO
centring and length penalties, MaxRL, distillation routing, the custom-file
contract and scope handling."""

from dataclasses import replace
from pathlib import Path

import pytest

from wavelet_b200.configs.config import (CustomAlgorithmConfig, GRPOAlgorithmConfig, MaxRLAlgorithmConfig,
                                         OPSDAlgorithmConfig, PassthroughAlgorithmConfig, RewardAlgorithmConfig,
                                         SFTDistillAlgorithmConfig)
from wavelet_b200.data.rl import RLExample
from wavelet_b200.orchestrator.algorithms import (BaseAlgorithm, DistillAlgorithm, GRPOAlgorithm, MaxRLAlgorithm,
                                                  PassthroughAlgorithm, RewardAlgorithm, algorithm_epsilon,
                                                  algorithm_loss_component, algorithm_scope, build_algorithm,
                                                  efficiency_shaped, register_algorithm, score_records,
                                                  uses_group_advantages)

FIXTURE = Path(__file__).parent / "fixtures" / "custom_algorithms_fixture.py"


def _ex(reward, **md):
    return RLExample(prompt=[{"role": "user", "content": "p"}], completion=[{"role": "assistant", "content": "c"}],
                     advantage=None, reward=reward, source="test", metadata=md or None)


def _custom(name, scope="group", **kwargs):
    return CustomAlgorithmConfig(file=FIXTURE, algorithm=name, scope=scope, kwargs=kwargs)


def test_grpo_centres_without_mutating_and_keeps_order():
    recs = [_ex(1.0), _ex(0.0)]
    out = GRPOAlgorithm().score_group(recs)
    assert [r.advantage for r in out] == pytest.approx([0.5, -0.5])
    assert [r.advantage for r in recs] == [None, None]
    recs = [replace(_ex(0.0), source="a"), replace(_ex(2.0), source="b"), replace(_ex(1.0), source="c")]
    out = GRPOAlgorithm().score_group(recs)
    assert [r.source for r in out] == ["a", "b", "c"] and [r.advantage for r in out] == pytest.approx([-1, 1, 0])


def test_grpo_linear_length_penalty():
    from wavelet_b200.configs.config import LinearLengthPenaltyConfig

    recs = [_ex(1.0, completion_token_count=10, input_token_count=5, turn_count=1),
            _ex(1.0, completion_token_count=20, input_token_count=5, turn_count=1),
            _ex(0.0, completion_token_count=20, input_token_count=5, turn_count=1)]
    lp = LinearLengthPenaltyConfig(num_output_tokens_weight=0.25, num_input_tokens_weight=0.0, num_turns_weight=0.0)
    out = GRPOAlgorithm(length_penalty=lp).score_group(recs)
    assert [r.advantage for r in out] == pytest.approx([7 / 18, 11 / 36, -25 / 36])


def test_grpo_truncation_penalty():
    from wavelet_b200.configs.config import TruncationLengthPenaltyConfig

    recs = [_ex(1.0, is_truncated=False), _ex(1.0, is_truncated=True), _ex(0.0, is_truncated=False)]
    out = GRPOAlgorithm(length_penalty=TruncationLengthPenaltyConfig(penalty=0.5)).score_group(recs)
    assert [r.advantage for r in out] == pytest.approx([0.5, 0.0, -0.5])
    nested = _ex(1.0, rollout={"is_truncated": True})
    out = GRPOAlgorithm(length_penalty=TruncationLengthPenaltyConfig(penalty=0.5)).score_group([nested, _ex(1.0)])
    assert [r.advantage for r in out] == pytest.approx([-0.25, 0.25])


def test_efficiency_shaping_rewards_cheaper_correct_rollouts():
    # best reward 1; mean cost of the best = 20: bonuses 0.5 and 0 -> shaped [1.5, 1, 0]
    assert efficiency_shaped([1.0, 1.0, 0.0], [10.0, 30.0, 5.0]) == pytest.approx([1.5 - 2.5 / 3, 1 - 2.5 / 3, -2.5 / 3])
    assert efficiency_shaped([0.0, 0.0], [1.0, 2.0]) == pytest.approx([0.0, 0.0])  # no success: centred
    assert efficiency_shaped([1.0, 0.0], [0.0, 3.0]) == pytest.approx([0.5, -0.5])  # zero-cost best: centred
    from wavelet_b200.configs.config import TokensLengthPenaltyConfig

    recs = [_ex(1.0, completion_token_count=10), _ex(1.0, completion_token_count=30), _ex(0.0, completion_token_count=5)]
    out = GRPOAlgorithm(length_penalty=TokensLengthPenaltyConfig()).score_group(recs)
    assert out[0].advantage > out[1].advantage > out[2].advantage


def test_grpo_requires_every_reward():
    with pytest.raises(ValueError, match=r"GRPO requires a reward for every rollout; missing at index\(es\): 1"):
        GRPOAlgorithm().score_group([_ex(1.0), _ex(None)])


def test_max_rl():
    assert [r.advantage for r in MaxRLAlgorithm().score_group([_ex(1.0), _ex(0.0)])] == pytest.approx([1.0, -1.0])
    assert [r.advantage for r in MaxRLAlgorithm().score_group([_ex(0.0), _ex(0.0)])] == pytest.approx([0.0, 0.0])


@pytest.mark.parametrize(("cfg", "kind", "scope"), [
    (PassthroughAlgorithmConfig(), PassthroughAlgorithm, "rollout"), (RewardAlgorithmConfig(), RewardAlgorithm, "rollout"),
    (GRPOAlgorithmConfig(), GRPOAlgorithm, "group"), (MaxRLAlgorithmConfig(), MaxRLAlgorithm, "group"),
    (OPSDAlgorithmConfig(), DistillAlgorithm, "rollout"), (SFTDistillAlgorithmConfig(), DistillAlgorithm, "rollout"),
])
def test_build_dispatches_named_config(cfg, kind, scope):
    assert isinstance(build_algorithm(cfg), kind) and algorithm_scope(cfg) == scope


@pytest.mark.parametrize(("cfg", "field", "component"), [
    (OPSDAlgorithmConfig(), "ref_kl_weight", "ref_kl"), (SFTDistillAlgorithmConfig(), "ce_weight", "ce")])
def test_distillation_routes_tokens_without_advantage(cfg, field, component):
    (r,) = score_records(build_algorithm(cfg), [_ex(1.0)], algorithm_scope(cfg))
    assert r.advantage is None and getattr(r, field) == pytest.approx(1.0)
    assert algorithm_loss_component(cfg) == component
    assert algorithm_loss_component(GRPOAlgorithmConfig()) == "rl"


def test_custom_algorithm_with_kwargs():
    cfg = CustomAlgorithmConfig(file=FIXTURE, algorithm="scale", scope="group", kwargs={"factor": 3.0}, epsilon=1e-4)
    assert build_algorithm(cfg).score_group([_ex(2.0)])[0].advantage == pytest.approx(6.0)
    assert uses_group_advantages(cfg) and algorithm_epsilon(cfg) == pytest.approx(1e-4)


def test_custom_algorithm_file_rules(tmp_path, monkeypatch):
    with pytest.raises(ValueError, match="file does not exist"):
        build_algorithm(CustomAlgorithmConfig(file=tmp_path / "missing.py", algorithm="x", scope="group"))
    monkeypatch.chdir(FIXTURE.parent)
    plain = build_algorithm(CustomAlgorithmConfig(file=FIXTURE.name, algorithm="PlainAlgorithm", scope="group"))
    assert isinstance(plain, BaseAlgorithm) and plain.score_group([_ex(1.0)])[0].advantage is None
    with pytest.raises(TypeError, match="score_group"):
        build_algorithm(_custom("rollout_only", scope="rollout"))
    with pytest.raises(ValueError, match="registered more than once"):
        build_algorithm(_custom("twice"))
    with pytest.raises(TypeError, match="is not callable"):
        build_algorithm(_custom("NOT_A_FACTORY"))


def test_custom_hook_results_are_checked():
    with pytest.raises(TypeError, match="score_rollout must return RLExample"):
        score_records(build_algorithm(_custom("bad_rollout", "rollout")), [_ex(1.0)], "rollout")
    with pytest.raises(ValueError, match="one RLExample for every input record"):
        score_records(build_algorithm(_custom("drops_one")), [_ex(1.0), _ex(0.0)], "group")
    (r,) = score_records(build_algorithm(_custom("offset", "rollout", offset=2.0)), [_ex(1.0)], "rollout")
    assert r.advantage == pytest.approx(3.0)


@pytest.mark.parametrize(("scope", "adv"), [("rollout", 1.0), ("group", 1.0), ("both", 2.0)])
def test_custom_scope_controls_hooks(scope, adv):
    (r,) = score_records(build_algorithm(_custom("both", scope)), [_ex(1.0)], scope)
    assert r.advantage == pytest.approx(adv)


def test_group_scoring_keeps_interleaved_order_and_prescored_records():
    recs = [_ex(1.0, g="a"), _ex(10.0, g="b"), _ex(0.0, g="a"), _ex(0.0, g="b")]
    out = score_records(GRPOAlgorithm(), recs, "group", group_key=lambda r: r.metadata["g"])
    assert [r.advantage for r in out] == pytest.approx([0.5, 5.0, -0.5, -5.0])
    pre = [replace(_ex(None), advantage=3.0)]
    assert score_records(GRPOAlgorithm(), pre, "group") == pre


@pytest.mark.parametrize("name", ["", "  ", " padded "])
def test_registration_name_must_be_clean(name):
    with pytest.raises(ValueError, match="registration name"):
        register_algorithm(name)
