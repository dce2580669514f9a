"""Per-step rollout metrics of a published batch (metric names of the
reference's monitor.py:849-1280)."""

from __future__ import annotations

import pytest

from wavelet_b200.orchestrator.rollout_metrics import rollout_metrics, series_stats


def _row(group, reward, adv, n_prompt, n_comp, env="math", policy=3, trunc=False, stop="stop", count=1, turns=1):
    return {"input_ids": [1] * (n_prompt + n_comp), "loss_mask": [False] * n_prompt + [True] * n_comp,
            "reward": reward, "advantage": adv,
            "metadata": {"group": group, "env": env, "policy_step": policy, "is_truncated": trunc,
                         "stop_condition": stop, "rollout_count": count, "turn_count": turns}}


def test_batch_metrics():
    rows = [_row("g0", 1.0, 0.5, 4, 6), _row("g0", 0.0, -0.5, 4, 2, trunc=True, stop="length"),
            _row("g1", 1.0, 0.0, 3, 3, env="code", turns=3), _row("g1", 1.0, 0.0, 3, 5, env="code", turns=3),
            _row("g1", 1.0, 0.0, 9, 2, env="code", count=0, turns=3)]  # second row of the previous rollout
    m = rollout_metrics(rows, step=5, group_size=2, policy_step=3, stats={"rollout/zero_advantage_dropped": 4.0})
    assert m["progress/samples"] == 4.0 and m["progress/problems"] == 2.0
    assert m["progress/tokens"] == 10 + 6 + 6 + 8 + 11 and m["progress/decode_tokens"] == 6 + 2 + 3 + 5 + 2
    assert m["policy/lag"] == 2.0 and m["off_policy/max"] == 2.0
    # g0 half solved, g1 fully solved (its rollout_count-0 row is not another sample)
    assert m["solve_all/all"] == 0.5 and m["solve_none/all"] == 0.0 and m["effective_batch_size/all"] == 0.5
    assert m["reward/all/mean"] == pytest.approx((0.5 + 1.0) / 2)
    assert m["stop_condition/all/length"] == pytest.approx(1 / 5)
    assert m["stop_condition/all/generation_truncated"] == pytest.approx(1 / 5)
    assert m["num_turns/all/max"] == 3.0 and m["is_truncated/all/mean"] == pytest.approx(0.25)
    assert m["batch/math"] == pytest.approx(2 / 5) and m["train/code/solve_all"] == 1.0
    assert m["train/math/group_fraction"] == 0.5
    assert m["fate/all/filtered"] == 4.0 and m["fate/all/trainable"] == 4.0
    assert m["advantage/all/min"] == -0.5


def test_single_environment_has_no_per_env_keys_and_stats_helper():
    rows = [_row("a", 0.0, 0.0, 2, 2, env=None), _row("a", 0.0, 0.0, 2, 2, env=None)]
    for r in rows:
        r["metadata"].pop("env")
    m = rollout_metrics(rows, step=0, group_size=2)
    assert m["solve_none/all"] == 1.0 and not any(k.startswith("train/") for k in m)
    assert "policy/lag" not in m
    assert series_stats("x", []) == {}
    assert series_stats("x", [1.0, 3.0]) == {"x/mean": 2.0, "x/max": 3.0, "x/std": 1.0, "x/min": 1.0}
