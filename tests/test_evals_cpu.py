"""Eval metrics against the values the reference's eval tests pin
(tests/test_eval_utils.py of the reference): unbiased pass@k, pass^k,
avg@n, failed rollouts."""

import pytest

from wavelet_b200.orchestrator.evals import group_metrics, pass_at_k, pass_hat_k


def test_pass_at_k_and_pass_hat_k_for_binary_rewards():
    n, c = 4, 2  # rewards [0, 1, 0, 1]
    assert [pass_at_k(n, c, k) for k in (1, 2, 4)] == pytest.approx([0.5, 5 / 6, 1.0])
    assert [pass_hat_k(n, c, k) for k in (1, 2, 4)] == pytest.approx([0.5, 1 / 6, 0.0])
    m = group_metrics("x", {"e": [0.0, 1.0, 0.0, 1.0]})
    assert (m["x/pass@1"], m["x/pass@2"], m["x/pass@4"]) == pytest.approx((0.5, 5 / 6, 1.0))
    assert (m["x/pass^1"], m["x/pass^2"], m["x/pass^4"]) == pytest.approx((0.5, 1 / 6, 0.0))


def test_eval_metrics_include_avg_pass_and_failures():
    m = group_metrics("eval/alphabet", {"a": [0.0, 1.0]})
    assert m["eval/alphabet/avg@2"] == pytest.approx(0.5)
    assert m["eval/alphabet/pass@1"] == pytest.approx(0.5) and m["eval/alphabet/pass@2"] == pytest.approx(1.0)
    assert m["eval/alphabet/pass^1"] == pytest.approx(0.5) and m["eval/alphabet/pass^2"] == pytest.approx(0.0)
    assert m["eval/alphabet/failed_rollouts"] == 0.0
    m = group_metrics("eval/alphabet", {"a": [None, 1.0], "b": [1.0, 1.0]})
    assert m["eval/alphabet/failed_rollouts"] == 1.0
    assert m["eval/alphabet/pass@1"] == pytest.approx((0.5 + 1.0) / 2)
    assert m["eval/alphabet/avg@2"] == pytest.approx(3.0 / 4)
