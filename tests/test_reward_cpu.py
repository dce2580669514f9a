"""``math_format`` / ``reference_match`` rewards against the values the
reference's reward tests pin (tests/test_reward.py of the reference)."""

import pytest

from wavelet_b200.configs.config import RLRewardConfig
from wavelet_b200.data.rl import RLExample
from wavelet_b200.orchestrator.reward import RLRewardScorer

MATH = RLRewardScorer(RLRewardConfig(mode="math_format"))


def _rec(response, expected="439"):
    return RLExample(prompt=[{"role": "user", "content": "problem"}],
                     completion=[{"role": "assistant", "content": response}],
                     target_completion=[{"role": "assistant", "content": expected}], advantage=None, reward=None)


def test_unknown_reasoning_start_option_is_rejected():
    with pytest.raises(ValueError, match="reasoning_start"):
        RLRewardConfig(reasoning_start="<start_working_out>")


@pytest.mark.parametrize(("response", "expected", "reward"), [
    ("<end_working_out><SOLUTION>3062</SOLUTION>", "439", 0.05),  # wrong but formatted
    ("<end_working_out><SOLUTION>439</SOLUTION>", "439", 1.0),
    ("Therefore the answer is \\boxed{439}.", "439", 0.9),
    ("<end_working_out><SOLUTION>440</SOLUTION>", "439", 0.39999999999999997),  # within 1 %
    ("<end_working_out><start_solution>439</start_solution>", "439", 0.9),
    ("<end_working_out><SOLUTION>\\frac{1}{2}</SOLUTION>", "0.5", 1.0),
    ("<end_working_out><SOLUTION>1,234</SOLUTION>", "1234", 1.0),
    ("<end_working_out><SOLUTION>12</SOLUTION>", "1,2", 0.05),  # only thousands separators are dropped
    ("The person has 42 apples", "7", 0.0),  # "so" inside "person" is no keyword
])
def test_math_format_pinned_values(response, expected, reward):
    assert MATH.score(_rec(response, expected)) == reward


@pytest.mark.parametrize("response", ["The answer is 42", "So the answer is 42.", "The person has 42 apples",
                                      "Answer: 42", "answer = 42", "The final result is 42"])
def test_math_format_keyword_and_last_line_fallbacks(response):
    assert MATH.score(_rec(response, "42")) == 0.9


def test_terminal_format_bonus_needs_tags_at_the_end():
    r = MATH.score(_rec("<end_working_out><SOLUTION>439</SOLUTION>\njunk\nmore"))
    assert r < 1.0 and r == pytest.approx(0.96)


def test_numeric_partial_credit_bands_and_fraction_without_math_verify(monkeypatch):
    from wavelet_b200.orchestrator import reward

    monkeypatch.setattr(reward, "_math_verify_equal", lambda a, b: False)
    assert MATH.score(_rec("<end_working_out><SOLUTION>\\frac{1}{2}</SOLUTION>", "0.5")) == 1.0
    assert MATH.score(_rec("<end_working_out><SOLUTION>1/2</SOLUTION>", "0.5")) == 1.0
    assert MATH.score(_rec("<end_working_out><SOLUTION>103</SOLUTION>", "100")) == pytest.approx(0.25)  # 3 %: 0.20
    assert MATH.score(_rec("<end_working_out><SOLUTION>0</SOLUTION>", "0.0")) == 1.0
    assert MATH.score(_rec("<end_working_out><SOLUTION>1</SOLUTION>", "0")) == 0.05


def test_reference_match_and_post_processing():
    s = RLRewardScorer(RLRewardConfig(mode="reference_match", case_sensitive=False))
    assert s.score(_rec("  Hello   World ", "hello world")) == 1.0
    s = RLRewardScorer(RLRewardConfig(mode="passthrough", rescale_min=-1.0, rescale_max=1.0, clamp_max=0.9))
    rec = _rec("x")
    assert s.score(RLExample(**{**rec.__dict__, "reward": 1.0})) == pytest.approx(0.9)
    assert s.score(RLExample(**{**rec.__dict__, "reward": 0.0})) == pytest.approx(0.5)
    with pytest.raises(ValueError, match="requires each rollout row to provide a reward"):
        s.score(rec)
