"""Native verifier environments: puzzle generation, safe equation checking,
the think/answer tag contract, Polaris filtering and answer equivalence, the
environment prompt source and reward scoring."""

import itertools
import json

import pytest

from wavelet_b200 import environments
from wavelet_b200.environments import split_tagged
from wavelet_b200.environments.equation_builder import build_examples, check_equation
from wavelet_b200.environments.polaris_math_tagged import (answers_match, build_polaris_rows, difficulty_numerator,
                                                           is_malformed_answer, is_proof_problem)


def _solve(numbers, target):
    for perm in itertools.permutations(numbers):
        for ops in itertools.product("+-", repeat=len(numbers) - 1):
            expr = str(perm[0]) + "".join(f" {o} {n}" for o, n in zip(ops, perm[1:]))
            if check_equation(f"{expr} = {target}", numbers, target).valid:
                return expr
    return None


def test_equation_examples_are_deterministic_and_solvable():
    a = build_examples(20, seed=3, num_numbers=4)
    assert a == build_examples(20, seed=3, num_numbers=4)
    for r in a:
        info = r["info"]
        assert len(set(info["numbers"])) == 4 and all(10 <= n <= 99 for n in info["numbers"])
        assert 0 <= info["target"] <= 99
        assert _solve(info["numbers"], info["target"]) is not None


@pytest.mark.parametrize("eq,ok", [
    ("71 - 23 + 40 - 15 = 73", True),
    ("(71 - 23) + (40 - 15) = 73", True),
    ("71 - 23 + 40 - 15 = 72", False),       # wrong target
    ("71 - 23 + 40 = 73", False),            # a number unused
    ("71 * 23 + 40 - 15 = 73", False),       # operator not allowed
    ("__import__('os') = 73", False),        # not an arithmetic expression
    ("71 - 23 + 40 - 15 == 73", False),      # two equals signs
])
def test_check_equation(eq, ok):
    assert check_equation(eq, [71, 23, 40, 15], 73).valid is ok


def test_tag_contract():
    assert split_tagged("<think>work</think>\n<answer>5</answer>") == ("work", "5")
    assert split_tagged("pre <think>w</think><answer>5</answer>") is None
    assert split_tagged("<think>w</think><answer>5</answer><answer>6</answer>") is None
    assert split_tagged("<answer>5</answer><think>w</think>") is None
    assert split_tagged("<think> </think><answer>5</answer>") is None


def test_equation_reward():
    env = environments.load_environment("equation_builder", num_examples=4, eval_examples=2, seed=1)
    row = env.examples[0]
    expr = _solve(row["info"]["numbers"], row["info"]["target"])
    good = f"<think>try</think><answer>{expr} = {row['info']['target']}</answer>"
    assert env.reward(good, row) == 1.0
    assert env.reward(f"{expr} = {row['info']['target']}", row) == 0.0


def test_polaris_filtering_and_matching(tmp_path):
    rows = [
        {"problem": "Find x if 2x = 4.", "answer": "2", "difficulty": "3/8"},
        {"problem": "find  X if 2x = 4.", "answer": "2", "difficulty": "3/8"},   # duplicate after normalising
        {"problem": "Prove that 2 is prime.", "answer": "2", "difficulty": "2/8"},  # proof request
        {"problem": "Compute 1/2 + 1/2.", "answer": "\\frac{}{2}", "difficulty": "2/8"},  # malformed answer
        {"problem": "Hard one.", "answer": "7", "difficulty": "8/8"},  # out of the difficulty range
        {"problem": "AIME problem.", "answer": "12", "difficulty": "4/8"},  # held out
        {"problem": "Half of 3?", "answer": "\\dfrac{3}{2}", "difficulty": "5/8"},
    ]
    out = build_polaris_rows(rows, held_out_problems=["AIME   problem."])
    assert [r["question"] for r in out] == ["Find x if 2x = 4.", "Half of 3?"]
    assert difficulty_numerator("3/8") == 3 and difficulty_numerator("9/8") is None
    assert is_proof_problem("Show that n is odd") and not is_proof_problem("Showcase the answer")
    assert is_malformed_answer("^2") and not is_malformed_answer("\\frac{1}{2}")
    assert answers_match("1.5", "\\dfrac{3}{2}") and answers_match("$\\boxed{1,024}$", "1024")
    assert not answers_match("3/4", "0.7")
    p = tmp_path / "polaris.jsonl"
    p.write_text("\n".join(json.dumps(r) for r in rows))
    env = environments.load_environment("polaris_math_tagged", path=str(p))
    row = env.examples[-1]
    assert row["question"] == "Half of 3?"
    assert env.reward("<think>3 halves</think><answer>1.5</answer>", row) == 1.0
    assert env.reward("<think>?</think><answer>2</answer>", row) == 0.0


def test_environment_prompt_source_and_scoring():
    from wavelet_b200.configs.config import RLRewardConfig
    from wavelet_b200.data.rl import RLExample
    from wavelet_b200.orchestrator.reward import RLRewardScorer, register_environment
    from wavelet_b200.orchestrator.sources import EnvironmentPromptSource

    class Tok:
        def encode(self, s):
            return [ord(c) % 250 + 3 for c in s[:64]]

    e1 = environments.load_environment("equation_builder", num_examples=10, eval_examples=2, seed=5)
    register_environment(e1)
    src = EnvironmentPromptSource([(e1, 1.0)], "none", tokenizer=Tok())
    recs = src.take(12)  # wraps into a second epoch
    assert len(recs) == 12 and all(r.metadata["env"] == "equation_builder" for r in recs)
    assert recs[0].prompt[0]["role"] == "system"
    row = recs[0].metadata["env_row"]
    expr = _solve(row["info"]["numbers"], row["info"]["target"])
    ex = RLExample(prompt=recs[0].prompt, reward=None, advantage=0.0,
                   completion=[{"role": "assistant",
                                "content": f"<think>x</think><answer>{expr} = {row['info']['target']}</answer>"}],
                   metadata=recs[0].metadata)
    assert RLRewardScorer(RLRewardConfig(mode="environment")).score(ex) == 1.0
