"""Equation-building puzzles (reference environments/equation_builder).

Task: 3-5 distinct two-digit numbers and a target; the model must write an
equation that uses every number exactly once with only ``+``, ``-`` and
parentheses, e.g. ``<answer>71 - 23 + 40 - 15 = 73</answer>``.  Puzzles are
generated from a seeded RNG by applying a random mixed +/- operator pattern to
a random ordering of the numbers, so every puzzle is solvable.  The reward is
1 for a valid equation inside a well-formed think/answer response, else 0;
the expression is evaluated by walking its Python AST (integer literals,
binary +/- and parentheses only), never with ``eval``.
"""

from __future__ import annotations

import ast
import random
from collections import Counter
from dataclasses import dataclass
from typing import Any

from . import Environment, split_tagged

SYSTEM_PROMPT = (
    "You solve arithmetic equation-building puzzles.\n\n"
    "Use each given number exactly once. You may reorder the numbers and use\n"
    "parentheses, but the only arithmetic operators allowed are + and -.\n\n"
    "Reason inside <think>...</think>. Put only the final equation inside\n"
    "<answer>...</answer>, including the target after an equals sign.\n"
)


@dataclass(frozen=True)
class Verdict:
    valid: bool
    reason: str


def _walk(node: ast.AST) -> tuple[int, list[int], int]:
    """(value, literals in order, operator count) of a +/- integer expression."""
    if isinstance(node, ast.Expression):
        return _walk(node.body)
    if isinstance(node, ast.Constant) and type(node.value) is int:
        return node.value, [node.value], 0
    if isinstance(node, ast.BinOp) and isinstance(node.op, (ast.Add, ast.Sub)):
        lv, ln, lo = _walk(node.left)
        rv, rn, ro = _walk(node.right)
        return (lv + rv if isinstance(node.op, ast.Add) else lv - rv), ln + rn, lo + ro + 1
    raise ValueError("only integer literals, +, - and parentheses are allowed")


def _is_int_text(s: str) -> bool:
    t = s[1:] if s[:1] in "+-" else s
    return t.isdigit() and t.isascii()


def check_equation(equation: str, numbers, target: int) -> Verdict:
    nums = list(numbers)
    if not 3 <= len(nums) <= 5:
        return Verdict(False, "the puzzle must contain 3, 4, or 5 numbers")
    if len(set(nums)) != len(nums):
        return Verdict(False, "all given numbers must be unique")
    if not all(type(n) is int and 10 <= n <= 99 for n in nums):
        return Verdict(False, "all given numbers must be two-digit integers")
    if equation.count("=") != 1:
        return Verdict(False, "the answer must contain exactly one equals sign")
    lhs, rhs = (p.strip() for p in equation.split("="))
    if not lhs or not _is_int_text(rhs):
        return Verdict(False, "the equation or integer target is missing")
    if int(rhs) != target:
        return Verdict(False, "the right-hand side does not match the target")
    try:
        value, used, ops = _walk(ast.parse(lhs, mode="eval"))
    except (SyntaxError, ValueError):
        return Verdict(False, "only integer literals, +, - and parentheses are allowed")
    if Counter(used) != Counter(nums):
        return Verdict(False, "the equation must use every given number exactly once")
    if ops != len(nums) - 1:
        return Verdict(False, "the equation must connect all given numbers")
    if value != target:
        return Verdict(False, "the left-hand expression does not equal the target")
    return Verdict(True, "correct")


def build_examples(num_examples: int, seed: int, num_numbers: int = 4, target_min: int = 0,
                   target_max: int = 99) -> list[dict[str, Any]]:
    if num_examples < 1:
        raise ValueError("num_examples must be at least 1")
    if not 3 <= num_numbers <= 5:
        raise ValueError("num_numbers must be 3, 4, or 5")
    if target_min > target_max:
        raise ValueError("target_min must be <= target_max")
    rng = random.Random(seed)
    out: list[dict[str, Any]] = []
    budget = max(1000, 1000 * num_examples)
    while len(out) < num_examples:
        budget -= 1
        if budget < 0:
            raise ValueError("could not generate enough puzzles in the requested target range")
        nums = rng.sample(range(10, 100), num_numbers)
        order = rng.sample(nums, num_numbers)
        while True:  # a mixed pattern: at least one + and one -
            ops = [rng.choice("+-") for _ in range(num_numbers - 1)]
            if len(set(ops)) == 2:
                break
        target = order[0]
        for op, n in zip(ops, order[1:]):
            target = target + n if op == "+" else target - n
        if not target_min <= target <= target_max:
            continue
        shown = ", ".join(map(str, nums))
        out.append({
            "question": (f"The {num_numbers} unique two-digit numbers are {shown}. Using each number exactly once "
                         f"and only the + and - operators, construct an equation whose result is {target}. You may "
                         f"reorder the numbers and use parentheses."),
            "info": {"numbers": nums, "target": target},
            "task": "equation-builder",
            "example_id": f"equation-{seed}-{len(out)}",
        })
    return out


def reward(completion: str, row: dict[str, Any]) -> float:
    parts = split_tagged(completion)
    if parts is None:
        return 0.0
    info = row.get("info", row)
    return float(check_equation(parts[1], info["numbers"], int(info["target"])).valid)


def load_environment(num_examples: int = 4096, eval_examples: int = 256, seed: int = 42, num_numbers: int = 4,
                     target_min: int = 0, target_max: int = 99) -> Environment:
    kw = dict(num_numbers=num_numbers, target_min=target_min, target_max=target_max)
    return Environment("equation_builder", SYSTEM_PROMPT, build_examples(num_examples, seed, **kw),
                       build_examples(eval_examples, seed + 1, **kw), reward)
