"""Competition-math RL on Polaris with held-out AIME 2024 evaluation
(reference environments/polaris_math_tagged).

Offline: the rows come from local files (``path``: Polaris rows with
``problem``, ``answer`` and a ``difficulty`` pass-count label such as "3/8";
``eval_path``: AIME rows with ``problem`` and ``answer``), JSONL, JSON or
Parquet.  Training rows are filtered like the reference: difficulty
numerator within [min_difficulty, max_difficulty], no proof requests ("prove",
"show that", ...), no structurally broken answers (an empty ``\\frac`` part, a
leading ``^``, only operator characters), deduplicated and decontaminated
against the evaluation problems by whitespace/case-normalised text.

Reward: 1 when the response is exactly ``<think>..</think><answer>..</answer>``
and the answer is equivalent to the target, else 0.  Equivalence
(``answers_match``) normalises LaTeX wrappers (``$``, ``\\boxed{}``,
``\\left``/``\\right``, ``\\dfrac``/``\\tfrac``, thin spaces, trailing
periods, thousands separators) and compares exactly as rationals when both
sides parse as numbers (integers, decimals, ``a/b``, ``\\frac{a}{b}``), else
as normalised strings.  The reference delegates this to ``math_verify`` in a
process pool; this check is a restricted, deterministic subset that needs no
subprocesses.
"""

from __future__ import annotations

import json
from fractions import Fraction
from pathlib import Path
from typing import Any, Iterable

from . import Environment, split_tagged

SYSTEM_PROMPT = (
    "You solve competition mathematics problems.\n\n"
    "Respond using exactly this structure:\n"
    "<think>your step-by-step reasoning</think>\n"
    "<answer>only the final answer</answer>\n\n"
    "Both tags are required. Do not put any text outside these tags.\n"
)

_PROOF_WORDS = ("prove", "demonstrate", "establish")
_LATEX_REWRITES = ((r"\left", ""), (r"\right", ""), (r"\dfrac", r"\frac"), (r"\tfrac", r"\frac"), (r"\!", ""),
                   (r"\,", ""), (r"\;", ""), ("\\ ", ""), ("{,}", ""))


def normalize_problem(problem: object) -> str:
    return " ".join(str(problem).split()).casefold()


def difficulty_numerator(value: object) -> int | None:
    s = str(value).strip()
    if len(s) == 3 and s[0].isdigit() and s[1:] == "/8" and int(s[0]) <= 8:
        return int(s[0])
    return None


def is_proof_problem(problem: object) -> bool:
    words = "".join(c if c.isalnum() else " " for c in str(problem).casefold()).split()
    if any(w in _PROOF_WORDS for w in words):
        return True
    return any(a == "show" and b == "that" for a, b in zip(words, words[1:]))


def _brace_group(s: str, j: int) -> tuple[str, int] | None:
    """Body and end index of the ``{...}`` group starting at or after j."""
    while j < len(s) and s[j] == " ":
        j += 1
    if j >= len(s) or s[j] != "{":
        return None
    depth = 0
    for k in range(j, len(s)):
        depth += {"{": 1, "}": -1}.get(s[k], 0)
        if depth == 0:
            return s[j + 1:k], k + 1
    return None


def is_malformed_answer(answer: object) -> bool:
    s = str(answer)
    t = s.strip()
    if t.startswith("^"):
        return True
    if t and all(c in "+-*/=^_" for c in t.replace(" ", "")):
        return True
    i = s.find(r"\frac")
    while i >= 0:  # a \frac with an empty numerator or denominator group
        g1 = _brace_group(s, i + 5)
        if g1 is not None:
            g2 = _brace_group(s, g1[1])
            if not g1[0].strip() or (g2 is not None and not g2[0].strip()):
                return True
        i = s.find(r"\frac", i + 5)
    return False


def build_polaris_rows(rows: Iterable[dict[str, Any]], held_out_problems: Iterable[object] = (),
                       min_difficulty: int = 1, max_difficulty: int = 6, exclude_proof_problems: bool = True,
                       exclude_malformed_answers: bool = True) -> list[dict[str, Any]]:
    if not 0 <= min_difficulty <= max_difficulty <= 8:
        raise ValueError("difficulty bounds must satisfy 0 <= min <= max <= 8")
    held = {normalize_problem(p) for p in held_out_problems}
    seen: set[str] = set()
    out = []
    for i, r in enumerate(rows):
        d = difficulty_numerator(r.get("difficulty"))
        if d is None or not min_difficulty <= d <= max_difficulty:
            continue
        problem, answer = str(r.get("problem", "")).strip(), str(r.get("answer", "")).strip()
        key = normalize_problem(problem)
        if not key or not answer or key in held or key in seen:
            continue
        if exclude_proof_problems and is_proof_problem(problem):
            continue
        if exclude_malformed_answers and is_malformed_answer(answer):
            continue
        seen.add(key)
        out.append({"question": problem, "answer": answer, "example_id": f"polaris-{i:05d}",
                    "info": {"difficulty": f"{d}/8"}})
    return out


def format_aime_rows(rows: Iterable[dict[str, Any]]) -> list[dict[str, Any]]:
    return [{"question": str(r["problem"]), "answer": str(int(r["answer"])), "example_id": f"aime2024-{i:02d}",
             "info": {}} for i, r in enumerate(rows)]


# ------------------------------------------------------------------ answers
def _strip_wrappers(s: str) -> str:
    s = s.strip()
    if s.startswith("$") and s.endswith("$"):
        s = s.strip("$").strip()
    for wrap in (r"\boxed{", r"\text{", r"\mathrm{"):
        if s.startswith(wrap) and s.endswith("}"):
            s = s[len(wrap):-1].strip()
    for a, b in _LATEX_REWRITES:
        s = s.replace(a, b)
    return s.rstrip(".").strip()


def _as_number(s: str) -> Fraction | None:
    t = s.replace(" ", "")
    if t.startswith(r"\frac{") and t.endswith("}"):
        body = t[6:-1]
        if body.count("}{") == 1:
            a, b = body.split("}{")
            na, nb = _as_number(a), _as_number(b)
            if na is not None and nb not in (None, 0):
                return na / nb
        return None
    if t.count("/") == 1:
        a, b = t.split("/")
        na, nb = _as_number(a), _as_number(b)
        return na / nb if na is not None and nb not in (None, 0) else None
    if "," in t:
        parts = t.lstrip("+-").split(",")
        if not all(p.isdigit() for p in parts) or any(len(p) != 3 for p in parts[1:]):
            return None
        t = t.replace(",", "")
    try:
        return Fraction(t)
    except (ValueError, ZeroDivisionError):
        return None


def answers_match(got: str, want: str) -> bool:
    a, b = _strip_wrappers(got), _strip_wrappers(want)
    na, nb = _as_number(a), _as_number(b)
    if na is not None and nb is not None:
        return na == nb
    return a.replace(" ", "") == b.replace(" ", "")


def reward(completion: str, row: dict[str, Any]) -> float:
    parts = split_tagged(completion)
    if parts is None:
        return 0.0
    want = row.get("answer")
    if want is None:
        want = (row.get("info") or {}).get("answer")
    return float(want is not None and answers_match(parts[1], str(want)))


def _read(path: str | Path) -> list[dict[str, Any]]:
    p = Path(path)
    if p.suffix == ".parquet":
        import pyarrow.parquet as pq

        return pq.read_table(p).to_pylist()
    text = p.read_text()
    if p.suffix == ".json":
        data = json.loads(text)
        return list(data if isinstance(data, list) else data.get("rows", []))
    return [json.loads(line) for line in text.splitlines() if line.strip()]


def load_environment(path: str | None = None, eval_path: str | None = None, min_difficulty: int = 1,
                     max_difficulty: int = 6, exclude_proof_problems: bool = True,
                     exclude_malformed_answers: bool = True, **_: Any) -> Environment:
    if path is None:
        raise ValueError("polaris_math_tagged needs args.path: a local Polaris file (problem, answer, difficulty); "
                         "this environment does not download datasets")
    evals = format_aime_rows(_read(eval_path)) if eval_path else []
    rows = build_polaris_rows(_read(path), held_out_problems=(r["question"] for r in evals),
                              min_difficulty=min_difficulty, max_difficulty=max_difficulty,
                              exclude_proof_problems=exclude_proof_problems,
                              exclude_malformed_answers=exclude_malformed_answers)
    if not rows:
        raise RuntimeError("Polaris filtering returned no training examples")
    return Environment("polaris_math_tagged", SYSTEM_PROMPT, rows, evals, reward)
