"""Reward scoring (orchestrator/reward.py:71 of the reference).

Modes:
* ``passthrough`` — the rollout carries its own reward;
* ``reference_match`` — 1 when the assistant completion equals the target
  completion after whitespace / case normalisation;
* ``math_format`` — the answer is taken from, in order: the strict
  ``reasoning_end ... solution_start X solution_end`` layout ending the
  response; the last ``solution_start``/``solution_end`` pair (or
  ``<start_solution>``, ``<answer>``, ``<final_answer>``, ``\\boxed{}``); an
  "answer / solution / therefore / so ... is|:|= X" line ending the
  response; the first number of the last line.  It scores 1 when it equals
  the target after LaTeX / thousands-separator compaction, is equivalent
  under ``math_verify`` (when installed) or as a number (``a/b`` and
  ``\\frac{a}{b}`` included); 0.35 / 0.20 within 1 % / 5 % relative error.
  Format bonus: 0.10 for the strict layout, 0.06 for exactly one tag pair,
  0.02 for any tag.  Reward = min(1, 0.9 + bonus) when right, min(0.6,
  partial + min(bonus, 0.05)) when close, else min(0.05, bonus) — the
  scoring of the reference's orchestrator/reward.py:12-254;
* ``reverse_match`` — the synthetic verifiable reward of the GRPO benchmark:
  the fraction of generated tokens equal to the reversed prompt tokens
  (position-wise), computed on token ids;
* ``environment`` — the reward function of the native environment named in
  the rollout's metadata (``wavelet_b200.environments``).  Rollouts from an
  environment are scored by it under ``passthrough`` too when they carry no
  reward of their own.

Post-processing: optional rescale to [0, 1] from [rescale_min, rescale_max],
then clamp.
"""

from __future__ import annotations

import re
from fractions import Fraction
from functools import lru_cache

from ..data.rl import RLExample


def assistant_text(messages) -> str:
    if not messages:
        return ""
    if isinstance(messages, str):
        return messages
    return "\n".join(str(m.get("content") or "") for m in messages if m.get("role") == "assistant")


def reverse_match_score(prompt_ids: list[int], completion_ids: list[int]) -> float:
    """Fraction of generated tokens that equal the reversed prompt, position by position."""
    if not completion_ids:
        return 0.0
    rev = list(reversed(prompt_ids))
    hits = sum(1 for i, t in enumerate(completion_ids) if i < len(rev) and rev[i] == t)
    return hits / len(completion_ids)


# environments built with non-default arguments, registered by the prompt
# source's owner so that scoring uses the same instance (name -> Environment)
_ENV_OVERRIDE: dict = {}


def register_environment(env) -> None:
    _ENV_OVERRIDE[env.name] = env


class RLRewardScorer:
    def __init__(self, cfg):
        self.cfg = cfg

    def score(self, r: RLExample) -> float:
        c = self.cfg
        md = r.metadata or {}
        if md.get("reward_source") in ("verifier", "custom") and r.reward is not None:
            return float(r.reward)  # scored by its verifiers-package environment / the user rollout function
        if md.get("env") and (c.mode == "environment" or (c.mode == "passthrough" and r.reward is None)):
            from .. import environments

            env = _ENV_OVERRIDE.get(md["env"]) or environments.load_environment(md["env"])
            return self._post(float(env.reward(assistant_text(r.completion), md.get("env_row") or {})))
        if c.mode == "environment":
            raise ValueError("reward.mode='environment' needs rollouts from a native environment (metadata.env)")
        if c.mode == "passthrough":
            if r.reward is None:
                raise ValueError("reward.mode='passthrough' requires each rollout row to provide a reward.")
            return self._post(float(r.reward))
        if c.mode == "reference_match":
            want = assistant_text(r.target_completion)
            if not want:
                raise ValueError("reward.mode='reference_match' requires a target assistant completion.")
            return self._post(1.0 if self._norm(assistant_text(r.completion)) == self._norm(want) else 0.0)
        if c.mode == "math_format":
            return self._post(self._math(r))
        if c.mode == "reverse_match":
            md = r.metadata or {}
            p = md.get("prompt_ids")
            comp = md.get("completion_ids")
            if p is None or comp is None:
                if r.input_ids is None or r.loss_mask is None:
                    raise ValueError("reward.mode='reverse_match' needs token ids")
                p = [t for t, m in zip(r.input_ids, r.loss_mask) if not m]
                comp = [t for t, m in zip(r.input_ids, r.loss_mask) if m]
            return self._post(reverse_match_score(list(p), list(comp)))
        raise ValueError(f"Unsupported reward mode: {c.mode}")

    def _post(self, s: float) -> float:
        c = self.cfg
        if c.rescale_min is not None and c.rescale_max is not None:
            s = (s - c.rescale_min) / (c.rescale_max - c.rescale_min)
        if c.clamp_min is not None:
            s = max(c.clamp_min, s)
        if c.clamp_max is not None:
            s = min(c.clamp_max, s)
        return s

    def _norm(self, t: str) -> str:
        if self.cfg.normalize_whitespace:
            t = re.sub(r"\s+", " ", t.strip())
        if not self.cfg.case_sensitive:
            t = t.casefold()
        return t

    # --------------------------------------------------------------- math
    def _math(self, r: RLExample) -> float:
        resp = assistant_text(r.completion)
        want = self._norm(assistant_text(r.target_completion))
        if not want:
            raise ValueError("reward.mode='math_format' requires target_completion/completion "
                             "to contain the expected answer.")
        ans = self._answer_score(self._extract(resp), want)
        fmt = self._format_bonus(resp)
        if ans >= 1.0:
            return min(1.0, 0.9 + fmt)
        if ans > 0.0:
            return min(0.6, ans + min(fmt, 0.05))
        return min(0.05, fmt)

    def _strict(self) -> re.Pattern[str]:
        c = self.cfg
        return re.compile(re.escape(c.reasoning_end) + r".*?" + re.escape(c.solution_start) + r"(.+?)"
                          + re.escape(c.solution_end) + r"\s*(?:<\|endoftext\|>)?\s*\Z", re.S)

    def _extract(self, resp: str) -> str | None:
        c = self.cfg
        m = self._strict().search(resp)
        if m:
            return m.group(1)
        pairs = [(c.solution_start, c.solution_end, re.S | re.M)] + [
            (a, b, re.S | re.M | re.I) for a, b in (("<start_solution>", "</start_solution>"), ("<answer>", "</answer>"),
                                                    ("<final_answer>", "</final_answer>"))]
        for a, b, flags in pairs:
            found = re.findall(re.escape(a) + r"(.+?)" + re.escape(b), resp, flags)
            if found:
                return found[-1]
        boxed = re.findall(r"\\boxed\{([^{}]+)\}", resp)
        if boxed:
            return boxed[-1]
        m = re.search(r"\b(?:answer|solution|therefore|so)\b[^\n]*?(?:[:=]|\bis\b)\s*([^\n]+)$", resp.strip(), re.I)
        if m:
            return m.group(1)
        return _first_number(resp.splitlines()[-1] if resp else "")

    def _format_bonus(self, resp: str) -> float:
        c = self.cfg
        if self._strict().search(resp):
            return 0.10
        if resp.count(c.solution_start) == 1 and resp.count(c.solution_end) == 1:
            return 0.06
        return 0.02 if (c.solution_start in resp or c.solution_end in resp) else 0.0

    def _answer_score(self, got: str | None, want: str) -> float:
        if got is None:
            return 0.0
        got = self._norm(got)
        if _compact(got) == _compact(want) or _math_verify_equal(got, want):
            return 1.0
        a = _as_number(got)
        if a is None:
            first = _first_number(got)
            a = _as_number(first) if first is not None else None
        b = _as_number(want)
        if a is None or b is None:
            return 0.0
        if a == b:
            return 1.0
        if b == 0:
            return 0.0
        rel = abs((a - b) / b)
        return 0.35 if rel <= Fraction(1, 100) else 0.20 if rel <= Fraction(5, 100) else 0.0


_NUMBER = re.compile(r"[-+]?(?:(?:\d{1,3}(?:,\d{3})+|\d+)(?:\.\d+)?|\.\d+)(?:/\d+(?:\.\d+)?)?")


def _first_number(text: str) -> str | None:
    for m in _NUMBER.finditer(text):
        t = m.group(0).replace(",", "")
        if t not in ("", "+", "-", ".", "+.", "-."):
            return t
    return None


def _compact(text: str) -> str:
    """Answer text without LaTeX wrappers, dollars, thousands separators and spaces."""
    t = re.sub(r"\\boxed\{([^{}]+)\}", r"\1", text.strip())
    t = re.sub(r"\\(?:text|mathrm)\{([^{}]+)\}", r"\1", t).replace("$", "")
    t = re.sub(r"(?<=\d),(?=\d{3}\b)", "", t)
    return re.sub(r"\s+", "", t).strip(" .,:;")


def _as_number(text: str) -> Fraction | None:
    """Integer, decimal, ``a/b`` or ``\\frac{a}{b}`` (also d/tfrac) as an exact fraction."""
    t = _compact(text).strip("()[]{}")
    m = re.fullmatch(r"\\[dt]?frac\{?([-+]?\d+(?:\.\d+)?)\}?\{([-+]?\d+(?:\.\d+)?)", t)
    try:
        if m:
            return Fraction(m.group(1)) / Fraction(m.group(2))
        if re.fullmatch(r"[-+]?\d+(?:\.\d+)?/[-+]?\d+(?:\.\d+)?", t):
            a, b = t.split("/")
            return Fraction(a) / Fraction(b)
        if re.fullmatch(r"[-+]?\d+(?:\.\d+)?", t):
            return Fraction(t)
    except (ValueError, ZeroDivisionError):
        return None
    return None


@lru_cache(maxsize=1)
def _math_verify():
    try:
        from math_verify import parse, verify
    except ImportError:
        return None
    return parse, verify


def _math_verify_equal(got: str, want: str) -> bool:
    api = _math_verify()
    if api is None:
        return False
    parse, verify = api
    try:
        a, b = parse(want), parse(got)
        return bool(a and b and verify(a, b))
    except Exception:  # a parser failure is no match
        return False
