"""Reward scoring (orchestrator/reward.py:71 of the reference).

Modes:
* ``passthrough`` — the rollout carries its own reward;
* ``reference_match`` — 1 when the assistant completion equals the target
  completion after whitespace / case normalisation;
* ``math_format`` — answer extracted between ``solution_start`` /
  ``solution_end`` after ``reasoning_end`` and compared numerically or
  textually, with a small format bonus;
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
from decimal import Decimal, InvalidOperation

from ..data.rl import RLExample


def assistant_text(messages) -> str:
    if not messages:
        return ""
    if isinstance(messages, str):
        return messages
    return "".join(str(m.get("content") or "") for m in messages if m.get("role") == "assistant")


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
            raise ValueError("reward.mode='math_format' requires the expected answer in target_completion.")
        got = self._extract(resp)
        ans = self._answer_score(got, want)
        fmt = self._format_bonus(resp)
        if ans >= 1.0:
            return min(1.0, 0.9 + fmt)
        if ans > 0.0:
            return min(0.6, ans + min(fmt, 0.05))
        return min(0.05, fmt)

    def _extract(self, resp: str) -> str | None:
        c = self.cfg
        tail = resp.split(c.reasoning_end, 1)[1] if c.reasoning_end in resp else resp
        m = re.search(re.escape(c.solution_start) + r"(.*?)" + re.escape(c.solution_end), tail, re.S)
        if m:
            return self._norm(m.group(1))
        m = re.search(re.escape(c.solution_start) + r"(.*)$", tail, re.S)
        return self._norm(m.group(1)) if m else None

    def _format_bonus(self, resp: str) -> float:
        c = self.cfg
        s = 0.0
        s += 0.025 if c.reasoning_end in resp else 0.0
        s += 0.025 if c.solution_start in resp else 0.0
        s += 0.05 if c.solution_end in resp else 0.0
        return s

    @staticmethod
    def _num(t: str) -> Decimal | None:
        m = re.search(r"-?\d[\d,]*\.?\d*(?:[eE]-?\d+)?", t or "")
        if not m:
            return None
        try:
            return Decimal(m.group(0).replace(",", ""))
        except InvalidOperation:
            return None

    def _answer_score(self, got: str | None, want: str) -> float:
        if got is None:
            return 0.0
        if got == want:
            return 1.0
        a, b = self._num(got), self._num(want)
        if a is not None and b is not None:
            if a == b:
                return 1.0
            if b != 0 and abs(a - b) / abs(b) <= Decimal("0.1"):
                return 0.5
        if want in got:
            return 0.5
        return 0.0
