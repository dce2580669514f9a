"""Credit assignment: advantages from rewards.

Algorithms expose two hooks, ``score_rollout(record)`` (per rollout) and
``score_group(records)`` (per prompt group), exactly like the reference's
orchestrator/algorithms.py:39-258 and advantage.py:15-206:

* passthrough — keep the record's advantage;
* reward — advantage = reward;
* grpo — group-centred rewards (optionally std-normalised), with length
  penalties: ``tokens`` / ``turns`` (efficiency shaping by cost), ``linear``
  (group-normalised linear costs scaled by the pass rate), ``truncation``
  (fixed penalty for length-truncated rollouts);
* max_rl — (r - mean) / mean, zero when mean <= 0;
* opd / opsd — route to reverse-KL distillation (ref_kl_weight = 1);
* sft — route to token cross-entropy (ce_weight = 1);
* custom — a registered algorithm from a user file (``custom_algorithms``).
"""

from __future__ import annotations

import importlib.util
import math
import sys
from dataclasses import replace
from pathlib import Path
from typing import Any, Callable, Protocol

from ..data.rl import RLExample


class Algorithm(Protocol):
    def score_rollout(self, record: RLExample) -> RLExample: ...

    def score_group(self, records: list[RLExample]) -> list[RLExample]: ...


class BaseAlgorithm:
    def score_rollout(self, record: RLExample) -> RLExample:
        return record

    def score_group(self, records: list[RLExample]) -> list[RLExample]:
        return records


class PassthroughAlgorithm(BaseAlgorithm):
    pass


class RewardAlgorithm(BaseAlgorithm):
    def score_rollout(self, record: RLExample) -> RLExample:
        return record if record.advantage is not None else replace(record, advantage=record.reward)


def _rewards(records: list[RLExample], name: str) -> list[float]:
    missing = [i for i, r in enumerate(records) if r.reward is None]
    if missing:
        raise ValueError(f"{name} requires a reward for every rollout; missing at index(es): {', '.join(map(str, missing))}.")
    return [float(r.reward) for r in records]


def _completion_tokens(r: RLExample) -> float:
    md = r.metadata or {}
    v = md.get("completion_token_count")
    if isinstance(v, (int, float)):
        return float(v)
    return float(sum(bool(x) for x in r.loss_mask)) if r.loss_mask is not None else 0.0


def _md_num(r: RLExample, key: str, default: float = 0.0) -> float:
    v = (r.metadata or {}).get(key)
    return float(v) if isinstance(v, (int, float)) else default


def _input_tokens(r: RLExample) -> float:
    md = r.metadata or {}
    if isinstance(md.get("prompt_token_count"), (int, float)):
        return float(md["prompt_token_count"])
    if r.input_ids is not None and r.loss_mask is not None:
        return float(sum(1 for x in r.loss_mask if not x))
    return 0.0


def _is_truncated(r: RLExample) -> bool:
    md = r.metadata or {}
    return bool(md.get("is_truncated") or md.get("finish_reason") == "length")


def center(values: list[float]) -> list[float]:
    m = sum(values) / len(values)
    return [v - m for v in values]


def efficiency_shaped(rewards: list[float], costs: list[float]) -> list[float]:
    """Among equal-reward rollouts prefer cheaper ones: centred reward minus a
    cost term normalised within the group and scaled by the reward spread."""
    adv = center(rewards)
    if not costs or max(costs) == min(costs):
        return adv
    cmean = sum(costs) / len(costs)
    cspan = max(costs) - min(costs)
    rspan = max(rewards) - min(rewards)
    scale = 0.5 * (rspan if rspan > 0 else 1.0) * (1.0 if any(r > 0 for r in rewards) else 0.0)
    return [a - scale * (c - cmean) / cspan for a, c in zip(adv, costs)]


def group_reward_advantages(rewards: list[float], *, costs: list[float] | None = None, normalize: bool = False,
                            epsilon: float = 1e-6) -> list[float]:
    if not rewards:
        return []
    adv = center(rewards) if costs is None else efficiency_shaped(rewards, costs)
    if normalize:
        std = math.sqrt(sum(a * a for a in adv) / len(adv))
        if std > epsilon:
            adv = [a / std for a in adv]
    return adv


class GRPOAlgorithm(BaseAlgorithm):
    def __init__(self, normalize_advantages: bool = False, epsilon: float = 1e-6, length_penalty: Any = None):
        self.normalize = normalize_advantages
        self.epsilon = epsilon
        self.lp = length_penalty

    def score_group(self, records: list[RLExample]) -> list[RLExample]:
        rewards = _rewards(records, "GRPO")
        lp = self.lp
        kind = getattr(lp, "type", None)
        costs = None
        if kind == "linear":
            outs = [max(_completion_tokens(r), 0.0) for r in records]
            ins = [_input_tokens(r) for r in records]
            turns = [_md_num(r, "turn_count", 1.0) for r in records]
            om, im, tm = max(max(outs), 1.0), max(max(ins), 1.0), max(max(turns), 1.0)
            pass_rate = sum(rewards) / len(rewards)
            rewards = [rw - pass_rate * (lp.num_output_tokens_weight * o / om + lp.num_input_tokens_weight * i / im
                                         + lp.num_turns_weight * t / tm)
                       for rw, o, i, t in zip(rewards, outs, ins, turns)]
        elif kind == "truncation":
            rewards = [rw - lp.penalty if _is_truncated(r) else rw for r, rw in zip(records, rewards)]
        elif kind == "tokens":
            costs = [lp.completion_weight * _completion_tokens(r) + lp.tool_response_weight * _md_num(r, "tool_response_token_count")
                     for r in records]
        elif kind == "turns":
            costs = [_md_num(r, "turn_count", 1.0) for r in records]
        adv = group_reward_advantages(rewards, costs=costs, normalize=self.normalize, epsilon=self.epsilon)
        return [replace(r, advantage=a) for r, a in zip(records, adv)]


class MaxRLAlgorithm(BaseAlgorithm):
    def score_group(self, records: list[RLExample]) -> list[RLExample]:
        rewards = _rewards(records, "MaxRL")
        mean = sum(rewards) / len(rewards) if rewards else 0.0
        adv = [0.0] * len(rewards) if mean <= 0 else [(r - mean) / mean for r in rewards]
        return [replace(r, advantage=a) for r, a in zip(records, adv)]


class DistillAlgorithm(BaseAlgorithm):
    def __init__(self, component: str):
        self.component = component

    def score_rollout(self, record: RLExample) -> RLExample:
        if self.component == "ce":
            return replace(record, advantage=None, ce_weight=1.0)
        return replace(record, advantage=None, ref_kl_weight=1.0)


# ------------------------------------------------------------------ custom
_REGISTRY: dict[str, Callable[..., Algorithm]] = {}


def register_algorithm(name: str):
    """Decorator for user files: ``@register_algorithm("mine")`` on a factory
    or class that accepts ``**kwargs`` (custom_algorithms.py:19-130)."""

    def deco(obj):
        _REGISTRY[name] = obj
        return obj

    return deco


def load_custom_algorithm(file: Path, name: str, kwargs: dict[str, Any]) -> Algorithm:
    file = Path(file)
    mod_name = f"_wavelet_custom_algo_{abs(hash(str(file.resolve())))}"
    if mod_name not in sys.modules:
        spec = importlib.util.spec_from_file_location(mod_name, file)
        if spec is None or spec.loader is None:
            raise ImportError(f"cannot import custom algorithm file {file}")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[mod_name] = mod
        spec.loader.exec_module(mod)
    if name not in _REGISTRY:
        raise KeyError(f"algorithm {name!r} is not registered by {file} (registered: {sorted(_REGISTRY)})")
    return _REGISTRY[name](**kwargs)


# ------------------------------------------------------------------ factory
def build_algorithm(cfg) -> Algorithm:
    t = cfg.type
    if t == "passthrough":
        return PassthroughAlgorithm()
    if t == "reward":
        return RewardAlgorithm()
    if t == "grpo":
        return GRPOAlgorithm(cfg.normalize_advantages, cfg.epsilon, cfg.length_penalty)
    if t == "max_rl":
        return MaxRLAlgorithm()
    if t in ("opd", "opsd"):
        return DistillAlgorithm("ref_kl")
    if t == "sft":
        return DistillAlgorithm("ce")
    if t == "custom":
        return load_custom_algorithm(cfg.file, cfg.algorithm, cfg.kwargs)
    raise ValueError(f"unknown algorithm {t}")


def algorithm_scope(cfg) -> str:
    if cfg.type == "custom":
        return cfg.scope
    return "group" if cfg.type in ("grpo", "max_rl") else "rollout"


def algorithm_epsilon(cfg) -> float:
    return getattr(cfg, "epsilon", 1e-6)


def score_records(algo: Algorithm, records: list[RLExample], scope: str,
                  group_key: Callable[[RLExample], Any] | None = None) -> list[RLExample]:
    out = list(records)
    if scope in ("rollout", "both"):
        out = [algo.score_rollout(r) for r in out]
    if scope == "rollout" or not out:
        return out
    if scope == "group" and all(r.advantage is not None for r in out):
        return out
    groups: dict[Any, list[int]] = {}
    for i, r in enumerate(out):
        groups.setdefault(group_key(r) if group_key else 0, []).append(i)
    for idx in groups.values():
        res = algo.score_group([out[i] for i in idx])
        if len(res) != len(idx):
            raise ValueError("score_group must return one record per input record")
        for i, r in zip(idx, res):
            out[i] = r
    return out
