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

import hashlib
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


def _md_num(r: RLExample, key: str, default: float = 0.0) -> float:
    v = (r.metadata or {}).get(key, default)
    return float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else default


def _completion_tokens(r: RLExample) -> float:
    """Metadata count when positive, else the trainable tokens of the record."""
    v = _md_num(r, "completion_token_count")
    if v > 0.0 or r.loss_mask is None:
        return v
    return float(sum(bool(x) for x in r.loss_mask))


def _input_tokens(r: RLExample) -> float:
    for key in ("input_token_count", "prompt_token_count"):
        v = _md_num(r, key)
        if v > 0.0:
            return v
    if r.input_ids is None:
        return 0.0
    return max(float(len(r.input_ids)) - _completion_tokens(r), 0.0)


def _is_truncated(r: RLExample) -> bool:
    md = r.metadata or {}
    if "is_truncated" in md:
        return bool(md["is_truncated"])
    ro = md.get("rollout")
    return isinstance(ro, dict) and bool(ro.get("is_truncated"))


def center(values: list[float]) -> list[float]:
    m = sum(values) / len(values)
    return [v - m for v in values]


def efficiency_shaped(rewards: list[float], costs: list[float]) -> list[float]:
    """Among the best-reward rollouts, the cheaper ones earn a bonus: each
    is scaled by 1 + clamp(1 - cost / mean cost of the best, 0, 1); the
    shaped rewards are then centred (orchestrator/advantage.py:126-149).
    Groups without a positive reward, or whose best rollouts cost nothing,
    are only centred."""
    if len(rewards) != len(costs):
        raise ValueError("rewards and costs must have the same length")
    best = max(rewards)
    if best <= 0:
        return center(rewards)
    top = [r >= best for r in rewards]
    top_costs = [c for c, t in zip(costs, top) if t]
    mean_cost = sum(top_costs) / len(top_costs)
    if mean_cost <= 0:
        return center(rewards)
    return center([r * (1.0 + min(max(1.0 - c / mean_cost, 0.0), 1.0)) if t else r
                   for r, c, t in zip(rewards, costs, top)])


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
_NAME_ATTR = "_wavelet_b200_algorithm_name"


def register_algorithm(name: str):
    """Decorator for user files: ``@register_algorithm("mine")`` names a class
    or factory (called with the config's ``kwargs``) within its own file
    (orchestrator/custom_algorithms.py:19-130 of the reference).  Names are
    file-local: two files may both define "mine"."""
    if not name.strip():
        raise ValueError("Custom algorithm registration name must not be empty.")
    if name != name.strip():
        raise ValueError("Custom algorithm registration name must not have surrounding whitespace.")

    def deco(obj):
        setattr(obj, _NAME_ATTR, name)
        return obj

    return deco


def _load_module(path: Path):
    mod_name = "_wavelet_b200_custom_algorithm_" + hashlib.sha256(str(path).encode()).hexdigest()[:16]
    spec = importlib.util.spec_from_file_location(mod_name, path)
    if spec is None or spec.loader is None:
        raise ImportError(f"cannot import custom algorithm file {path}")
    mod = importlib.util.module_from_spec(spec)
    previous = sys.modules.get(mod_name)
    sys.modules[mod_name] = mod
    try:
        spec.loader.exec_module(mod)
    except Exception:
        if previous is None:
            sys.modules.pop(mod_name, None)
        else:
            sys.modules[mod_name] = previous
        raise
    return mod


def load_custom_algorithm(file: Path | str, name: str, kwargs: dict[str, Any] | None = None) -> Algorithm:
    """Import ``file`` (relative paths from the working directory), find the
    object registered as ``name`` (else the module attribute of that name),
    call it with ``kwargs`` and check that both hooks exist."""
    path = Path(file).expanduser().resolve()
    if not path.is_file():
        raise ValueError(f"Custom algorithm file does not exist: {path}")
    mod = _load_module(path)
    named = [v for v in vars(mod).values() if getattr(v, _NAME_ATTR, None) == name]
    if len(named) > 1:
        raise ValueError(f"Custom algorithm name {name!r} is registered more than once in {path}")
    factory = named[0] if named else getattr(mod, name, None)
    if not callable(factory):
        raise TypeError(f"Custom algorithm {name!r} is not callable in {path}")
    algo = factory(**(kwargs or {}))
    missing = [h for h in ("score_rollout", "score_group") if not callable(getattr(algo, h, None))]
    if missing:
        raise TypeError(f"Custom algorithm {name!r} from {path} is missing callable hooks: {', '.join(missing)}.")
    return algo


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


def uses_group_advantages(cfg) -> bool:
    """Whether scoring needs complete rollout groups."""
    return algorithm_scope(cfg) in ("group", "both")


def algorithm_loss_component(cfg) -> str:
    """The token-loss component an algorithm's records train."""
    return {"sft": "ce", "opd": "ref_kl", "opsd": "ref_kl"}.get(cfg.type, "rl")


def algorithm_epsilon(cfg) -> float:
    return getattr(cfg, "epsilon", 1e-6)


def score_records(algo: Algorithm, records: list[RLExample], scope: str,
                  group_key: Callable[[RLExample], Any] | None = None) -> list[RLExample]:
    out = list(records)
    if scope in ("rollout", "both"):
        out = [algo.score_rollout(r) for r in out]
        if not all(isinstance(r, RLExample) for r in out):
            raise TypeError("score_rollout must return RLExample")
    if scope == "rollout" or not out:
        return out
    if scope == "group" and all(r.advantage is not None for r in out):
        return out
    groups: dict[Any, list[int]] = {}
    for i, r in enumerate(out):
        groups.setdefault(group_key(r) if group_key else 0, []).append(i)
    for idx in groups.values():
        res = list(algo.score_group([out[i] for i in idx]))
        if len(res) != len(idx) or not all(isinstance(r, RLExample) for r in res):
            raise ValueError("score_group must return one RLExample for every input record")
        for i, r in zip(idx, res):
            out[i] = r
    return out
