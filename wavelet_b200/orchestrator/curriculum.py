"""Task curriculum: which prompt to sample next, and which scored rollout
groups to admit into a training batch (reference orchestrator/curriculum.py).

Samplers over a finite task list:
* ``StandardSampler`` — epoch-shuffled cycling (seed + epoch), resumable
  through its cursor;
* ``DifficultyPoolSampler`` — every task carries an EMA of its group-mean
  reward; pools are reward thresholds (ascending) with sampling weights, an
  unseen task has weight 1; the next task is drawn with probability
  proportional to its pool weight.
Gates (applied after a whole group is scored):
* ``AdvRangeGate`` — reject a group whose advantages all lie in
  [reject_min, reject_max] (e.g. all zero: no learning signal).
All state round-trips through ``state_dict`` / ``load_state_dict``.

``Curriculum`` composes one sampler with named gates: the prompt source asks
it for the next record index (and its ``record:<i>`` task key), the
orchestrator reports each scored group back through ``on_result``, which
feeds the sampler and returns whether every gate admits the group.  Group
outputs are ``{"reward": r, "advantage": a}`` dicts (``a`` a number or a
per-token list) or plain numbers.
"""

from __future__ import annotations

import math
import random
from typing import Any, Iterable, Mapping


def _rewards(outputs) -> list[float]:
    out = []
    for o in outputs:
        r = o.get("reward") if isinstance(o, Mapping) else o
        if r is not None and math.isfinite(float(r)):
            out.append(float(r))
    return out


def _advantages(outputs) -> list[float]:
    out = []
    for o in outputs:
        a = o.get("advantage") if isinstance(o, Mapping) else o
        if a is None:
            continue
        out.extend(float(x) for x in (a if isinstance(a, (list, tuple)) else [a]) if x is not None)
    return out


class StandardSampler:
    def __init__(self, task_count: int, seed: int = 0, shuffle: bool = True, cursor: int = 0):
        if task_count < 1:
            raise ValueError("a curriculum needs at least one task")
        self.n, self.seed, self.shuffle, self.cursor = task_count, seed, shuffle, cursor
        self._epoch, self._order = None, []

    def next_index(self) -> int:
        epoch, off = divmod(self.cursor, self.n)
        if self._epoch != epoch:
            self._order = list(range(self.n))
            if self.shuffle:
                random.Random(self.seed * 7919 + epoch).shuffle(self._order)
            self._epoch = epoch
        self.cursor += 1
        return self._order[off]

    def observe(self, task_key: str, rewards: Iterable[float]) -> None:
        pass

    def state_dict(self) -> dict[str, Any]:
        return {"cursor": self.cursor, "task_count": self.n}

    def load_state_dict(self, sd: Mapping[str, Any]) -> None:
        if int(sd["task_count"]) != self.n:
            raise ValueError(f"task count changed across resume ({sd['task_count']} -> {self.n})")
        self.cursor, self._epoch = int(sd["cursor"]), None

    def metrics(self) -> dict[str, float]:
        return {"cursor": float(self.cursor)}


class DifficultyPoolSampler:
    def __init__(self, cfg, task_count: int):
        if task_count < 1:
            raise ValueError("a curriculum needs at least one task")
        self.cfg = cfg
        self.n = task_count
        self.pools = sorted(cfg.pools.items(), key=lambda kv: kv[1].threshold)
        self.rng = random.Random(cfg.seed)
        self.ema: dict[int, float] = {}
        self.selections = 0

    def pool_of(self, idx: int) -> str | None:
        r = self.ema.get(idx)
        if r is None:
            return None
        for name, p in self.pools:
            if r <= p.threshold:
                return name
        return self.pools[-1][0]

    def weight(self, idx: int) -> float:
        p = self.pool_of(idx)
        return 1.0 if p is None else self.cfg.pools[p].weight

    def next_index(self) -> int:
        w = [self.weight(i) for i in range(self.n)]
        if not any(x > 0 for x in w):
            raise RuntimeError("no task has a positive sampling weight")
        self.selections += 1
        return self.rng.choices(range(self.n), weights=w, k=1)[0]

    @property
    def task_rewards(self) -> dict[str, float]:
        return {f"record:{k}": v for k, v in sorted(self.ema.items())}

    def task_pool(self, task_key: str) -> str | None:
        return self.pool_of(int(str(task_key).rsplit(":", 1)[-1]))

    def observe(self, task_key, rewards: Iterable) -> None:
        idx = int(str(task_key).rsplit(":", 1)[-1])
        vals = _rewards(rewards)
        if not vals:
            return
        m = sum(vals) / len(vals)
        prev = self.ema.get(idx)
        a = self.cfg.ema_alpha
        self.ema[idx] = m if prev is None else a * m + (1 - a) * prev

    def state_dict(self) -> dict[str, Any]:
        return {"rng": self.rng.getstate(), "selections": self.selections, "task_count": self.n,
                "task_rewards": {f"record:{k}": v for k, v in self.ema.items()}}

    def load_state_dict(self, sd: Mapping[str, Any]) -> None:
        if int(sd["task_count"]) != self.n:
            raise ValueError(f"task count changed across resume ({sd['task_count']} -> {self.n})")
        st = sd["rng"]
        self.rng.setstate((st[0], tuple(st[1]), st[2]) if isinstance(st, list) else st)
        self.selections = int(sd["selections"])
        self.ema = {int(str(k).rsplit(":", 1)[-1]): float(v) for k, v in sd["task_rewards"].items()}

    def metrics(self) -> dict[str, float]:
        occ = {name: 0 for name, _ in self.pools}
        for i in self.ema:
            occ[self.pool_of(i)] += 1
        m = {"pool/unseen": float(self.n - len(self.ema)), "selections": float(self.selections),
             "reward_ema/mean": sum(self.ema.values()) / len(self.ema) if self.ema else 0.0}
        m.update({f"pool/{k}": float(v) for k, v in occ.items()})
        return m


class AdvRangeGate:
    def __init__(self, cfg):
        self.cfg = cfg
        self.admitted = 0
        self.rejected = 0

    def admit(self, outputs: Iterable) -> bool:
        """False when every advantage of the group lies in [reject_min, reject_max]."""
        adv = _advantages(outputs)
        ok = not adv or not all(self.cfg.reject_min <= a <= self.cfg.reject_max for a in adv)
        if ok:
            self.admitted += 1
        else:
            self.rejected += 1
        return ok

    def state_dict(self) -> dict[str, Any]:
        return {"admitted": self.admitted, "rejected": self.rejected}

    def load_state_dict(self, sd: Mapping[str, Any]) -> None:
        self.admitted, self.rejected = int(sd["admitted"]), int(sd["rejected"])

    def metrics(self) -> dict[str, float]:
        tot = self.admitted + self.rejected
        return {"admitted": float(self.admitted), "rejected": float(self.rejected),
                "admission_rate": self.admitted / tot if tot else 1.0}


def build_curriculum(cfg, task_count: int, seed: int = 0, shuffle: bool = True):
    """(sampler, {name: gate}) from an ``RLCurriculumConfig`` (None: standard, no gates)."""
    if cfg is None or cfg.sampler.type == "standard":
        sampler = StandardSampler(task_count, seed, shuffle)
    else:
        sampler = DifficultyPoolSampler(cfg.sampler, task_count)
    gates = {name: AdvRangeGate(g) for name, g in (cfg.gates.items() if cfg is not None else [])}
    return sampler, gates


class Curriculum:
    """Sampler + gates with one checkpointable state (reference
    orchestrator/curriculum.py: ``Curriculum``)."""

    def __init__(self, cfg, task_count: int, data_seed: int = 0, shuffle: bool = True):
        self.sampler, self.gates = build_curriculum(cfg, task_count, data_seed, shuffle)

    def next_record_index(self) -> tuple[int, str]:
        i = self.sampler.next_index()
        return i, f"record:{i}"

    def on_result(self, task_key: str, outputs: list) -> bool:
        self.sampler.observe(task_key, outputs)
        ok = True
        for g in self.gates.values():  # every gate sees (and counts) the group
            ok = g.admit(outputs) and ok
        return ok

    def state_dict(self) -> dict[str, Any]:
        return {"sampler": self.sampler.state_dict(), "gates": {k: g.state_dict() for k, g in self.gates.items()}}

    def load_state_dict(self, sd: Mapping[str, Any]) -> None:
        self.sampler.load_state_dict(sd["sampler"])
        for k, g in self.gates.items():
            if k in sd.get("gates", {}):
                g.load_state_dict(sd["gates"][k])

    def metrics(self) -> dict[str, float]:
        m = {f"sampler/{k}": v for k, v in self.sampler.metrics().items()}
        for name, g in self.gates.items():
            m.update({f"gate/{name}/{k}": v for k, v in g.metrics().items()})
        return m
