"""Schedule arithmetic shared by the trainer and rollout roles
(orchestrator/schedule.py:14-153 of the reference).

* ``max_policy_lag`` — how many optimizer steps behind the newest policy a
  rollout batch may be generated: ``max_async_level`` (+ ``max_off_policy_steps``).
* ``required_policy_step(step)`` — the oldest policy snapshot allowed for the
  batch of optimizer step ``step``.
* ``retained_policy_snapshots`` — snapshots to keep so every allowed policy
  is still on disk.
"""

from __future__ import annotations


def target_steps(cfg) -> int:
    return int(cfg.max_steps if cfg.max_steps is not None else 1)


def chunks_per_step(cfg) -> int:
    o = cfg.orchestrator
    if o.rollout_chunk_examples and o.examples_per_step:
        return max(1, -(-o.examples_per_step // o.rollout_chunk_examples))
    return 1


def max_policy_lag(cfg) -> int:
    o = cfg.orchestrator
    return int(o.max_async_level) + int(o.max_off_policy_steps)


def required_policy_step(step: int, cfg) -> int:
    return max(0, step - max_policy_lag(cfg))


def retained_policy_snapshots(cfg) -> int:
    return max(cfg.policy_transfer.keep_last, max_policy_lag(cfg) + 2)
