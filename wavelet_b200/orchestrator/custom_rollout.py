"""User rollout functions (``orchestrator.custom_rollout_function``).

A value of the form ``"module.path:function"`` that does not select the
``verifiers`` environments names a function that replaces generation and
scoring for every step (ref orchestrator/rollouts.py:263-275, 510-525).  It is
called as ``function(orchestrator, records, inference_engine)`` with one
``RLExample`` per prompt drawn for the step and returns the scored rollouts:

* each returned record carries its ``reward`` (the configured reward mode is
  not applied to them) and, for training, ``input_ids``, ``loss_mask`` and
  ``inference_logprobs`` (or chat ``prompt`` / ``completion`` messages that
  the trainer tokenises);
* ``metadata["group"]`` groups rollouts for the group-relative advantage; the
  records handed in carry one group per prompt, and a returned record
  without one is grouped with the rollouts of the same prompt messages.

Advantages, the zero-advantage filter and the curriculum gates then run as
for native rollouts.
"""

from __future__ import annotations

import importlib
import json
from dataclasses import replace
from typing import Any, Callable

from ..data.rl import RLExample


def load_rollout_function(path: str) -> Callable[..., Any]:
    if ":" not in path:
        raise ValueError("orchestrator.custom_rollout_function must be formatted as 'module.path:function_name'.")
    module_name, fn_name = path.split(":", 1)
    fn = getattr(importlib.import_module(module_name), fn_name)
    if not callable(fn):
        raise TypeError(f"custom rollout function is not callable: {path}")
    return fn


class CustomRollout:
    """``RLOrchestrator``'s rollout function that calls a user function."""

    def __init__(self, orchestrator, path: str, engine: Any | None = None):
        self.orchestrator = orchestrator
        self.path = path
        self.fn = load_rollout_function(path)
        self.engine = engine

    def __call__(self, prompts, step: int) -> tuple[list[RLExample], dict[str, float]]:
        records = [RLExample(prompt=list(p.prompt), completion=[], advantage=None, reward=None,
                             target_completion=p.target_completion,
                             metadata={**p.metadata, "group": f"{step}:{i}", "example_id": p.example_id,
                                       "prompt_ids": list(p.prompt_ids)},
                             source="orchestrator")
                   for i, p in enumerate(prompts)]
        out = self.fn(self.orchestrator, records, self.engine)
        if not isinstance(out, (list, tuple)) or not all(isinstance(r, RLExample) for r in out):
            raise TypeError(f"custom rollout function {self.path} must return a list of RLExample")
        res = []
        for r in out:
            if r.reward is None:
                raise ValueError(f"custom rollout function {self.path} returned a record without a reward")
            md = dict(r.metadata or {})
            md.setdefault("group", "prompt:" + json.dumps(r.prompt, sort_keys=True, default=str))
            md["reward_source"] = "custom"
            res.append(replace(r, metadata=md))
        return res, {"rollout/custom_records": float(len(res))}
