"""Native verifier environments (reference environments/*, which are
``verifiers`` SingleTurnEnv plugins; that package is not in this image).

An ``Environment`` is a system prompt, training and evaluation example rows
(``question``, ``info``, optional ``answer``) and a reward function
``reward(completion_text, row) -> float``.  The orchestrator turns its rows
into chat prompts (``orchestrator.sources.EnvironmentPromptSource``) and
scores completions with its reward (``reward.mode: environment`` or any
rollout whose metadata names an environment).

Built-ins: ``equation_builder`` and ``polaris_math_tagged``.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable


@dataclass
class Environment:
    name: str
    system_prompt: str
    examples: list[dict[str, Any]]
    eval_examples: list[dict[str, Any]]
    reward: Callable[[str, dict[str, Any]], float]
    metadata: dict[str, Any] = field(default_factory=dict)

    def chat(self, row: dict[str, Any]) -> list[dict[str, str]]:
        return [{"role": "system", "content": self.system_prompt}, {"role": "user", "content": str(row["question"])}]


def split_tagged(text: str) -> tuple[str, str] | None:
    """(reasoning, answer) of a response that is exactly ``<think>...</think>``
    followed by ``<answer>...</answer>`` (whitespace around the blocks only,
    each tag once, both bodies non-empty); None for anything else."""
    tags = ("<think>", "</think>", "<answer>", "</answer>")
    if any(text.count(t) != 1 for t in tags):
        return None
    pos = [text.index(t) for t in tags]
    if pos != sorted(pos):
        return None
    if text[: pos[0]].strip() or text[pos[1] + len(tags[1]): pos[2]].strip() or text[pos[3] + len(tags[3]):].strip():
        return None
    think = text[pos[0] + len(tags[0]): pos[1]].strip()
    answer = text[pos[2] + len(tags[2]): pos[3]].strip()
    if not think or not answer:
        return None
    return think, answer


def _registry() -> dict[str, Callable[..., Environment]]:
    from . import equation_builder, polaris_math_tagged

    return {"equation_builder": equation_builder.load_environment,
            "equation-builder": equation_builder.load_environment,
            "polaris_math_tagged": polaris_math_tagged.load_environment,
            "polaris-math-tagged": polaris_math_tagged.load_environment}


def available() -> list[str]:
    return sorted(k for k in _registry() if "_" in k)


def is_native(env_id: str) -> bool:
    return env_id.split("@", 1)[0] in _registry()


_CACHE: dict[tuple, Environment] = {}


def load_environment(env_id: str, **kwargs) -> Environment:
    """Build (once per id and arguments) a native environment."""
    name = env_id.split("@", 1)[0]
    reg = _registry()
    if name not in reg:
        raise ValueError(f"unknown environment {env_id!r} (native: {', '.join(available())})")
    key = (name, tuple(sorted((k, repr(v)) for k, v in kwargs.items())))
    if key not in _CACHE:
        _CACHE[key] = reg[name](**kwargs)
    return _CACHE[key]
