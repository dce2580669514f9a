"""Multi-turn / tool rollouts to training rows (reference
orchestrator/agent_trajectory.py:9-408).

An agent episode arrives as token segments, one per model call: the prompt
tokens the model saw and the tokens it produced (with their sampling
log-probs).  ``merge_token_segments`` stitches consecutive calls into one
training row when the later prompt starts with the earlier row's full token
sequence (prompt + outputs): the new prompt suffix (tool responses, user
turns) is appended untrained, the new outputs trained.  A call whose prompt
does not extend any open row (the context was rewritten, a sub-agent
branch) starts a new row.  Output tokens carry their inference log-probs;
every other position carries 0 and is masked out.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


@dataclass
class TokenSegment:
    prompt_ids: list[int]
    output_ids: list[int]
    output_logprobs: list[float]
    output_loss_mask: list[bool] | None = None  # default: every output token trained
    turn_id: str | None = None
    metadata: dict[str, Any] | None = None

    def __post_init__(self):
        self.prompt_ids = [int(t) for t in self.prompt_ids]
        self.output_ids = [int(t) for t in self.output_ids]
        self.output_logprobs = [float(x) for x in self.output_logprobs]
        if len(self.output_logprobs) != len(self.output_ids):
            raise ValueError(f"output_logprobs ({len(self.output_logprobs)}) must align with output_ids "
                             f"({len(self.output_ids)})")
        if self.output_loss_mask is None:
            self.output_loss_mask = [True] * len(self.output_ids)
        elif len(self.output_loss_mask) != len(self.output_ids):
            raise ValueError("output_loss_mask must align with output_ids")


@dataclass
class TrajectorySample:
    input_ids: list[int] = field(default_factory=list)
    loss_mask: list[bool] = field(default_factory=list)
    inference_logprobs: list[float] = field(default_factory=list)
    turn_ids: list[str | None] = field(default_factory=list)
    segments: list[int] = field(default_factory=list)  # indices of the merged segments

    def append(self, ids: list[int], trained: list[bool], lps: list[float], turn: str | None) -> None:
        self.input_ids += ids
        self.loss_mask += trained
        self.inference_logprobs += lps
        self.turn_ids += [turn] * len(ids)


def merge_token_segments(segments: list[TokenSegment], *, mask_outputs: bool = False) -> list[TrajectorySample]:
    """Rows of merged segments in order of first appearance.  ``mask_outputs``
    keeps every output untrained (scoring-only episodes)."""
    rows: list[TrajectorySample] = []
    for i, seg in enumerate(segments):
        trained = [m and not mask_outputs for m in seg.output_loss_mask]
        target = None
        for row in rows:
            n = len(row.input_ids)
            if len(seg.prompt_ids) >= n and seg.prompt_ids[:n] == row.input_ids and \
                    (seg.metadata or {}).get("media_fingerprint") == _fp(segments, row):
                target = row
                break
        if target is None:
            target = TrajectorySample()
            target.append(seg.prompt_ids, [False] * len(seg.prompt_ids), [0.0] * len(seg.prompt_ids), seg.turn_id)
            rows.append(target)
        else:
            extra = seg.prompt_ids[len(target.input_ids):]
            target.append(extra, [False] * len(extra), [0.0] * len(extra), seg.turn_id)
        target.append(seg.output_ids, trained, seg.output_logprobs, seg.turn_id)
        target.segments.append(i)
    return [r for r in rows if r.input_ids]


def _fp(segments, row: TrajectorySample):
    return (segments[row.segments[-1]].metadata or {}).get("media_fingerprint") if row.segments else None


def to_rl_example(sample: TrajectorySample, reward: float | None = None, advantage: float | None = None,
                  temperature: float = 1.0, metadata: dict | None = None):
    """A merged row as an ``RLExample`` for the trainer."""
    from ..data.rl import RLExample

    return RLExample(prompt=[], completion=[], advantage=advantage, reward=reward, input_ids=sample.input_ids,
                     loss_mask=sample.loss_mask, inference_logprobs=sample.inference_logprobs,
                     temperatures=temperature, metadata={"turn_ids": sample.turn_ids, **(metadata or {})},
                     source="agent")
