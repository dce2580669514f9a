"""Multi-turn / tool rollouts to training rows (reference
orchestrator/agent_trajectory.py:9-408).

An agent episode arrives as token segments, one per model call: the prompt
tokens the model saw and the tokens it produced (with their sampling
log-probs).  ``merge_token_segments`` stitches consecutive calls into one
training row when the later prompt starts with the earlier row's full token
sequence (prompt + outputs): the new prompt suffix (tool responses, user
turns) is appended untrained, the new outputs trained.  A call whose prompt
does not extend any open row is matched against it once more as a
re-rendered history (chat templates that re-render earlier assistant turns,
e.g. without thinking framing): if every earlier output of the row occurs in
the new prompt in order at exactly one set of non-overlapping places, the
row is rebuilt on the new prompt with those places trained; with no or
several placements the call starts a new row (a rewritten context, a
sub-agent branch).  Output tokens carry their inference log-probs and
sampling masks; every other position carries 0 / None and is masked out.
Rows are aligned to ``input_ids`` (the trainer shifts them to targets).
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
    output_sampling_mask: list[list[int]] | None = None  # per output token: the sampler's support

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
        if self.output_sampling_mask is not None and len(self.output_sampling_mask) != len(self.output_ids):
            raise ValueError("output_sampling_mask must align with output_ids")


@dataclass
class _Output:
    seg: int
    ids: list[int]
    trained: list[bool]
    lps: list[float]
    masks: list[list[int] | None]
    turn: str | None


@dataclass
class TrajectorySample:
    input_ids: list[int] = field(default_factory=list)
    loss_mask: list[bool] = field(default_factory=list)
    inference_logprobs: list[float] = field(default_factory=list)
    turn_ids: list[str | None] = field(default_factory=list)
    sampling_masks: list[list[int] | None] = field(default_factory=list)
    segments: list[int] = field(default_factory=list)  # indices of the merged segments
    temperature: float = 1.0
    outputs: list[_Output] = field(default_factory=list, repr=False)

    @property
    def temperatures(self) -> list[float]:
        return [self.temperature] * len(self.input_ids)

    @property
    def terminal_segment_index(self) -> int:
        return self.segments[-1]

    def append(self, ids: list[int], trained: list[bool], lps: list[float], turn: str | None,
               masks: list | None = None) -> None:
        self.input_ids += ids
        self.loss_mask += trained
        self.inference_logprobs += lps
        self.turn_ids += [turn] * len(ids)
        self.sampling_masks += masks if masks is not None else [None] * len(ids)

    def add_output(self, o: _Output) -> None:
        self.append(o.ids, o.trained, o.lps, o.turn, o.masks)
        self.outputs.append(o)

    def rebase(self, prompt: list[int], starts: list[int], turn: str | None) -> None:
        """Rebuild on a re-rendered prompt; earlier outputs sit at ``starts``."""
        self.input_ids = list(prompt)
        self.loss_mask = [False] * len(prompt)
        self.inference_logprobs = [0.0] * len(prompt)
        self.turn_ids = [turn] * len(prompt)
        self.sampling_masks = [None] * len(prompt)
        for o, a in zip(self.outputs, starts):
            b = a + len(o.ids)
            self.loss_mask[a:b] = o.trained
            self.inference_logprobs[a:b] = o.lps
            self.turn_ids[a:b] = [o.turn] * len(o.ids)
            self.sampling_masks[a:b] = o.masks


def _unique_ordered_output_matches(outputs: list[list[int]], prompt: list[int]) -> list[int] | None:
    """Start offsets of ``outputs`` as ordered, non-overlapping sub-sequences
    of ``prompt`` when exactly one such placement exists, else None.  A
    count-capped dynamic programme: ways[j][i] = placements of outputs j..
    inside prompt[i:], saturating at 2."""
    m, n = len(outputs), len(prompt)
    if any(not o for o in outputs):
        return None
    ways = [[0] * (n + 2) for _ in range(m + 1)]
    ways[m] = [1] * (n + 2)

    def hit(j: int, i: int) -> bool:
        o = outputs[j]
        return i + len(o) <= n and prompt[i : i + len(o)] == o

    for j in range(m - 1, -1, -1):
        L, row, nxt = len(outputs[j]), ways[j], ways[j + 1]
        for i in range(n, -1, -1):
            w = row[i + 1] if i < n else 0
            if hit(j, i):
                w += nxt[i + L]
            row[i] = 2 if w > 2 else w
    if ways[0][0] != 1:
        return None
    starts, i = [], 0
    for j in range(m):
        while not (hit(j, i) and ways[j + 1][i + len(outputs[j])] >= 1):
            i += 1
        starts.append(i)
        i += len(outputs[j])
    return starts


def merge_token_segments(segments: list[TokenSegment], *, mask_outputs: bool = False,
                         temperature: float = 1.0) -> list[TrajectorySample]:
    """Rows of merged segments in order of first appearance.  ``mask_outputs``
    keeps every output untrained (scoring-only episodes)."""
    rows: list[TrajectorySample] = []
    for i, seg in enumerate(segments):
        out = _Output(i, seg.output_ids, [m and not mask_outputs for m in seg.output_loss_mask], seg.output_logprobs,
                      list(seg.output_sampling_mask) if seg.output_sampling_mask is not None
                      else [None] * len(seg.output_ids), seg.turn_id)
        fp = (seg.metadata or {}).get("media_fingerprint")
        target = None
        for row in rows:
            if fp != _fp(segments, row):
                continue
            n = len(row.input_ids)
            if len(seg.prompt_ids) >= n and seg.prompt_ids[:n] == row.input_ids:
                extra = seg.prompt_ids[n:]
                row.append(extra, [False] * len(extra), [0.0] * len(extra), seg.turn_id)
                target = row
                break
            starts = _unique_ordered_output_matches([o.ids for o in row.outputs], seg.prompt_ids)
            if row.outputs and starts is not None:
                row.rebase(seg.prompt_ids, starts, seg.turn_id)
                target = row
                break
        if target is None:
            target = TrajectorySample(temperature=temperature)
            target.append(seg.prompt_ids, [False] * len(seg.prompt_ids), [0.0] * len(seg.prompt_ids), seg.turn_id)
            rows.append(target)
        target.add_output(out)
        target.segments.append(i)
    return [r for r in rows if r.input_ids]


def _fp(segments, row: TrajectorySample):
    return (segments[row.segments[-1]].metadata or {}).get("media_fingerprint") if row.segments else None


def to_rl_example(sample: TrajectorySample, reward: float | None = None, advantage: float | None = None,
                  temperature: float | None = None, metadata: dict | None = None):
    """A merged row as an ``RLExample`` for the trainer."""
    from ..data.rl import RLExample

    # RLExample lists per-token fields once per trainable token (token 0 has no
    # predicting position and is never trained)
    keep = [i for i in range(1, len(sample.input_ids)) if sample.loss_mask[i]]
    mask = [False] + [bool(m) for m in sample.loss_mask[1:]]
    masks = [sample.sampling_masks[i] for i in keep]
    use_masks = any(m is not None for m in masks)
    return RLExample(prompt=[], completion=[], advantage=advantage, reward=reward, input_ids=sample.input_ids,
                     loss_mask=mask, inference_logprobs=[sample.inference_logprobs[i] for i in keep],
                     temperatures=sample.temperature if temperature is None else temperature,
                     sampling_mask=[m if m is not None else [] for m in masks] if use_masks else None,
                     metadata={"turn_ids": sample.turn_ids, **(metadata or {})}, source="agent")
