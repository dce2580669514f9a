"""RL rollout records, token alignment, packing and collation.

``RLExample`` is the rollout wire record shared by the orchestrator and the
trainer (same fields as the reference's data/rl.py:95).  A record carries the
exact token ids the generator produced (``input_ids`` = prompt + completion,
``loss_mask`` over completion tokens) plus the generator's log-probs and,
optionally, the sampling support set (``sampling_mask``) of each sampled
token.

Packing: samples are bin-packed first-fit-decreasing into ``seq_len`` rows
(data/rl.py:301), rows are spread over data-parallel ranks so every rank gets
a similar attention + matmul cost (data/rl.py:357), and each rank's rows are
collated into packed micro-batches with ``cu_seqlens``.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any

import torch

from ..trainer.engine import PackedBatch


@dataclass
class RLExample:
    prompt: list[dict[str, str]]
    completion: list[dict[str, str]]
    advantage: float | list[float] | None
    reward: float | None
    input_ids: list[int] | None = None
    target_ids: list[int] | None = None
    loss_mask: list[bool] | None = None
    target_completion: list[dict[str, str]] | None = None
    inference_logprobs: list[float] | None = None
    teacher_logprobs: list[float] | None = None
    temperatures: float | list[float] | None = None
    ce_weight: float | list[float] | None = None
    ref_kl_weight: float | list[float] | None = None
    sampling_mask: list[list[int]] | None = None
    tools: list[dict[str, Any]] | None = None
    chat_template_kwargs: dict[str, Any] | None = None
    metadata: dict[str, Any] | None = None
    source: str = "dataset"
    mm_kwargs: dict[str, Any] | None = None


# record field -> data-config attribute naming its column in rollout files
_COLUMNS = {"advantage": "advantage_column", "reward": "reward_column",
            "inference_logprobs": "inference_logprobs_column", "teacher_logprobs": "teacher_logprobs_column",
            "sampling_mask": "sampling_mask_column", "temperatures": "temperature_column",
            "ce_weight": "ce_weight_column", "ref_kl_weight": "ref_kl_weight_column", "metadata": "metadata_column",
            "tools": "tools_column", "chat_template_kwargs": "chat_template_kwargs_column"}


def _renames(data_cfg) -> dict[str, str]:
    """Field -> column for the columns ``data_cfg`` renames away from the
    schema defaults (the default names are the fields' own)."""
    if data_cfg is None:
        return {}
    fields = type(data_cfg).model_fields
    out = {}
    for field, attr in _COLUMNS.items():
        if attr in fields and getattr(data_cfg, attr) != fields[attr].default:
            out[field] = getattr(data_cfg, attr)
    return out


def example_from_payload(p: dict[str, Any], data_cfg=None) -> RLExample:
    """A rollout record from its JSON row; ``data_cfg`` (the ``data``
    section) maps renamed columns (``data.advantage_column`` ...) back."""
    ren = _renames(data_cfg)
    if ren:
        p = dict(p)
        for field, col in ren.items():
            if col in p:
                p[field] = p.pop(col)
    known = set(RLExample.__dataclass_fields__)
    return RLExample(**{k: v for k, v in p.items() if k in known})


def example_to_payload(e: RLExample, data_cfg=None) -> dict[str, Any]:
    d = asdict(e)
    for field, col in _renames(data_cfg).items():
        if field in d:
            d[col] = d.pop(field)
    return d


@dataclass
class RLSample:
    """One sequence in trainer layout: position t predicts token t+1."""

    input_ids: torch.Tensor  # [L] int64
    loss_mask: torch.Tensor  # [L] bool (target positions)
    inference_logprobs: torch.Tensor  # [L] float
    teacher_logprobs: torch.Tensor | None
    advantages: torch.Tensor  # [L]
    temperature: float
    ce_weights: torch.Tensor | None
    ref_kl_weights: torch.Tensor | None
    sampling_mask: list[list[int]] | None  # per target position (only masked ones used)
    reward: float = 0.0
    has_inference: torch.Tensor | None = None  # [L] bool: target positions with a recorded inference log-prob


def _per_token(v, n: int, default: float | None) -> torch.Tensor | None:
    if v is None:
        return None if default is None else torch.full((n,), float(default))
    if isinstance(v, (int, float)):
        return torch.full((n,), float(v))
    t = torch.tensor(v, dtype=torch.float32)
    if t.numel() != n:
        raise ValueError(f"per-token field has {t.numel()} values for {n} trainable tokens")
    return t


def sample_from_example(e: RLExample, default_temperature: float = 1.0) -> RLSample:
    """Align a pretokenised record to trainer positions.

    ``loss_mask[i]`` marks whether token i of ``input_ids`` is trainable; the
    log-prob of token i is predicted at position i-1.  Per-token fields (log
    probs, advantages, weights) list one value per trainable token in order.
    """
    if e.input_ids is None or e.loss_mask is None:
        raise ValueError("RL training records must be pretokenised (input_ids and loss_mask)")
    ids = torch.tensor(e.input_ids, dtype=torch.long)
    tok_mask = torch.tensor(e.loss_mask, dtype=torch.bool)
    if tok_mask.numel() != ids.numel():
        raise ValueError("loss_mask must align with input_ids")
    L = ids.numel()
    pos_mask = torch.zeros(L, dtype=torch.bool)
    pos_mask[:-1] = tok_mask[1:]
    n = int(pos_mask.sum())
    idx = pos_mask.nonzero().flatten()

    def scatter(vals: torch.Tensor | None) -> torch.Tensor | None:
        if vals is None:
            return None
        out = torch.zeros(L, dtype=torch.float32)
        out[idx] = vals
        return out

    ilp = scatter(_per_token(e.inference_logprobs, n, 0.0))
    tlp = scatter(_per_token(e.teacher_logprobs, n, None)) if e.teacher_logprobs is not None else None
    adv = scatter(_per_token(e.advantage, n, 0.0))
    ce = scatter(_per_token(e.ce_weight, n, None)) if e.ce_weight is not None else None
    rk = scatter(_per_token(e.ref_kl_weight, n, None)) if e.ref_kl_weight is not None else None
    temp = e.temperatures if isinstance(e.temperatures, (int, float)) else (e.temperatures[0] if e.temperatures else default_temperature)
    sm = None
    if e.sampling_mask is not None:
        if len(e.sampling_mask) != n:
            raise ValueError("sampling_mask must list one support set per trainable token")
        sm = [[] for _ in range(L)]
        for k, i in enumerate(idx.tolist()):
            sm[i] = list(e.sampling_mask[k])
    has_inf = pos_mask.clone() if e.inference_logprobs is not None else torch.zeros(L, dtype=torch.bool)
    return RLSample(ids, pos_mask, ilp, tlp, adv, float(temp), ce, rk, sm, float(e.reward or 0.0), has_inf)


# -------------------------------------------------------------------- packing
def pack_ffd(lengths: list[int], capacity: int) -> list[list[int]]:
    """First-fit-decreasing bin packing; returns bins of sample indices."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    bins: list[list[int]] = []
    room: list[int] = []
    for i in order:
        L = lengths[i]
        if L > capacity:
            raise ValueError(f"sample of {L} tokens exceeds data.seq_len={capacity}")
        for b, r in enumerate(room):
            if r >= L:
                bins[b].append(i)
                room[b] -= L
                break
        else:
            bins.append([i])
            room.append(capacity - L)
    return bins


def bin_cost(lengths: list[int], hidden: int = 4096) -> float:
    """Relative cost of a packed row: matmul ~ tokens * hidden, attention ~ sum L^2."""
    return sum(L * hidden + L * L for L in lengths)


def distribute_bins(bins: list[list[int]], lengths: list[int], world: int) -> list[list[list[int]]]:
    """Greedy longest-processing-time assignment of bins to ranks; every rank
    gets the same number of rows (empty rows pad short ranks)."""
    costs = [bin_cost([lengths[i] for i in b]) for b in bins]
    order = sorted(range(len(bins)), key=lambda b: -costs[b])
    per_rank: list[list[list[int]]] = [[] for _ in range(world)]
    load = [0.0] * world
    for b in order:
        r = min(range(world), key=lambda k: (load[k], len(per_rank[k])))
        per_rank[r].append(bins[b])
        load[r] += costs[b]
    n = max(len(x) for x in per_rank) if per_rank else 0
    for x in per_rank:
        while len(x) < n:
            x.append([])
    return per_rank


@dataclass
class RLPackedBatch:
    base: PackedBatch
    inference_logprobs: torch.Tensor
    teacher_logprobs: torch.Tensor | None
    advantages: torch.Tensor
    loss_mask: torch.Tensor  # bool
    temperature: float
    ce_weights: torch.Tensor | None
    ref_kl_weights: torch.Tensor | None
    sampling_mask: list[list[int]] | None
    num_samples: int
    rewards: list[float] = field(default_factory=list)
    has_inference: torch.Tensor | None = None  # bool [T]

    def to(self, device) -> "RLPackedBatch":
        mv = lambda t: None if t is None else t.to(device, non_blocking=True)  # noqa: E731
        return RLPackedBatch(self.base.to(device), mv(self.inference_logprobs), mv(self.teacher_logprobs),
                             mv(self.advantages), mv(self.loss_mask), self.temperature, mv(self.ce_weights),
                             mv(self.ref_kl_weights), self.sampling_mask, self.num_samples, self.rewards,
                             mv(self.has_inference))

    def missing_inference(self) -> torch.Tensor:
        """Target positions whose RL or reference-KL term needs an inference
        log-prob that the record did not carry (host tensors)."""
        need = self.loss_mask.clone()
        if self.ce_weights is not None:  # cross-entropy-only tokens use no inference log-prob
            need &= ~((self.ce_weights != 0) & (self.advantages == 0))
        if self.ref_kl_weights is not None:
            need |= self.loss_mask & (self.ref_kl_weights != 0)
        has = self.has_inference if self.has_inference is not None else torch.ones_like(need)
        return need & ~has


def collate(samples: list[RLSample], pad_token: int = 0) -> RLPackedBatch:
    if not samples:
        # an empty padding row: one dummy token, no loss
        ids = torch.tensor([pad_token])
        z = torch.zeros(1)
        base = PackedBatch(ids, torch.zeros(1, dtype=torch.int32), torch.tensor([0, 1], dtype=torch.int32), 1,
                           torch.full((1,), -100), z.clone())
        return RLPackedBatch(base, z.clone(), None, z.clone(), torch.zeros(1, dtype=torch.bool), 1.0, None, None, None, 0,
                             [], torch.zeros(1, dtype=torch.bool))
    temps = {s.temperature for s in samples}
    if len(temps) > 1:
        raise ValueError("one packed micro-batch must use a single sampling temperature")
    ids = torch.cat([s.input_ids for s in samples])
    lens = [s.input_ids.numel() for s in samples]
    cu = torch.zeros(len(samples) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lens, dtype=torch.int32).cumsum(0)
    pos = torch.cat([torch.arange(L, dtype=torch.int32) for L in lens])
    tg = []
    for s in samples:
        t = torch.full_like(s.input_ids, -100)
        t[:-1] = s.input_ids[1:]
        tg.append(torch.where(s.loss_mask, t, torch.full_like(t, -100)))
    mask = torch.cat([s.loss_mask for s in samples])
    cat = lambda f: None if getattr(samples[0], f) is None else torch.cat([getattr(s, f) for s in samples])  # noqa: E731
    sm = None
    if any(s.sampling_mask is not None for s in samples):
        sm = []
        for s in samples:
            sm += s.sampling_mask if s.sampling_mask is not None else [[] for _ in range(s.input_ids.numel())]
    base = PackedBatch(ids, pos, cu, max(lens), torch.cat(tg), mask.float())
    has = torch.cat([s.has_inference if s.has_inference is not None else s.loss_mask for s in samples])
    return RLPackedBatch(base, cat("inference_logprobs"), cat("teacher_logprobs"), cat("advantages"), mask,
                         samples[0].temperature, cat("ce_weights"), cat("ref_kl_weights"), sm, len(samples),
                         [s.reward for s in samples], has)


def make_rank_batches(examples: list[RLExample], seq_len: int, dp_rank: int, dp_world: int,
                      default_temperature: float = 1.0) -> list[RLPackedBatch]:
    samples = [sample_from_example(e, default_temperature) for e in examples]
    lengths = [s.input_ids.numel() for s in samples]
    # the LM-head kernels take one temperature per micro-batch: rollouts sampled
    # at different temperatures (per-environment sampling) are packed apart
    by_temp: dict[float, list[int]] = {}
    for i, smp in enumerate(samples):
        by_temp.setdefault(float(smp.temperature), []).append(i)
    bins = []
    for idx in by_temp.values():
        bins += [[idx[j] for j in b] for b in pack_ffd([lengths[i] for i in idx], seq_len)]
    mine = distribute_bins(bins, lengths, dp_world)[dp_rank]
    return [collate([samples[i] for i in b]) for b in mine]
