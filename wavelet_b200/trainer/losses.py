"""RL losses on the packed token layout.

Every tensor is 1-D over the packed tokens of a micro-batch ([T]); ``seg``
gives each token's sequence index (from ``cu_seqlens``).  The reference
loops over sequence spans in Python (trainer/losses.py:323-591); here every
reduction is a vectorised segment sum, with identical semantics:

* per-token component losses (``dppo``, ``ipo``, ``icepop``, ``custom`` RL
  loss; ``ce``; ``ref_kl``) from trainer / inference / teacher log-probs and
  advantages (trainer/losses.py:100-272);
* token normalisation (sum / global token count) or sequence normalisation
  (each sequence's mean, summed, / global sequence count) for the RL part;
  CE and ref-KL are token-normalised;
* metrics are per-sequence masked means, over the sequences that have
  tokens of the metric's component, averaged over those sequences, plus
  mean / median / std / min / max across them.

A ``custom`` RL loss keeps the reference's contract: it is called once per
sequence span with 1-D inputs and returns a scalar (or per-token) loss and
scalar (or ``(values, mask)``) metrics.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
from torch import Tensor


@dataclass
class LossInputs:
    trainer_logprobs: Tensor
    inference_logprobs: Tensor
    teacher_logprobs: Tensor | None
    advantages: Tensor
    loss_mask: Tensor  # bool
    loss_weights: Tensor | None = None


@dataclass
class LossOutput:
    loss: Tensor  # per-token loss vector [T] (summed by compute_loss)
    # name -> (values, mask) for the vectorised losses; a custom loss may give scalars
    metrics: dict[str, tuple[Tensor, Tensor] | Tensor] = field(default_factory=dict)


def _trust_region(inp: LossInputs, cfg, invalid, masked_high, masked_low, teacher_logprobs) -> LossOutput:
    lp, adv, mask = inp.trainer_logprobs, inp.advantages, inp.loss_mask
    keep = mask & ~invalid
    log_ratio = lp - inp.inference_logprobs
    ratio = torch.exp(torch.where(keep, log_ratio, torch.zeros_like(log_ratio)))
    with torch.no_grad():
        mismatch = torch.exp(log_ratio) - log_ratio - 1
    sadv = cfg.adv_tau * adv
    tkl = None
    if teacher_logprobs is not None:
        tkl = teacher_logprobs - lp
        sadv = sadv + cfg.teacher_tau * tkl.detach()
    pg = torch.where(keep, sadv, torch.zeros_like(sadv)) * ratio
    kl = torch.where(mask, log_ratio, torch.zeros_like(log_ratio)).square()
    per = -pg + cfg.kl_tau * kl
    if inp.loss_weights is not None:
        per = per * inp.loss_weights
    per = torch.where(mask, per, torch.zeros_like(per))
    m = {
        "mismatch_kl": (mismatch, mask),
        "masked_mismatch_kl": (mismatch, mask & invalid),
        "unmasked_mismatch_kl": (mismatch, keep),
        "is_masked": (invalid.float(), mask),
        "is_masked_low": (masked_low.float(), mask),
        "is_masked_high": (masked_high.float(), mask),
        "policy_loss": (-pg.detach(), mask),
        "kl_loss": (kl.detach(), mask),
        "advantage_mean": (adv, mask),
    }
    if tkl is not None:
        m["teacher_kl"] = (tkl.detach(), mask)
    return LossOutput(per, m)


def dppo_loss(inp: LossInputs, cfg) -> LossOutput:
    """DPPO: mask tokens whose probability moved past the advantage-signed band."""
    d = torch.exp(inp.trainer_logprobs) - torch.exp(inp.inference_logprobs)
    hi = d > cfg.dppo_mask_high
    lo = d < -cfg.dppo_mask_low
    pos = inp.advantages > 0
    return _trust_region(inp, cfg, torch.where(pos, hi, lo), pos & hi, (inp.advantages < 0) & lo, inp.teacher_logprobs)


def ipo_loss(inp: LossInputs, cfg) -> LossOutput:
    """IPO: symmetric probability trust region of width ipo_epsilon."""
    d = torch.exp(inp.trainer_logprobs) - torch.exp(inp.inference_logprobs)
    return _trust_region(inp, cfg, d.abs() > cfg.ipo_epsilon, d > cfg.ipo_epsilon, d < -cfg.ipo_epsilon, None)


def icepop_loss(inp: LossInputs, cfg) -> LossOutput:
    """IcePop: importance-ratio PG, tokens outside [ratio_low, ratio_high] dropped."""
    log_ratio = inp.trainer_logprobs - inp.inference_logprobs
    lo = torch.log(torch.tensor(cfg.ratio_low, device=log_ratio.device))
    hi = torch.log(torch.tensor(cfg.ratio_high, device=log_ratio.device))
    rej = (log_ratio.detach() < lo) | (log_ratio.detach() > hi)
    keep = inp.loss_mask & ~rej
    ratio = torch.exp(torch.where(keep, log_ratio, torch.zeros_like(log_ratio)))
    per = -keep.to(inp.advantages.dtype) * cfg.adv_tau * inp.advantages * ratio
    if inp.loss_weights is not None:
        per = per * inp.loss_weights
    mismatch = (torch.exp(log_ratio) - log_ratio - 1).detach()
    return LossOutput(per, {
        "masked_mismatch_kl": (mismatch, inp.loss_mask & rej),
        "unmasked_mismatch_kl": (mismatch, keep),
        "is_masked": (rej.float(), inp.loss_mask),
    })


def ce_loss(inp: LossInputs) -> LossOutput:
    per = -inp.trainer_logprobs
    if inp.loss_weights is not None:
        per = per * inp.loss_weights
    per = torch.where(inp.loss_mask, per, torch.zeros_like(per))
    return LossOutput(per, {"ce/nll": (-inp.trainer_logprobs.detach(), inp.loss_mask)})


def ref_kl_loss(inp: LossInputs) -> LossOutput:
    """Reverse-KL to a teacher with a one-sided probability trust region."""
    if inp.teacher_logprobs is None:
        raise ValueError("ref_kl loss requires teacher_logprobs for every weighted token.")
    log_ratio = inp.trainer_logprobs - inp.inference_logprobs
    with torch.no_grad():
        mismatch = torch.exp(log_ratio) - log_ratio - 1
    delta = torch.exp(inp.trainer_logprobs) - torch.exp(inp.inference_logprobs)
    invalid = delta < -0.2
    keep = inp.loss_mask & ~invalid
    ratio = torch.exp(torch.where(keep, log_ratio, torch.zeros_like(log_ratio)))
    tkl = inp.teacher_logprobs - inp.trainer_logprobs
    pol = -(torch.where(keep, tkl.detach(), torch.zeros_like(tkl)) * ratio)
    reg = torch.where(inp.loss_mask, log_ratio, torch.zeros_like(log_ratio)).square()
    per = pol + 1e-3 * reg
    if inp.loss_weights is not None:
        per = per * inp.loss_weights
    per = torch.where(inp.loss_mask, per, torch.zeros_like(per))
    return LossOutput(per, {
        "ref_kl/masked_mismatch_kl": (mismatch, inp.loss_mask & invalid),
        "ref_kl/unmasked_mismatch_kl": (mismatch, keep),
        "ref_kl/is_masked": (invalid.float(), inp.loss_mask),
        "ref_kl": (tkl.detach(), inp.loss_mask),
    })


LossFn = Callable[[LossInputs], LossOutput]


def setup_rl_loss_fn(cfg) -> LossFn:
    if cfg.type == "custom":
        mod, _, attr = cfg.import_path.rpartition(".")
        if not mod:
            raise ValueError("Custom loss import_path must include a module and attribute name.")
        fn = getattr(importlib.import_module(mod), attr)
        if not callable(fn):
            raise TypeError(f"Custom loss object {cfg.import_path!r} is not callable.")
        kwargs = dict(cfg.kwargs)

        def custom(inp: LossInputs) -> LossOutput:
            out = fn(inp, **kwargs)
            if not isinstance(out, LossOutput):
                raise TypeError("Custom RL loss must return LossOutput.")
            return out

        custom.per_span = True  # called once per sequence span (trainer/losses.py:433-490)
        return custom
    return {"ipo": lambda i: ipo_loss(i, cfg), "icepop": lambda i: icepop_loss(i, cfg)}.get(
        cfg.type, lambda i: dppo_loss(i, cfg))


# ------------------------------------------------------------- segmentation
def segment_ids(cu_seqlens: Tensor, T: int) -> Tensor:
    lens = (cu_seqlens[1:] - cu_seqlens[:-1]).long()
    return torch.repeat_interleave(torch.arange(len(lens), device=cu_seqlens.device), lens, output_size=T)


def seg_sum(x: Tensor, seg: Tensor, n: int) -> Tensor:
    return torch.zeros(n, device=x.device, dtype=x.dtype).index_add_(0, seg, x)


def _seq_means(values: Tensor, mask: Tensor, seg: Tensor, n: int, active: Tensor) -> Tensor:
    """Per-sequence masked means, only for sequences in ``active``."""
    num = seg_sum(torch.where(mask, values.float(), torch.zeros_like(values, dtype=torch.float32)), seg, n)
    den = seg_sum(mask.float(), seg, n).clamp_min(1.0)
    return (num / den)[active]


def component_unit_counts(loss_mask: Tensor, seg: Tensor, n: int, rl_weights=None, ce_weights=None,
                          ref_kl_weights=None, rl_normalization="token") -> dict[str, float]:
    rl_mask = loss_mask if rl_weights is None else loss_mask & (rl_weights != 0)
    if rl_normalization == "sequence":
        rl = float((seg_sum(rl_mask.float(), seg, n) > 0).sum())
    else:
        rl = float(rl_mask.sum())
    ce = float((loss_mask & (ce_weights != 0)).sum()) if ce_weights is not None else 0.0
    rk = float((loss_mask & (ref_kl_weights != 0)).sum()) if ref_kl_weights is not None else 0.0
    return {"rl": rl, "ce": ce, "ref_kl": rk}


def compute_loss(trainer_logprobs: Tensor, inference_logprobs: Tensor, teacher_logprobs: Tensor | None,
                 advantages: Tensor, loss_mask: Tensor, cfg, *, cu_seqlens: Tensor,
                 rl_weights: Tensor | None = None, ce_weights: Tensor | None = None,
                 ref_kl_weights: Tensor | None = None, component_scales: dict[str, float] | None = None,
                 rl_loss_fn: LossFn | None = None, present: dict[str, bool] | None = None, sync: bool = True,
                 seg: Tensor | None = None, n_seq: int | None = None,
                 seq_counts: Tensor | None = None) -> tuple[Tensor, dict[str, Any]]:
    """Scalar loss (already divided by the component scales) and metrics.

    ``component_scales`` are the global normalisers (token / sequence counts
    summed over data-parallel ranks and micro-batches); when absent the local
    counts are used (trainer/losses.py:520-591).

    Host-synchronisation-free use (the trainer's micro-batch loop): pass every
    component scale, ``present`` (whether the batch has any RL / CE / ref-KL
    token, known on the host before the copy) and ``sync=False``: the metrics
    are then 0-d device tensors, converted once per step by the caller.

    Context parallelism: ``seg`` / ``n_seq`` give each local token's sequence
    (local tokens of one sequence need not be contiguous) and ``seq_counts`` the
    sequence's RL-token count over all ranks (the sequence normaliser).
    """
    T = trainer_logprobs.shape[0]
    if seg is None:
        seg = segment_ids(cu_seqlens, T)
        n = cu_seqlens.numel() - 1
    else:
        n = int(n_seq)
    loss_mask = loss_mask.bool()
    fn = rl_loss_fn or setup_rl_loss_fn(cfg)
    given = dict(component_scales or {})
    if all(k in given for k in ("rl", "ce", "ref_kl")):
        scales = {k: max(float(v), 1.0) for k, v in given.items()}
    else:
        counts = component_unit_counts(loss_mask, seg, n, rl_weights, ce_weights, ref_kl_weights, cfg.normalization)
        scales = {k: max(float(v), 1.0) for k, v in counts.items()}
        scales.update({k: max(float(v), 1.0) for k, v in given.items()})

    def has(name: str, mask: Tensor) -> bool:
        if present is not None and name in present:
            return bool(present[name])
        return bool(mask.any())
    total = trainer_logprobs.sum() * 0.0
    seq_metrics: list[tuple[str, Tensor, Tensor, Tensor]] = []  # name, values, mask, active sequences
    span_metrics: dict[str, list[Tensor]] = {}

    def active_of(mask: Tensor) -> Tensor:
        return seg_sum(mask.float(), seg, n) > 0

    rl_mask = loss_mask if rl_weights is None else loss_mask & (rl_weights != 0)
    rl_present = has("rl", rl_mask)
    if rl_present and getattr(fn, "per_span", False):
        if seq_counts is not None:
            raise NotImplementedError("per-span custom RL losses need whole sequences (no context parallelism)")
        total = total + _per_span_rl(fn, trainer_logprobs, inference_logprobs, teacher_logprobs, advantages,
                                     rl_mask, rl_weights, cu_seqlens, cfg.normalization, span_metrics) / scales["rl"]
    elif rl_present:
        out = fn(LossInputs(trainer_logprobs, inference_logprobs, teacher_logprobs, advantages, rl_mask, rl_weights))
        per = out.loss
        if cfg.normalization == "sequence":
            per_seq = seg_sum(per, seg, n)
            cnt = (seq_counts.float() if seq_counts is not None else seg_sum(rl_mask.float(), seg, n)).clamp_min(1.0)
            total = total + (per_seq / cnt).sum() / scales["rl"]
        else:
            total = total + per.sum() / scales["rl"]
        act = active_of(rl_mask)
        seq_metrics += [(k, v, m, act) for k, (v, m) in out.metrics.items()]
    for name, w, f in (("ce", ce_weights, ce_loss), ("ref_kl", ref_kl_weights, ref_kl_loss)):
        if w is None:
            continue
        cm = loss_mask & (w != 0)
        if has(name, cm):
            out = f(LossInputs(trainer_logprobs, inference_logprobs, teacher_logprobs, advantages, cm, w))
            total = total + out.loss.sum() / scales[name]
            act = active_of(cm)
            seq_metrics += [(k, v, m, act) for k, (v, m) in out.metrics.items()]

    dev_metrics: dict[str, Tensor] = {}
    per_seq_values = {k: _seq_means(v.detach(), m, seg, n, act) for k, v, m, act in seq_metrics}
    per_seq_values.update({k: torch.stack(v) for k, v in span_metrics.items()})
    for k, per_seq in per_seq_values.items():
        if per_seq.numel() == 0:
            continue
        per_seq = per_seq.float()
        mean = per_seq.mean()
        dev_metrics[k] = mean
        dev_metrics[f"{k}/mean"] = mean
        dev_metrics[f"{k}/median"] = per_seq.median()
        dev_metrics[f"{k}/std"] = per_seq.std(unbiased=False) if per_seq.numel() > 1 else torch.zeros_like(mean)
        dev_metrics[f"{k}/min"] = per_seq.min()
        dev_metrics[f"{k}/max"] = per_seq.max()
    if not sync:
        return total, dev_metrics
    return total, tensors_to_floats(dev_metrics)


def tensors_to_floats(d: dict[str, Tensor]) -> dict[str, float]:
    """0-d tensors -> floats with one device-to-host transfer."""
    if not d:
        return {}
    keys = list(d)
    vals = torch.stack([d[k].detach().float().reshape(()) for k in keys]).cpu().tolist()
    return dict(zip(keys, vals))


def _per_span_rl(fn: LossFn, tl: Tensor, il: Tensor, teacher: Tensor | None, adv: Tensor, rl_mask: Tensor,
                 weights: Tensor | None, cu_seqlens: Tensor, normalization: str,
                 span_metrics: dict[str, list[Tensor]]) -> Tensor:
    """Sum of a per-span loss over the sequences with RL tokens (each span's
    loss divided by its token count under sequence normalisation)."""
    total = tl.sum() * 0.0
    bounds = cu_seqlens.tolist()
    for a, b in zip(bounds[:-1], bounds[1:]):
        m = rl_mask[a:b]
        if not bool(m.any()):
            continue
        out = fn(LossInputs(tl[a:b], il[a:b], None if teacher is None else teacher[a:b], adv[a:b], m,
                            None if weights is None else weights[a:b]))
        loss = out.loss if out.loss.dim() == 0 else out.loss.sum()
        if normalization == "sequence":
            loss = loss / m.sum().clamp_min(1)
        total = total + loss
        for k, v in out.metrics.items():
            if isinstance(v, tuple):
                vals, vm = v
                den = vm.float().sum()
                v = (torch.where(vm, vals.float(), torch.zeros_like(vals, dtype=torch.float32)).sum()
                     / den.clamp_min(1.0))
            span_metrics.setdefault(k, []).append(v.detach().float().reshape(()))
    return total
