"""LR schedules: ``lr_at`` (closed form) against torch's own schedulers
chained the way the reference builds them (trainer/optim.py:513-832 of the
reference: LinearLR warmup from the floor factor, hold, LinearLR / cosine /
sqrt decay), step by step over whole runs; plus the reference's pinned
constant-with-warmup case."""

import math

import pytest
import torch
from torch.optim.lr_scheduler import ConstantLR, CosineAnnealingLR, LambdaLR, LinearLR, SequentialLR

from wavelet_b200.configs.config import SchedulerConfig
from wavelet_b200.trainer.optim import lr_at

LR = 3e-4


def _floor(c):
    if c.min_lr_factor is not None:
        return c.min_lr_factor
    return c.min_lr / LR if c.min_lr > 0 else 1e-8


def _torch_chain(c: SchedulerConfig, T: int):
    opt = torch.optim.SGD([torch.nn.Parameter(torch.zeros(1))], lr=LR)
    W = c.warmup_steps if c.warmup_steps is not None else int(T * c.warmup_ratio)
    D = c.decay_steps if c.decay_steps is not None else max(int(T * c.decay_ratio) - W, 1)
    f, eff = _floor(c), max(T - 1, 1)
    parts, marks = [], []

    def warm(w):
        if w > 0:
            parts.append(LinearLR(opt, start_factor=f, end_factor=1.0, total_iters=w))
            marks.append(w)

    if c.type == "constant":
        W = min(W, T)
        if W == 0:
            return opt, ConstantLR(opt, factor=1.0)
        warm(W)
        parts.append(LinearLR(opt, 1.0, 1.0, total_iters=max(T - W, 1)))
    elif c.type == "linear":
        W = min(W, T)
        D = max(min(D, eff), 1)
        if T - W > 0:
            D = min(D, T - W)
        warm(W)
        start = min(T - D, eff)
        if start >= W:
            if start - W > 0:
                parts.append(LinearLR(opt, 1.0, 1.0, total_iters=start - W))
                marks.append(start)
            parts.append(LinearLR(opt, 1.0, f, total_iters=max(D - 1, 1)))
    elif c.type == "cosine":
        warm(W)
        parts.append(CosineAnnealingLR(opt, T_max=min(max(eff - W, 1), D), eta_min=max(c.min_lr, f * LR)))
    else:
        W = W
        warm(W)
        post = max(T - W - 1, 1)
        span = min(max(D, 1), post)

        def fac(t):
            d = t - (post - span)
            return 1.0 if d <= 0 else f + (1 - f) * math.sqrt(max(1 - min(d / span, 1.0), 0.0))

        parts.append(LambdaLR(opt, fac))
    marks = marks[: len(parts) - 1]
    return opt, parts[0] if len(parts) == 1 else SequentialLR(opt, parts, milestones=marks)


CASES = [
    dict(type="constant", warmup_steps=10, min_lr_factor=0.1),
    dict(type="constant"),
    dict(type="constant", warmup_ratio=0.1, min_lr=1e-5),
    dict(type="linear", warmup_steps=5),
    dict(type="linear", warmup_steps=5, decay_steps=20, min_lr_factor=0.1),
    dict(type="linear", decay_ratio=0.5, min_lr=3e-5),
    dict(type="cosine", warmup_steps=8, min_lr_factor=0.05),
    dict(type="cosine", warmup_ratio=0.2, min_lr=1e-6),
    dict(type="sqrt", warmup_steps=4, decay_steps=30, min_lr_factor=0.1),
    dict(type="sqrt", warmup_ratio=0.1),
]


@pytest.mark.parametrize("kw", CASES, ids=lambda kw: "-".join(f"{k}={v}" for k, v in kw.items()))
@pytest.mark.parametrize("T", [60, 7])
def test_closed_form_matches_torch_chain(kw, T):
    c = SchedulerConfig(**kw)
    opt, sch = _torch_chain(c, T)
    for k in range(T):
        want = opt.param_groups[0]["lr"]
        assert lr_at(k, LR, T, c) == pytest.approx(want, rel=1e-6, abs=1e-14), (k, kw)
        opt.step()
        sch.step()


def test_constant_warmup_then_hold_pinned():
    c = SchedulerConfig(type="constant", warmup_steps=10, min_lr_factor=0.1)
    lrs = [lr_at(k, 1e-6, 100, c) for k in range(1, 16)]  # the LR after each scheduler step
    assert lrs[0] > 1e-7 and lrs[8] < 1e-6 and lrs[9] == 1e-6 and lrs[-1] == 1e-6
    assert lr_at(0, 1e-6, 100, c) == pytest.approx(1e-7)  # warmup starts at the floor factor
