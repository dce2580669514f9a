"""Optimizers and LR schedules over the flat sharded parameter store.

``build_optimizer`` maps ``optim.type`` to an update rule applied to the
local fp32 master shard after the gradient reduce-scatter:

* ``adamw`` / ``adam`` — the fused AdamW kernel (``adam`` = no decay);
* ``sgd`` — momentum SGD (optionally Nesterov) with decoupled decay;
* ``sign_sgd`` — sign of the gradient times lr (trainer/optim.py:30);
* ``muon`` — Newton–Schulz orthogonalised momentum for 2-D weights (5
  quintic iterations on the Gram of the smaller side), AdamW for the rest
  (trainer/optim.py:67-188).  Muon needs whole matrices, so with data
  parallelism the rank that owns a matrix's first element updates it from the
  all-gathered gradient.
* 8-bit variants are served by the fp32 AdamW (bitsandbytes is not part of
  this framework).

Schedules: constant, linear, cosine, sqrt with warmup (trainer/optim.py:513-832).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops
from ..models.params import FlatParams
from ..parallel.zero import AdamWHyper, NonFiniteGradientError, ShardedAdamW


def lr_at(step: int, base_lr: float, total_steps: int, sched) -> float:
    """LR for optimizer step ``step`` (0-based) under a SchedulerConfig."""
    warm = sched.warmup_steps if sched.warmup_steps is not None else int(round(sched.warmup_ratio * total_steps))
    min_lr = sched.min_lr
    if sched.min_lr_factor is not None:
        min_lr = base_lr * sched.min_lr_factor
    if warm > 0 and step < warm:
        return base_lr * (step + 1) / warm
    if sched.type == "constant":
        return base_lr
    decay_total = sched.decay_steps if sched.decay_steps is not None else max(1, int(round((total_steps - warm) * sched.decay_ratio)))
    decay_start = total_steps - decay_total if sched.decay_steps is None else warm
    decay_start = max(decay_start, warm)
    if step < decay_start:
        return base_lr
    t = min(1.0, (step - decay_start + 1) / max(1, decay_total))
    if sched.type == "linear":
        f = 1.0 - t
    elif sched.type == "cosine":
        f = 0.5 * (1.0 + math.cos(math.pi * t))
    elif sched.type == "sqrt":
        f = 1.0 - math.sqrt(t)
    else:
        raise ValueError(f"unknown scheduler {sched.type}")
    return min_lr + (base_lr - min_lr) * f


def newton_schulz5(g: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Quintic Newton–Schulz iteration towards the orthogonal polar factor
    (coefficients a, b, c = 3.4445, -4.7750, 2.0315 from the Muon write-up)."""
    a, b, c = 3.4445, -4.7750, 2.0315
    x = g.float()
    transposed = x.shape[0] > x.shape[1]
    if transposed:
        x = x.t()
    x = x / (x.norm() + eps)
    for _ in range(steps):
        A = x @ x.t()
        B = b * A + c * (A @ A)
        x = a * x + B @ x
    return x.t() if transposed else x


class FlatOptimizer:
    """Common driver: reduce-scatter, norm/clip, per-type update, all-gather."""

    def __init__(self, flat: FlatParams, cfg, max_grad_norm: float, dp_group=None, dp_world: int = 1, fabric=None,
                 expert_flat: FlatParams | None = None, ep_dp_group=None, ep_dp_world: int = 1):
        self.flat = flat
        self.cfg = cfg
        self.type = cfg.type
        self.group = dp_group
        self.world = dp_world
        hyper = AdamWHyper(
            lr=cfg.lr, betas=(cfg.betas1, cfg.betas2), eps=1e-8,
            weight_decay=0.0 if cfg.type in ("adam", "adam_8bit") else cfg.weight_decay,
            max_grad_norm=max_grad_norm,
        )
        if expert_flat is not None:
            # expert parallelism: dense + expert stores, one global clip
            if cfg.type not in ("adamw", "adam", "adamw_8bit", "adam_8bit"):
                raise NotImplementedError("expert parallelism supports the AdamW family only")
            from ..parallel.zero import CompositeAdamW

            self.adamw = CompositeAdamW([ShardedAdamW(flat, hyper, dp_group, dp_world),
                                         ShardedAdamW(expert_flat, hyper, ep_dp_group, ep_dp_world)],
                                        distributed=dist.is_initialized() and dp_world > 1)
        elif fabric is not None and cfg.type in ("adamw", "adam", "adamw_8bit", "adam_8bit"):
            from ..parallel.zero import FusedShardedAdamW

            self.adamw = FusedShardedAdamW(flat, hyper, fabric)  # fused peer-memory RS + AdamW + AG
        else:
            self.adamw = ShardedAdamW(flat, hyper, dp_group, dp_world,
                                      offload=bool(getattr(cfg, "cpu_offload", False)))
        self.momentum_buf = None

    @property
    def step_count(self) -> int:
        return self.adamw.step_count

    def step(self, lr: float) -> dict[str, float]:
        if self.type in ("adamw", "adam", "adamw_8bit", "paged_adamw_8bit", "adam_8bit"):
            return self.adamw.step(lr)
        return self._step_other(lr)

    @torch.no_grad()
    def _step_other(self, lr: float) -> dict[str, float]:
        a = self.adamw
        flat = self.flat
        g = a.reduce_grads()
        a.stats.zero_()
        ops.sumsq_(g, a.stats)
        if self.world > 1:
            dist.all_reduce(a.stats, group=self.group)
        norm_sq, bad = a.stats.tolist()
        if bad > 0:
            raise NonFiniteGradientError(f"non-finite gradients detected ({int(bad)} elements)")
        norm = norm_sq**0.5
        factor = min(1.0, a.h.max_grad_norm / (norm + 1e-6)) if a.h.max_grad_norm > 0 else 1.0
        a.step_count += 1
        gs = g * factor
        p = flat.master
        wd = self.cfg.weight_decay
        if self.type == "sign_sgd":
            if wd > 0:
                p.mul_(1 - lr * wd)
            p.add_(gs.sign(), alpha=-lr)
        elif self.type == "sgd":
            if self.momentum_buf is None:
                self.momentum_buf = torch.zeros_like(p)
            buf = self.momentum_buf.mul_(self.cfg.momentum).add_(gs)
            upd = gs.add(buf, alpha=self.cfg.momentum) if self.cfg.nesterov else buf
            if wd > 0:
                p.mul_(1 - lr * wd)
            p.add_(upd, alpha=-lr)
        elif self.type == "muon":
            self._muon(gs, lr)
        else:
            raise ValueError(f"unsupported optimizer {self.type}")
        compute = flat.compute.detach()
        p16 = compute[flat.shard_slice]
        p16.copy_(p.to(p16.dtype))
        if self.world > 1:
            dist.all_gather_into_tensor(compute, p16.clone(), group=self.group)
        flat.zero_grad()
        return {"grad_norm": norm, "clip_factor": factor}

    def _muon(self, gs: torch.Tensor, lr: float) -> None:
        """Muon on 2-D weight shards that lie entirely inside this rank's shard;
        AdamW-style update on everything else."""
        flat = self.flat
        if self.momentum_buf is None:
            self.momentum_buf = torch.zeros_like(flat.master)
        mu = self.cfg.muon_momentum
        buf = self.momentum_buf.mul_(mu).add_(gs)
        lo = flat.dp_rank * flat.shard_numel
        hi = lo + flat.shard_numel
        handled = torch.zeros(flat.shard_numel, dtype=torch.bool, device=gs.device)
        for s in flat.specs:
            off, n = flat.offsets[s.name]
            if len(s.shape) != 2 or off < lo or off + n > hi or s.name in ("embed", "lm_head"):
                continue
            a, b = off - lo, off - lo + n
            u = (gs[a:b] + mu * buf[a:b]) if self.cfg.nesterov else buf[a:b]
            o = newton_schulz5(u.view(s.shape))
            scale = max(1.0, s.shape[0] / s.shape[1]) ** 0.5
            if self.cfg.weight_decay > 0:
                flat.master[a:b].mul_(1 - lr * self.cfg.weight_decay)
            flat.master[a:b].add_(o.reshape(-1), alpha=-lr * scale)
            handled[a:b] = True
        rest = ~handled
        if rest.any():
            m = flat.exp_avg
            v = flat.exp_avg_sq
            b1, b2 = self.cfg.betas1, self.cfg.betas2
            t = self.adamw.step_count
            m[rest] = b1 * m[rest] + (1 - b1) * gs[rest]
            v[rest] = b2 * v[rest] + (1 - b2) * gs[rest] ** 2
            den = (v[rest] / (1 - b2**t)).sqrt() + 1e-8
            flat.master[rest] -= lr * (m[rest] / (1 - b1**t)) / den

    def state_dict(self) -> dict:
        sd = dict(self.adamw.state_dict())
        sd["type"] = self.type
        if self.momentum_buf is not None:
            sd["momentum"] = self.momentum_buf
        return sd

    def load_state_dict(self, sd: dict) -> None:
        self.adamw.load_state_dict(sd)
        if "momentum" in sd:
            self.momentum_buf = sd["momentum"].clone()
