"""Optimizers and LR schedules over the flat sharded parameter store.

``build_optimizer`` maps ``optim.type`` to an update rule applied to the
local fp32 master shard after the gradient reduce-scatter:

* ``adamw`` / ``adam`` — the fused AdamW kernel (``adam`` = no decay);
* ``sgd`` — ``torch.optim.SGD`` semantics: L2 decay added to the gradient,
  momentum, optionally Nesterov (trainer/optim.py:429-437);
* ``sign_sgd`` — sign of the gradient times lr, decoupled decay
  (trainer/optim.py:30);
* ``muon`` — for every weight of two or more dimensions except embeddings and
  the LM head: EMA momentum, Newton–Schulz orthogonalisation (5 quintic
  iterations on the Gram of the smaller side, batched over leading dims),
  rescaled to the gradient's norm; AdamW for the rest; decoupled decay on
  both (trainer/optim.py:67-188, 402-428).  Muon needs whole matrices while
  the flat store is sharded over data-parallel ranks, so the momentum
  source is all-gathered into the (then unused) replicated gradient buffer
  and each rank orthogonalises every matrix that overlaps its shard; the
  per-matrix gradient norms are summed over the shards with one small
  all-reduce.
* ``adamw_8bit`` / ``adam_8bit`` / ``paged_adamw_8bit`` — AdamW with 8-bit
  block-scaled moments (``parallel.zero.ShardedAdamW8bit``); the paged
  variant keeps the 8-bit state in CUDA managed memory (the reference uses
  bitsandbytes for these, trainer/optim.py:393-512).

Schedules: constant, linear, cosine, sqrt with warmup, as closed forms of
the reference's torch scheduler chains (trainer/optim.py:513-832).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops
from ..models.params import FlatParams
from ..parallel.zero import AdamWHyper, NonFiniteGradientError, ShardedAdamW, skip_reason


def lr_at(step: int, base_lr: float, total_steps: int, sched) -> float:
    """LR of optimizer step ``step`` (0-based): the closed form of the
    reference's torch scheduler chains (trainer/optim.py:513-832) after
    ``step`` scheduler steps.

    * floor factor f = min_lr_factor, else min_lr / lr, else 1e-8;
    * warmup over W steps (warmup_steps, else int(T * warmup_ratio)): the
      factor rises linearly from f at step 0 to 1 at step W;
    * constant: 1 after warmup;
    * linear: hold 1 until the last D steps (D = decay_steps, else
      int(T * decay_ratio) - W, clamped to [1, T - W]), then fall linearly to
      f over D - 1 steps;
    * cosine: cosine from 1 to the floor over min(T - 1 - W, D) steps after
      warmup, then stay at the floor;
    * sqrt: hold, then f + (1 - f) * sqrt(1 - t) over the last D of the
      T - 1 - W post-warmup steps.
    """
    T = total_steps
    if T <= 0:
        raise ValueError("the LR schedule needs total_steps > 0")
    W = sched.warmup_steps if sched.warmup_steps is not None else int(T * sched.warmup_ratio)
    D = sched.decay_steps if sched.decay_steps is not None else max(int(T * sched.decay_ratio) - W, 1)
    if sched.min_lr_factor is not None:
        f = sched.min_lr_factor
    else:
        f = sched.min_lr / base_lr if sched.min_lr > 0.0 else 1e-8
    k = step
    if sched.type != "cosine":  # the constant, linear and sqrt chains clamp warmup to the run
        W = min(W, T)
    if W > 0 and k < W:
        return base_lr * (f + (1.0 - f) * k / W)
    t = k - W  # steps since warmup ended
    if sched.type == "constant":
        return base_lr
    eff = max(T - 1, 1)
    if sched.type == "linear":
        D = max(min(D, eff), 1)
        if T - W > 0:
            D = min(D, T - W)
        start = min(T - D, eff)
        if start < W or k < start:
            return base_lr
        n = max(D - 1, 1)
        return base_lr * (1.0 + (f - 1.0) * min(k - start, n) / n)
    if sched.type == "cosine":
        span = min(max(eff - W, 1), D)
        floor = max(sched.min_lr, f * base_lr)
        t = min(t, span)
        return floor + (base_lr - floor) * (1.0 + math.cos(math.pi * t / span)) / 2.0
    if sched.type == "sqrt":
        post = max(T - W - 1, 1)
        span = min(max(D, 1), post)
        d = t - (post - span)
        if d <= 0:
            return base_lr
        return base_lr * (f + (1.0 - f) * math.sqrt(max(1.0 - min(d / span, 1.0), 0.0)))
    raise ValueError(f"unknown scheduler type {sched.type!r}")


def newton_schulz5(g: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Quintic Newton–Schulz iteration towards the orthogonal polar factor
    (coefficients a, b, c = 3.4445, -4.7750, 2.0315 from the Muon write-up),
    over the last two dims; leading dims (stacked experts) are a batch."""
    a, b, c = 3.4445, -4.7750, 2.0315
    x = g.float()
    transposed = x.shape[-2] > x.shape[-1]
    if transposed:
        x = x.transpose(-2, -1)
    shape = x.shape
    x = x.reshape(-1, shape[-2], shape[-1])
    x = x / (x.norm(dim=(1, 2), keepdim=True) + eps)
    for _ in range(steps):
        A = x @ x.transpose(1, 2)
        B = b * A + c * (A @ A)
        x = a * x + B @ x
    x = x.reshape(shape)
    return x.transpose(-2, -1) if transposed else x


def is_muon_matrix(name: str, shape: tuple[int, ...]) -> bool:
    n = name.lower()
    return len(shape) >= 2 and "embed" not in n and "lm_head" not in n


class FlatOptimizer:
    """Common driver: reduce-scatter, norm/clip, per-type update, all-gather."""

    def __init__(self, flat: FlatParams, cfg, max_grad_norm: float, dp_group=None, dp_world: int = 1, fabric=None,
                 expert_flat: FlatParams | None = None, ep_dp_group=None, ep_dp_world: int = 1,
                 norm_fabric=None, replicate_group=None):
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
            if cfg.type not in ("adamw", "adam"):
                raise NotImplementedError("expert parallelism supports optim.type adamw / adam only")
            from ..parallel.zero import CompositeAdamW

            self.adamw = CompositeAdamW([ShardedAdamW(flat, hyper, dp_group, dp_world),
                                         ShardedAdamW(expert_flat, hyper, ep_dp_group, ep_dp_world)],
                                        distributed=dist.is_initialized() and dp_world > 1)
        elif cfg.type in ("adamw_8bit", "adam_8bit", "paged_adamw_8bit"):
            if getattr(cfg, "cpu_offload", False):
                raise ValueError("optim.cpu_offload does not apply to the 8-bit optimizers")
            from ..parallel.zero import ShardedAdamW8bit

            self.adamw = ShardedAdamW8bit(flat, hyper, dp_group, dp_world, paged=cfg.type == "paged_adamw_8bit",
                                          norm_world=flat.tp_size > 1, replicate_group=replicate_group)
        elif fabric is not None and cfg.type in ("adamw", "adam"):
            from ..parallel.zero import FusedShardedAdamW

            self.adamw = FusedShardedAdamW(flat, hyper, fabric, norm_fabric)  # fused peer-memory RS + AdamW + AG
        else:
            self.adamw = ShardedAdamW(flat, hyper, dp_group, dp_world,
                                      offload=bool(getattr(cfg, "cpu_offload", False)),
                                      norm_world=flat.tp_size > 1, replicate_group=replicate_group)
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
        a.local_sumsq_(g, a.stats)
        a.reduce_stats_(a.stats)
        norm_sq, bad = a.stats.tolist()
        why = skip_reason(norm_sq, bad, a.h.max_grad_norm)
        if why is not None:
            flat.zero_grad()
            raise NonFiniteGradientError(why)
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
            d = gs.add(p, alpha=wd) if wd > 0 else gs
            if self.momentum_buf is None:  # first step: the buffer is the gradient
                self.momentum_buf = d.clone()
            else:
                self.momentum_buf.mul_(self.cfg.momentum).add_(d)
            buf = self.momentum_buf
            upd = d.add(buf, alpha=self.cfg.momentum) if self.cfg.nesterov else buf
            p.add_(upd, alpha=-lr)
        elif self.type == "muon":
            self._muon(gs, lr)
        else:
            raise ValueError(f"unsupported optimizer {self.type}")
        compute = flat.compute.detach()
        p16 = compute[flat.shard_slice]
        p16.copy_(p.to(p16.dtype))
        if self.world > 1 and not flat.sharded_compute:  # ZeRO-3 gathers lazily, unit by unit
            dist.all_gather_into_tensor(compute, p16.clone(), group=self.group)
        flat.zero_grad()
        return {"grad_norm": norm, "clip_factor": factor}

    def _muon(self, gs: torch.Tensor, lr: float) -> None:
        flat = self.flat
        beta, wd = self.cfg.muon_momentum, self.cfg.weight_decay
        if self.momentum_buf is None:
            self.momentum_buf = torch.zeros_like(flat.master)
        mom = self.momentum_buf.mul_(beta).add_(gs, alpha=1 - beta)
        src = gs.add(mom, alpha=beta) if self.cfg.nesterov else mom
        lo = flat.dp_rank * flat.shard_numel
        hi = lo + flat.shard_numel
        mats = [s for s in flat.specs if is_muon_matrix(s.name, s.shape)]
        spans = []
        sq = torch.zeros(len(mats), dtype=torch.float64, device=gs.device)
        for i, s in enumerate(mats):
            off, n = flat.offsets[s.name]
            a, b = max(off, lo), min(off + n, hi)
            spans.append((off, n, a, b))
            if a < b:
                sq[i] = gs[a - lo : b - lo].double().pow(2).sum()
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
            full = flat.grad  # replicated gradient buffer: free after the reduce-scatter
            dist.all_gather_into_tensor(full, src.contiguous(), group=self.group)
        else:
            full = src
        gnorm = sq.sqrt().tolist()
        handled = torch.zeros(flat.shard_numel, dtype=torch.bool, device=gs.device)
        for s, (off, n, a, b), gn in zip(mats, spans, gnorm):
            if a >= b:
                continue
            upd = newton_schulz5(full[off : off + n].view(s.shape)).reshape(-1)
            upd = upd[a - off : b - off] * (gn / max(float(upd.norm()), 1e-7))
            seg = flat.master[a - lo : b - lo]
            if wd > 0:
                seg.mul_(1 - lr * wd)
            seg.add_(upd, alpha=-lr)
            handled[a - lo : b - lo] = True
        rest = ~handled
        if rest.any():
            m, v = flat.exp_avg, flat.exp_avg_sq
            b1, b2 = self.cfg.betas1, self.cfg.betas2
            t = self.adamw.step_count
            g = gs[rest]
            m[rest] = b1 * m[rest] + (1 - b1) * g
            v[rest] = b2 * v[rest] + (1 - b2) * g * g
            upd = (m[rest] / (1 - b1**t)) / ((v[rest] / (1 - b2**t)).sqrt() + 1e-8)
            pr = flat.master[rest]
            if wd > 0:
                pr = pr * (1 - lr * wd)
            flat.master[rest] = pr - lr * upd

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
