"""Sharded optimizer step over flat buffers (ZeRO-2 with resident bf16 params).

Per optimizer step, on every data-parallel rank:

1. reduce-scatter the fp32 gradient accumulator (sum over ranks) so rank r
   holds the summed gradient of its shard;
2. squared norm + non-finite count of the shard (one fused kernel), summed
   over ranks, turned into a clip factor on the device;
3. fused AdamW on the shard (fp32 master / m / v) that also writes the bf16
   shard into the resident compute buffer;
4. all-gather the bf16 compute buffer.

With world size 1 steps 1 and 4 disappear.  Parity: the reference's FSDP
reduce-scatter + ``torch.optim.AdamW`` (fused) + ``clip_grad_norm_`` path
(trainer/optim.py:393-512, trainer/trainer.py:1034-1101).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops
from ..models.params import FlatParams


class NonFiniteGradientError(RuntimeError):
    pass


@dataclass
class AdamWHyper:
    lr: float = 1e-3
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0


class ShardedAdamW:
    def __init__(self, flat: FlatParams, hyper: AdamWHyper, dp_group=None, dp_world: int = 1):
        self.flat = flat
        self.h = hyper
        self.group = dp_group
        self.world = dp_world
        self.step_count = 0
        dev = flat.device
        self.g_shard = (
            torch.empty(flat.shard_numel, device=dev, dtype=torch.float32) if dp_world > 1 else None
        )
        self.stats = torch.zeros(2, device=dev, dtype=torch.float32)
        self.clip = torch.ones(2, device=dev, dtype=torch.float32)

    def reduce_grads(self) -> torch.Tensor:
        if self.world > 1:
            dist.reduce_scatter_tensor(self.g_shard, self.flat.grad, op=dist.ReduceOp.SUM, group=self.group)
            return self.g_shard
        return self.flat.grad

    @torch.no_grad()
    def step(self, lr: float | None = None, check_finite: bool = True) -> dict[str, float]:
        flat = self.flat
        lr = self.h.lr if lr is None else lr
        g = self.reduce_grads()
        self.stats.zero_()
        ops.sumsq_(g, self.stats)
        if self.world > 1:
            dist.all_reduce(self.stats, group=self.group)
        norm_sq, bad = self.stats.tolist()
        if check_finite and bad > 0:
            raise NonFiniteGradientError(f"non-finite gradients detected ({int(bad)} elements)")
        norm = norm_sq**0.5
        factor = 1.0
        if self.h.max_grad_norm and self.h.max_grad_norm > 0:
            factor = min(1.0, self.h.max_grad_norm / (norm + 1e-6))
        self.step_count += 1
        compute = flat.compute.detach()
        p16 = compute[flat.shard_slice]
        ops.adamw_flat_(
            flat.master, g, flat.exp_avg, flat.exp_avg_sq, p16 if flat.compute.dtype == torch.bfloat16 else None,
            lr=lr, betas=self.h.betas, eps=self.h.eps, weight_decay=self.h.weight_decay,
            step=self.step_count, gscale_host=factor,
        )
        if compute.dtype != torch.bfloat16:
            p16.copy_(flat.master)
        if self.world > 1:
            src = p16 if compute.is_cuda else p16.clone()
            dist.all_gather_into_tensor(compute, src, group=self.group)
        flat.zero_grad()
        return {"grad_norm": norm, "clip_factor": factor}

    # ---------------------------------------------------------------- state
    def state_dict(self) -> dict:
        return {
            "step": self.step_count,
            "master": self.flat.master,
            "exp_avg": self.flat.exp_avg,
            "exp_avg_sq": self.flat.exp_avg_sq,
        }

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.flat.master.copy_(sd["master"])
        self.flat.exp_avg.copy_(sd["exp_avg"])
        self.flat.exp_avg_sq.copy_(sd["exp_avg_sq"])
        compute = self.flat.compute.detach()
        p16 = compute[self.flat.shard_slice]
        p16.copy_(self.flat.master.to(p16.dtype))
        if self.world > 1:
            dist.all_gather_into_tensor(compute, p16.clone(), group=self.group)
