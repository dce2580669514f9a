"""Sharded optimizer step over flat buffers (ZeRO-2 with resident bf16 params).

Per optimizer step, on every data-parallel rank:

1. reduce-scatter the fp32 gradient accumulator (sum over ranks) so rank r
   holds the summed gradient of its shard;
2. squared norm + non-finite count of the shard (one fused kernel), summed
   over ranks, turned into a clip factor on the device;
3. fused AdamW on the shard (fp32 master / m / v) that also writes the bf16
   shard into the resident compute buffer;
4. all-gather the bf16 compute buffer.

With world size 1 steps 1 and 4 disappear.  ``FusedShardedAdamW`` runs the
same step as three kernels over peer memory (parallel.fabric): a
reduce-scatter that pulls every rank's gradient slice over NVLink and sums,
scales and squares it in one pass; a norm exchange; and an AdamW kernel that
stores the updated bf16 shard straight into every rank's compute buffer (the
all-gather rides on the update's stores).  Parity: the reference's FSDP
reduce-scatter + ``torch.optim.AdamW`` (fused) + ``clip_grad_norm_`` path
(trainer/optim.py:393-512, trainer/trainer.py:1034-1101).
"""

from __future__ import annotations

import math

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops
from ..models.params import FlatParams


class NonFiniteGradientError(RuntimeError):
    pass


def skip_reason(norm_sq: float, bad: float, max_grad_norm: float) -> str | None:
    """Why an optimizer step must be skipped, or None.

    Non-finite gradient elements always skip the step.  A squared norm that
    overflows float32 while every element is finite skips it only when
    clipping is on (its clip factor would be 0); with ``max_grad_norm <= 0``
    the step proceeds, as in the reference, which looks at the norm only when
    clipping (trainer/trainer.py:1034-1101, trainer/rl.py:939)."""
    if bad > 0:
        return f"non-finite gradients detected ({int(bad)} elements)"
    if not math.isfinite(norm_sq) and max_grad_norm and max_grad_norm > 0:
        return "the squared gradient norm overflows float32 (every element is finite); the clip cannot scale it"
    return None


@dataclass
class AdamWHyper:
    lr: float = 1e-3
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0


class ShardedAdamW:
    def __init__(self, flat: FlatParams, hyper: AdamWHyper, dp_group=None, dp_world: int = 1,
                 offload: bool = False, offload_chunk: int = 1 << 26, norm_world: bool = False,
                 replicate_group=None):
        self.flat = flat
        self.h = hyper
        self.group = dp_group
        self.world = dp_world
        # hybrid sharding: the sharded store is replicated over this group,
        # whose members all-reduce their reduced gradient shards
        self.replicate_group = replicate_group
        # norm_world: the squared norm is summed over every rank of the job
        # (tensor parallelism: each TP rank holds a different part of the model)
        self.norm_world = norm_world
        self.step_count = 0
        dev = flat.device
        # optim.cpu_offload: fp32 master / moments live in pinned host memory and
        # stream through the GPU AdamW kernel in chunks (reference
        # trainer/optim.py:191-390 offloads optimizer state to pinned CPU)
        self.offload = offload and dev.type == "cuda"
        self.offload_chunk = offload_chunk
        if self.offload:
            for name in ("master", "exp_avg", "exp_avg_sq"):
                t = getattr(flat, name)
                setattr(flat, name, t.cpu().pin_memory())
                del t
            self._stage = [torch.empty(min(offload_chunk, flat.shard_numel), device=dev, dtype=torch.float32)
                           for _ in range(3)]
        self.g_shard = (
            torch.empty(flat.shard_numel, device=dev, dtype=torch.float32)
            if dp_world > 1 and not flat.sharded_compute else None
        )
        self.stats = torch.zeros(2, device=dev, dtype=torch.float32)
        self.clip = torch.ones(2, device=dev, dtype=torch.float32)

    def reduce_grads(self) -> torch.Tensor:
        if self.flat.sharded_compute:  # ZeRO-3: each unit's gradients were reduced into the shard in backward
            if self.replicate_group is not None:
                dist.all_reduce(self.flat.grad, group=self.replicate_group)
            return self.flat.grad
        if self.world > 1:
            dist.reduce_scatter_tensor(self.g_shard, self.flat.grad, op=dist.ReduceOp.SUM, group=self.group)
            return self.g_shard
        return self.flat.grad

    # Two phases so several stores (dense + expert shards) can share one clip:
    # ``prepare`` reduces the gradients and returns this rank's (sumsq,
    # non-finite) of its shard; ``apply`` runs the update with a clip factor.
    @torch.no_grad()
    def prepare(self) -> torch.Tensor:
        self._g = self.reduce_grads()
        self.stats.zero_()
        self.local_sumsq_(self._g, self.stats)
        return self.stats

    def local_sumsq_(self, g: torch.Tensor, stats: torch.Tensor) -> None:
        """(sum of squares, non-finite count) of this rank's reduced gradient
        ``g`` added into ``stats``; TP-replicated elements weigh 1/tp."""
        flat = self.flat
        k = flat.shard_repl_split() if self.world > 1 else min(flat.tp_repl_end, g.numel())
        if flat.tp_size > 1 and k > 0:
            part = torch.zeros_like(stats)
            ops.sumsq_(g[:k], part)
            part[0] /= flat.tp_size
            stats.add_(part)
            if k < g.numel():
                ops.sumsq_(g[k:], stats)
        else:
            ops.sumsq_(g, stats)

    def reduce_stats_(self, stats: torch.Tensor) -> None:
        if self.norm_world and dist.is_initialized():
            dist.all_reduce(stats)
        elif self.world > 1:
            dist.all_reduce(stats, group=self.group)

    @torch.no_grad()
    def apply(self, lr: float, factor: float) -> None:
        flat = self.flat
        self.step_count += 1
        compute = flat.compute.detach()
        p16 = compute[flat.shard_slice]
        if self.offload:
            self._apply_offloaded(p16, lr, factor)
        else:
            ops.adamw_flat_(
                flat.master, self._g, flat.exp_avg, flat.exp_avg_sq,
                p16 if flat.compute.dtype == torch.bfloat16 else None,
                lr=lr, betas=self.h.betas, eps=self.h.eps, weight_decay=self.h.weight_decay,
                step=self.step_count, gscale_host=factor,
            )
        if compute.dtype != torch.bfloat16:
            p16.copy_(flat.master)
        if self.world > 1 and not flat.sharded_compute:  # ZeRO-3 gathers lazily, unit by unit
            src = p16 if compute.is_cuda else p16.clone()
            dist.all_gather_into_tensor(compute, src, group=self.group)
        flat.zero_grad()
        self._g = None

    def _apply_offloaded(self, p16, lr: float, factor: float) -> None:
        """Chunk by chunk: host -> device, fused AdamW (writes the bf16 shard),
        device -> host; all on the current stream, so each chunk's staging
        buffers are reused only after its copy-back has been issued in order."""
        flat = self.flat
        n = flat.shard_numel
        sp, sm, sv = self._stage
        for lo in range(0, n, self.offload_chunk):
            hi = min(n, lo + self.offload_chunk)
            k = hi - lo
            sp[:k].copy_(flat.master[lo:hi], non_blocking=True)
            sm[:k].copy_(flat.exp_avg[lo:hi], non_blocking=True)
            sv[:k].copy_(flat.exp_avg_sq[lo:hi], non_blocking=True)
            ops.adamw_flat_(sp[:k], self._g[lo:hi], sm[:k], sv[:k],
                            p16[lo:hi] if flat.compute.dtype == torch.bfloat16 else None,
                            lr=lr, betas=self.h.betas, eps=self.h.eps, weight_decay=self.h.weight_decay,
                            step=self.step_count, gscale_host=factor)
            flat.master[lo:hi].copy_(sp[:k], non_blocking=True)
            flat.exp_avg[lo:hi].copy_(sm[:k], non_blocking=True)
            flat.exp_avg_sq[lo:hi].copy_(sv[:k], non_blocking=True)
        torch.cuda.current_stream(flat.device).synchronize()  # host copies complete before the next step reads them

    def clip_factor(self, norm: float) -> float:
        if self.h.max_grad_norm and self.h.max_grad_norm > 0:
            return min(1.0, self.h.max_grad_norm / (norm + 1e-6))
        return 1.0

    @torch.no_grad()
    def step(self, lr: float | None = None, check_finite: bool = True) -> dict[str, float]:
        lr = self.h.lr if lr is None else lr
        stats = self.prepare()
        self.reduce_stats_(stats)
        norm_sq, bad = stats.tolist()
        why = skip_reason(norm_sq, bad, self.h.max_grad_norm)
        if check_finite and why is not None:
            self.flat.zero_grad()
            raise NonFiniteGradientError(why)
        norm = norm_sq**0.5
        factor = self.clip_factor(norm)
        self.apply(lr, factor)
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
        if self.world > 1 and not self.flat.sharded_compute:
            dist.all_gather_into_tensor(compute, p16.clone(), group=self.group)


class ShardedAdamW8bit(ShardedAdamW):
    """ZeRO step with 8-bit moments: the fp32 master shard is kept, the two
    AdamW moments are stored as 8-bit block-scaled log codes (one fp32 scale
    per 256 elements; ``ops.adamw8_flat_``), 2 bytes per element instead of 8.
    ``paged``: the codes live in CUDA managed memory, which migrates to host
    memory under device memory pressure (the role of bitsandbytes' paged
    optimizers, reference trainer/optim.py:393-512)."""

    def __init__(self, flat: FlatParams, hyper: AdamWHyper, dp_group=None, dp_world: int = 1,
                 paged: bool = False, norm_world: bool = False, replicate_group=None):
        super().__init__(flat, hyper, dp_group, dp_world, norm_world=norm_world, replicate_group=replicate_group)
        n = flat.shard_numel
        nb = (n + ops.Q8_BLOCK - 1) // ops.Q8_BLOCK
        dev = flat.device
        self.paged = paged and dev.type == "cuda"
        if self.paged:
            m = ops.ext()
            idx = dev.index if dev.index is not None else torch.cuda.current_device()
            self.m8 = m.managed_empty(n, idx).view(torch.int8)
            self.v8 = m.managed_empty(n, idx)
        else:
            self.m8 = torch.zeros(n, device=dev, dtype=torch.int8)
            self.v8 = torch.zeros(n, device=dev, dtype=torch.uint8)
        self.am = torch.zeros(nb, device=dev, dtype=torch.float32)
        self.av = torch.zeros(nb, device=dev, dtype=torch.float32)
        # the fp32 moments of the store are not used: free them
        flat.exp_avg = None
        flat.exp_avg_sq = None

    @torch.no_grad()
    def apply(self, lr: float, factor: float) -> None:
        flat = self.flat
        self.step_count += 1
        compute = flat.compute.detach()
        p16 = compute[flat.shard_slice]
        ops.adamw8_flat_(flat.master, self._g, self.m8, self.v8, self.am, self.av,
                         p16 if flat.compute.dtype == torch.bfloat16 else None,
                         lr=lr, betas=self.h.betas, eps=self.h.eps, weight_decay=self.h.weight_decay,
                         step=self.step_count, gscale_host=factor)
        if compute.dtype != torch.bfloat16:
            p16.copy_(flat.master)
        if self.world > 1 and not flat.sharded_compute:  # ZeRO-3 gathers lazily, unit by unit
            src = p16 if compute.is_cuda else p16.clone()
            dist.all_gather_into_tensor(compute, src, group=self.group)
        flat.zero_grad()
        self._g = None

    def state_dict(self) -> dict:
        return {"step": self.step_count, "master": self.flat.master, "m8": self.m8, "v8": self.v8,
                "m8_scale": self.am, "v8_scale": self.av}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.flat.master.copy_(sd["master"])
        if "m8" in sd:
            self.m8.copy_(sd["m8"])
            self.v8.copy_(sd["v8"])
            self.am.copy_(sd["m8_scale"])
            self.av.copy_(sd["v8_scale"])
        else:  # fp32 moments (a re-sharded or fp32-AdamW checkpoint): quantise
            m8, v8, am, av = ops.q8_quant_moments(sd["exp_avg"].to(self.am.device), sd["exp_avg_sq"].to(self.am.device))
            self.m8.copy_(m8)
            self.v8.copy_(v8)
            self.am.copy_(am)
            self.av.copy_(av)
        compute = self.flat.compute.detach()
        p16 = compute[self.flat.shard_slice]
        p16.copy_(self.flat.master.to(p16.dtype))
        if self.world > 1 and not self.flat.sharded_compute:
            dist.all_gather_into_tensor(compute, p16.clone(), group=self.group)


class FusedShardedAdamW(ShardedAdamW):
    """ZeRO step as fused peer-memory kernels (one node, world <= 8).

    Per step: barrier (every rank's gradients complete) -> reduce-scatter +
    squared norm -> norm exchange + clip factor -> AdamW + bf16 all-gather ->
    barrier (every rank's parameters complete).  No host synchronisation
    inside; the finite check reads the totals after the step, and a
    non-finite step leaves the parameters unchanged on every rank.
    """

    def __init__(self, flat: FlatParams, hyper: AdamWHyper, fabric, norm_fabric=None):
        super().__init__(flat, hyper, dp_group=fabric.group, dp_world=fabric.world)
        self.fabric = fabric
        # norm_fabric: pads spanning every rank of the job, for the norm exchange
        # under tensor parallelism (the data-parallel fabric spans one TP slice)
        self.norm_fabric = norm_fabric if norm_fabric is not None else fabric
        if self.g_shard is None:
            self.g_shard = torch.empty(flat.shard_numel, device=flat.device, dtype=torch.float32)
        self.tot = torch.zeros(3, device=flat.device, dtype=torch.float32)
        self.grad_ptrs = fabric.ptrs_of(flat.grad)
        self.compute_ptrs = fabric.ptrs_of(flat.compute)

    @torch.no_grad()
    def step(self, lr: float | None = None, check_finite: bool = True) -> dict[str, float]:
        from .fabric import SLOT_NORM

        flat, fab, m = self.flat, self.fabric, ops.ext()
        lr = self.h.lr if lr is None else lr
        lo = flat.dp_rank * flat.shard_numel
        fab.barrier()
        self.stats.zero_()
        m.rs_sum_sumsq(self.grad_ptrs, self.world, lo, flat.shard_numel, 1.0, self.g_shard, self.stats,
                       flat.tp_repl_end, 1.0 / flat.tp_size)
        nf = self.norm_fabric
        e = nf.next_epoch(SLOT_NORM)
        max_norm = float(self.h.max_grad_norm or 0.0)
        m.norm_exchange(nf.pads.ptrs, nf.rank, nf.world, e, self.stats, max_norm, self.tot, nf.budget_s)
        self.step_count += 1
        b1, b2 = self.h.betas
        m.adamw_allgather(self.compute_ptrs, self.world, lo, flat.master, self.g_shard, flat.exp_avg,
                          flat.exp_avg_sq, lr, b1, b2, self.h.eps, self.h.weight_decay, self.step_count, self.tot)
        fab.barrier()
        flat.zero_grad()
        norm_sq, bad, factor = self.tot.tolist()
        fab.check()
        if nf is not fab:
            nf.check()
        if bad > 0:  # the kernels skipped the update on every rank
            self.step_count -= 1
            overflow = 1.0 if (not math.isfinite(norm_sq) and max_norm > 0) else 0.0  # norm_exchange adds it
            why = skip_reason(norm_sq, bad - overflow, max_norm)
            if check_finite:
                raise NonFiniteGradientError(f"{why}; step skipped")
        return {"grad_norm": norm_sq**0.5, "clip_factor": factor}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.flat.master.copy_(sd["master"])
        self.flat.exp_avg.copy_(sd["exp_avg"])
        self.flat.exp_avg_sq.copy_(sd["exp_avg_sq"])
        shard = self.flat.master.to(torch.bfloat16)
        lo = self.flat.dp_rank * self.flat.shard_numel
        self.fabric.barrier()
        ops.ext().allgather_bf16(self.compute_ptrs, self.world, lo, shard)
        self.fabric.barrier()
        torch.cuda.synchronize(self.flat.device)
        self.fabric.check()


class CompositeAdamW:
    """One optimizer step over several flat stores with a single global clip.

    Used with expert parallelism: the dense store is sharded over the whole
    data-parallel group and the expert store over the ranks that hold the same
    experts.  Every (store, rank) shard is disjoint, so the global squared
    norm is one all-reduce over ``norm_group`` of the per-rank shard sums.
    """

    def __init__(self, parts: list[ShardedAdamW], norm_group=None, distributed: bool = False):
        self.parts = parts
        self.norm_group = norm_group
        self.distributed = distributed
        self.h = parts[0].h

    @property
    def step_count(self) -> int:
        return self.parts[0].step_count

    @torch.no_grad()
    def step(self, lr: float | None = None, check_finite: bool = True) -> dict[str, float]:
        lr = self.h.lr if lr is None else lr
        total = None
        for p in self.parts:
            st = p.prepare()
            total = st.clone() if total is None else total + st
        if self.distributed:
            dist.all_reduce(total, group=self.norm_group)
        norm_sq, bad = total.tolist()
        why = skip_reason(norm_sq, bad, self.h.max_grad_norm)
        if check_finite and why is not None:
            for p in self.parts:
                p.flat.zero_grad()
            raise NonFiniteGradientError(why)
        norm = norm_sq**0.5
        factor = self.parts[0].clip_factor(norm)
        for p in self.parts:
            p.apply(lr, factor)
        return {"grad_norm": norm, "clip_factor": factor}

    def state_dict(self) -> dict:
        return {f"part{i}": p.state_dict() for i, p in enumerate(self.parts)}

    def load_state_dict(self, sd: dict) -> None:
        for i, p in enumerate(self.parts):
            p.load_state_dict(sd[f"part{i}"])
