"""Training engine: micro-steps and optimizer steps on a ``CausalLM``.

The engine owns no data logic; trainers (SFT, RL) feed it device tensors in
the packed layout (``input_ids`` [T], ``position_ids`` [T], ``cu_seqlens``)
and per-token loss weights.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from ..models.qwen import CausalLM
from ..ops import lm_head
from ..parallel.zero import AdamWHyper, CompositeAdamW, FusedShardedAdamW, ShardedAdamW
from ..utils import nvtx


@dataclass
class PackedBatch:
    input_ids: torch.Tensor  # int64 [T]
    position_ids: torch.Tensor  # int32 [T]
    cu_seqlens: torch.Tensor  # int32 [n+1]
    max_seqlen: int
    targets: torch.Tensor  # int64 [T], -100 = ignore
    loss_mask: torch.Tensor  # float [T]
    cp: Any = None  # parallel.context_parallel.CPPlan of a context-parallel shard
    # processor fields of the row's images (pixel_values, image_grid_thw, ...)
    # and ``doc_images``: images per document, in document order
    mm: dict | None = None

    def to(self, device, non_blocking=True) -> "PackedBatch":
        mm = None
        if self.mm is not None:
            mm = {k: (v.to(device, non_blocking=non_blocking) if torch.is_tensor(v) else v) for k, v in self.mm.items()}
        return PackedBatch(
            self.input_ids.to(device, non_blocking=non_blocking),
            self.position_ids.to(device, non_blocking=non_blocking),
            self.cu_seqlens.to(device, non_blocking=non_blocking),
            self.max_seqlen,
            self.targets.to(device, non_blocking=non_blocking),
            self.loss_mask.to(device, non_blocking=non_blocking),
            None if self.cp is None else self.cp.to(device),
            mm,
        )

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.numel())

    def pin_memory(self) -> "PackedBatch":
        mm = None if self.mm is None else {k: (v.pin_memory() if torch.is_tensor(v) else v) for k, v in self.mm.items()}
        return PackedBatch(
            self.input_ids.pin_memory(), self.position_ids.pin_memory(), self.cu_seqlens.pin_memory(),
            self.max_seqlen, self.targets.pin_memory(), self.loss_mask.pin_memory(), self.cp, mm,
        )

    def nbytes(self) -> int:
        ts = [self.input_ids, self.position_ids, self.cu_seqlens, self.targets, self.loss_mask]
        ts += [v for v in (self.mm or {}).values() if torch.is_tensor(v)]
        return sum(t.numel() * t.element_size() for t in ts)


class Engine:
    def __init__(self, model: CausalLM, hyper: AdamWHyper, dp_group=None, dp_world: int = 1,
                 lm_head_chunk: int = lm_head.DEFAULT_CHUNK, fabric=None, ep_dp_group=None, ep_dp_world: int = 1,
                 norm_fabric=None):
        self.model = model
        # the optimizer owns the trainable store: the full model, or only the
        # LoRA adapters when the base is frozen; with expert parallelism the
        # expert store is a second part sharded over the expert-replica group
        if model.expert_flat is not None:
            self.opt = CompositeAdamW(
                [ShardedAdamW(model.flat, hyper, dp_group, dp_world),
                 ShardedAdamW(model.expert_flat, hyper, ep_dp_group, ep_dp_world)],
                norm_group=None, distributed=dist.is_initialized() and dp_world > 1)
        elif fabric is not None:
            self.opt = FusedShardedAdamW(model.trainable, hyper, fabric, norm_fabric)
        else:
            self.opt = ShardedAdamW(model.trainable, hyper, dp_group, dp_world,
                                    norm_world=model.trainable.tp_size > 1)
        self.fabric = fabric
        self.dp_group = dp_group
        self.dp_world = dp_world
        self.chunk = lm_head_chunk

    def _ctx(self, b: PackedBatch):
        m = self.model
        ctx = m.batch_ctx(b.position_ids, b.cu_seqlens, b.max_seqlen, cp=b.cp)
        if b.mm is not None:
            if not getattr(m.cfg, "is_vlm", False):
                raise ValueError("the batch carries image inputs but the model has no vision tower")
            ctx.mm = b.mm
        return ctx

    # --------------------------------------------------------------- SFT
    def sft_micro_step(self, b: PackedBatch, token_scale: float) -> torch.Tensor:
        """Forward + backward of the token-normalised CE on one micro-batch.

        ``token_scale`` = 1 / (loss tokens of the whole step over all ranks),
        so that summing gradients across micro-batches and ranks yields the
        global token mean (parity: trainer/trainer.py:1317-1372).
        Returns the (scaled) loss contribution as a device scalar.
        """
        m = self.model
        ctx = self._ctx(b)
        h = m.hidden(b.input_ids, ctx)
        weights = b.loss_mask.float() * token_scale
        with nvtx.range("lm_head.loss"):
            loss, dh = lm_head.sft_loss_and_grad(h.detach(), m.head_weight(), b.targets, weights, m.head_grad(),
                                                 self.chunk)
        with nvtx.range("backward"):
            h.backward(dh)
        if not b.input_ids.is_cuda or getattr(m, "eager", False):
            m.collect_cpu_grads()  # autograd gradients -> the fp32 flat gradient store
        return loss

    @torch.no_grad()
    def sft_eval(self, b: PackedBatch) -> tuple[torch.Tensor, float]:
        """Forward-only masked CE sum and loss-token count of one micro-batch."""
        m = self.model
        ctx = self._ctx(b)
        h = m.hidden(b.input_ids, ctx)
        valid = (b.targets >= 0).float() * b.loss_mask.float()
        lp, _ = lm_head.logprob_entropy(h.detach(), m.head_weight(), b.targets.clamp_min(0), 1.0,
                                        chunk=self.chunk, want_entropy=False)
        return -(lp * valid).sum(), float(valid.sum())

    def optimizer_step(self, lr: float) -> dict[str, float]:
        with nvtx.range("optimizer.step"):
            self.model.finalize_grads()
            out = self.opt.step(lr)
            hook = getattr(self.model, "after_optimizer_step", None)
            if hook is not None:
                hook()
            return out

    def global_token_count(self, local: float, device) -> float:
        if self.dp_world > 1 and dist.is_initialized():
            t = torch.tensor([local], device=device, dtype=torch.float64)
            dist.all_reduce(t, group=self.dp_group)
            return float(t.item())
        return float(local)
