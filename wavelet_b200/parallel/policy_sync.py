"""Trainer -> generator weight refresh for expert-parallel training
(the reference reloads the rollout engine from a broadcast of the trainer's
weights: transport/policy.py:120-560).

Under expert parallelism every rank trains 1/ep of the experts, but a
rollout replica needs all of them (the 30B-A3B shape is ~61 GB of bf16
weights, well inside one B200).  ``ExpertPolicySync`` keeps a full-weight
generator model per rank and refreshes it after each optimizer step:
* dense tensors: local device copies (identical on every rank);
* expert tensors: one pull-gather kernel per tensor that loads every rank's
  shard straight from its (peer-visible) expert store over NVLink into the
  right rows of the full tensor (reshard fused with the transfer).
A barrier before (every rank's update is complete) and after (every rank has
finished reading) brackets the pulls.
"""

from __future__ import annotations

import torch

from .. import ops
from .fabric import Fabric


class ExpertPolicySync:
    def __init__(self, trainer_model, gen_model, fabric: Fabric):
        self.t = trainer_model
        self.g = gen_model
        self.fab = fabric
        ef = trainer_model.expert_flat
        self.expert_ptrs = fabric.ptrs_of(ef.compute)
        if trainer_model.ep_size != fabric.world:
            raise ValueError("the fabric must span the expert-parallel group")

    @torch.no_grad()
    def refresh(self) -> None:
        t, g, ef = self.t, self.g, self.t.expert_flat
        for n in t.flat.names():
            g.flat.view(n).copy_(t.flat.view(n))
        self.fab.barrier()
        m = ops.ext()
        for n in ef.names():
            off, numel = ef.offsets[n]
            m.gather_from_peers(self.expert_ptrs, self.fab.world, off, numel, g.flat.view(n).reshape(-1))
        self.fab.barrier()
