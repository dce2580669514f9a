"""One optimizer step of token-normalised SFT over a list of host micro-batches.

``SFTStepper.train_step`` is the public call a user (and ``bench.py``) makes
per optimizer step: it copies each micro-batch from (pinned) host memory to
the device, runs forward + backward, performs the sharded AdamW step and
returns the step loss read back to the host.
"""

from __future__ import annotations

import torch

from .engine import Engine, PackedBatch


class SFTStepper:
    def __init__(self, engine: Engine, device: torch.device, copy_stream: bool = True):
        self.engine = engine
        self.device = device
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    def train_step(self, micro_batches: list[PackedBatch], lr: float, device_resident: bool = False) -> dict:
        eng = self.engine
        local_tokens = float(sum(float(b.loss_mask.sum()) for b in micro_batches))
        total = eng.global_token_count(local_tokens, self.device)
        scale = 1.0 / max(total, 1.0)
        loss = torch.zeros((), device=self.device, dtype=torch.float32)
        for b in micro_batches:
            if not device_resident:
                self.h2d_bytes += b.nbytes()
                b = b.to(self.device)
            loss += eng.sft_micro_step(b, scale)
        stats = eng.optimizer_step(lr)
        if eng.dp_world > 1:
            import torch.distributed as dist

            dist.all_reduce(loss, group=eng.dp_group)
        loss_host = float(loss.item())
        self.d2h_bytes += 4
        return {"loss": loss_host, "optim/grad_norm": stats["grad_norm"], "loss_tokens": total}
