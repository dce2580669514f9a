"""DeepSeek-V4 behind the trainer's model interface (the eager module with
its parameters living in flat stores, so the data-parallel sharded AdamW,
checkpointing and the chunked LM-head loss work unchanged).

Parameters are split over two stores: the bulk in the compute dtype
(``flat``) and the numerically sensitive tensors (hyper-connection maps,
sinks, compressor position biases, norms) in an fp32 store.  The second store
sits in the ``expert_flat`` slot that the engine and optimizers already treat
as an independently sharded part of one composite AdamW step.  The module's
parameters are views of the stores; autograd gradients are added into the
stores' fp32 gradient buffers after each backward (``collect_cpu_grads``).
Routing-bias buffers (``selection_bias``, ``tid2eid``) stay module buffers,
updated by the auxiliary-loss-free balancing rule once per optimizer step.

Not supported with this model (as in the reference's eager DeepSeek-V4):
tensor, expert and context parallelism, LoRA / QLoRA.
"""

from __future__ import annotations

from pathlib import Path

import torch
from torch import nn

from ..layers import BatchCtx
from ..params import FlatParams, ParamSpec
from .config import DeepseekV4Config
from .model import DeepseekV4ForCausalLM


class DeepseekV4Trainable:
    eager = True  # the engine collects autograd gradients after every backward

    def __init__(self, cfg: DeepseekV4Config, device, dtype=None, dp_rank: int = 0, dp_world: int = 1, seed: int = 0,
                 init: bool = True, with_grad: bool = True, with_optimizer: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        dtype = dtype or torch.float32
        torch.manual_seed(seed)
        self.module = DeepseekV4ForCausalLM(cfg, init=init).to(self.device)
        self.module.train()
        named = list(self.module.named_parameters())
        keep32 = DeepseekV4ForCausalLM.keep_in_fp32_for_weight_transfer
        main = [ParamSpec(n, tuple(p.shape), weight_decay=p.dim() >= 2) for n, p in named if not keep32(n)]
        fp32 = [ParamSpec(n, tuple(p.shape), weight_decay=False) for n, p in named if keep32(n)]
        self.flat = FlatParams(main, self.device, dtype, dp_rank, dp_world, with_grad, with_optimizer)
        self.expert_flat = FlatParams(fp32, self.device, torch.float32, dp_rank, dp_world, with_grad, with_optimizer)
        self._bind()
        # trainer-interface attributes of the Qwen models
        self.lora = None
        self.quant = None
        self.tp_size, self.tp_rank, self.tp_group, self.tp_fabric = 1, 0, None, None
        self.ep_size, self.ep_rank, self.ep_dp_rank, self.ep_group = 1, 0, 0, None
        self.fused_cpu = True
        self.checkpoint_layers = False

    def _store_of(self, name: str) -> FlatParams:
        return self.expert_flat if DeepseekV4ForCausalLM.keep_in_fp32_for_weight_transfer(name) else self.flat

    def _bind(self) -> None:
        """Copy the module's values into the stores and make every module
        parameter a view of its store (requires_grad as before)."""
        params = dict(self.module.named_parameters())
        with torch.no_grad():
            for n, p in params.items():
                self._store_of(n).view(n).copy_(p.detach())
        for f in (self.flat, self.expert_flat):
            f.sync_master_from_compute()
        for n, p in params.items():
            owner_name, _, leaf = n.rpartition(".")
            owner = self.module.get_submodule(owner_name) if owner_name else self.module
            setattr(owner, leaf, nn.Parameter(self._store_of(n).view(n), requires_grad=p.requires_grad))

    # ------------------------------------------------------ trainer interface
    @property
    def trainable(self) -> FlatParams:
        return self.flat

    @property
    def inv_freq(self):
        return None

    def batch_ctx(self, position_ids, cu_seqlens, max_seqlen, cp=None) -> BatchCtx:
        if cp is not None:
            raise NotImplementedError("the eager DeepSeek-V4 model has no context parallelism")
        return BatchCtx(pos=position_ids.reshape(-1).to(self.device), cu_seqlens=cu_seqlens.to(self.device),
                        max_seqlen=int(max_seqlen), inv_freq=None)

    def hidden(self, input_ids: torch.Tensor, batch: BatchCtx) -> torch.Tensor:
        ids = input_ids.reshape(-1).to(self.device)
        lens = (batch.cu_seqlens[1:] - batch.cu_seqlens[:-1]).to(torch.int64)
        body = self.module.model
        if not self.checkpoint_layers:
            return body(ids, lens)
        return _checkpointed_body(body, ids, lens)

    def head_weight(self) -> torch.Tensor:
        return self.flat.view("lm_head.weight")

    def head_grad(self) -> torch.Tensor | None:
        return self.flat.grad_view("lm_head.weight")

    def collect_cpu_grads(self) -> None:
        for n, p in self.module.named_parameters():
            if p.grad is not None:
                g = self._store_of(n).grad_view(n)
                if g is not None:
                    g.add_(p.grad.float())
                p.grad = None

    def finalize_grads(self) -> None:
        self.module.balance_experts_(1e-3)

    def set_activation_checkpointing(self, every: int | None) -> None:
        self.checkpoint_layers = every is not None

    def enable_activation_offload(self, on: bool = True) -> None:
        if on:
            raise NotImplementedError("activation offload is not available for the eager DeepSeek-V4 model")

    def extra_state(self) -> dict[str, torch.Tensor]:
        """Persistent buffers (routing bias, hash table) for trainer checkpoints."""
        return {n: b for n, b in self.module.named_buffers() if n.endswith(("selection_bias", "tid2eid"))}

    def load_extra_state(self, tensors: dict[str, torch.Tensor]) -> None:
        with torch.no_grad():
            for n, t in tensors.items():
                b = self.module.get_buffer(n)
                b.copy_(t.to(b.device, b.dtype))

    def load_pretrained(self, path: str | Path) -> None:
        """Load a native checkpoint directory into the stores."""
        from safetensors.torch import load_file

        state = load_file(str(Path(path) / "model.safetensors"))
        params = dict(self.module.named_parameters())
        with torch.no_grad():
            for k, v in state.items():
                if k in params:
                    self._store_of(k).view(k).copy_(v.to(self.device))
                else:
                    buf = self.module.get_buffer(k)
                    buf.copy_(v.to(buf.device, buf.dtype))
        for f in (self.flat, self.expert_flat):
            f.sync_master_from_compute()


def _checkpointed_body(body, ids, lens):
    from torch.utils.checkpoint import checkpoint

    from .attention import PackedLayout

    x = body.embed_tokens(ids)
    layout = PackedLayout.build(body.rotary_emb, lens, x.dtype, x.device)
    streams = x.unsqueeze(1).expand(-1, body.config.hc_mult, -1).contiguous()
    for layer in body.layers:
        streams = checkpoint(layer, streams, ids, layout, use_reentrant=False)
    return body.norm(body.hc_head(streams))
