"""DeepSeek-V4 mixture of experts (reference trainer/models/deepseek_v4/moe.py).

Scores are ``sqrt(softplus(x W_gate^T))`` (fp32).  Top-k layers pick the k
largest ``score + selection_bias`` (the bias is the auxiliary-loss-free
balancing term: it steers selection only, never the weights); hash layers
take their experts from a token-id table ``tid2eid``.  The weights are the
selected scores normalised to sum 1 and multiplied by
``routed_scaling_factor``, kept in fp32 until the expert output is scaled.
Experts and the shared expert are SwiGLU with the gate clamped from above
and the up projection clamped to ``[-limit, limit]``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .config import DeepseekV4Config


def clamped_swiglu(gate: Tensor, up: Tensor, limit: float) -> Tensor:
    return F.silu(gate.clamp(max=limit)) * up.clamp(-limit, limit)


class Router(nn.Module):
    def __init__(self, config: DeepseekV4Config, hashed: bool):
        super().__init__()
        self.k = config.num_experts_per_tok
        self.n = config.n_routed_experts
        self.scale = config.routed_scaling_factor
        self.norm = config.norm_topk_prob
        self.gate = nn.Linear(config.hidden_size, self.n, bias=False)
        if hashed:
            self.register_buffer("tid2eid", torch.zeros(config.vocab_size, self.k, dtype=torch.long))
            self.selection_bias = None
        else:
            self.register_buffer("selection_bias", torch.zeros(self.n))

    def forward(self, x: Tensor, chosen: Tensor | None = None) -> tuple[Tensor, Tensor]:
        """x [T, H] -> (weights fp32 [T, k], experts [T, k])."""
        s = F.softplus(self.gate(x).float()).sqrt()
        if chosen is None:
            sel = s if self.selection_bias is None else s + self.selection_bias.float()
            chosen = sel.topk(self.k, dim=-1).indices
        w = s.gather(-1, chosen)
        if self.norm:
            w = w / (w.sum(-1, keepdim=True) + 1e-20)
        return w * self.scale, chosen


class Experts(nn.Module):
    """Stacked expert weights: gate / up [E, I, H], down [E, H, I]."""

    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        E, I, H = config.n_routed_experts, config.moe_intermediate_size, config.hidden_size
        self.limit = config.swiglu_limit
        self.gate_proj = nn.Parameter(torch.empty(E, I, H))
        self.up_proj = nn.Parameter(torch.empty(E, I, H))
        self.down_proj = nn.Parameter(torch.empty(E, H, I))

    def forward(self, x: Tensor, experts: Tensor, weights: Tensor) -> Tensor:
        out = torch.zeros_like(x)
        for e in torch.unique(experts).tolist():
            rows, slot = (experts == e).nonzero(as_tuple=True)
            xe = x[rows]
            y = F.linear(clamped_swiglu(F.linear(xe, self.gate_proj[e]), F.linear(xe, self.up_proj[e]), self.limit),
                         self.down_proj[e])
            out.index_add_(0, rows, (y * weights[rows, slot, None]).to(out.dtype))
        return out


class SharedExpert(nn.Module):
    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        H, I = config.hidden_size, config.moe_intermediate_size
        self.limit = config.swiglu_limit
        self.gate_proj = nn.Linear(H, I, bias=False)
        self.up_proj = nn.Linear(H, I, bias=False)
        self.down_proj = nn.Linear(I, H, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.down_proj(clamped_swiglu(self.gate_proj(x), self.up_proj(x), self.limit))


class MoE(nn.Module):
    def __init__(self, config: DeepseekV4Config, layer_idx: int):
        super().__init__()
        if config.scoring_func != "sqrtsoftplus":
            raise ValueError("DeepSeek-V4 routing supports scoring_func='sqrtsoftplus' only")
        if config.hidden_act != "silu" or config.mlp_bias:
            raise ValueError("DeepSeek-V4 experts are bias-free SwiGLU (hidden_act='silu')")
        self.hashed = layer_idx < config.num_hash_layers
        self.router = Router(config, self.hashed)
        self.experts = Experts(config)
        self.shared_expert = SharedExpert(config) if config.n_shared_experts else None
        # routed-token counts since the last balance update (optimizer-step state, not saved)
        self.register_buffer("tokens_per_expert", torch.zeros(config.n_routed_experts), persistent=False)

    def forward(self, x: Tensor, input_ids: Tensor | None = None) -> Tensor:
        chosen = None
        if self.hashed:
            if input_ids is None:
                raise ValueError("a hash-routed DeepSeek-V4 layer needs the input ids")
            chosen = self.router.tid2eid[input_ids]
        w, chosen = self.router(x, chosen)
        if self.training and torch.is_grad_enabled():
            with torch.no_grad():
                self.tokens_per_expert += torch.bincount(chosen.reshape(-1), minlength=self.tokens_per_expert.numel())
        out = self.experts(x, chosen, w)
        return out + self.shared_expert(x) if self.shared_expert is not None else out

    @torch.no_grad()
    def balance_(self, rate: float = 1e-3) -> None:
        """Auxiliary-loss-free balancing (DeepSeek-V3 report, section 2.1.2):
        raise the selection bias of under-loaded experts and lower it for
        over-loaded ones by ``rate``, then reset the counts."""
        if self.router.selection_bias is not None and self.tokens_per_expert.sum() > 0:
            load = self.tokens_per_expert
            self.router.selection_bias += rate * torch.sign(load.mean() - load)
        self.tokens_per_expert.zero_()
