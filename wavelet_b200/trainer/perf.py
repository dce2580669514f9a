"""Throughput / MFU accounting.

FLOPs per trained token = 6 * N_active_matmul + 12 * L * H * S (attention
scores), the formula of the reference (trainer/perf.py:149-202); with LoRA the
frozen base contributes 4 * N (no weight gradient) and adapters 6 * N_lora.
The MFU denominator is the dense bf16 peak of the device (B200: 2.25e15,
trainer/perf.py:233-256).
"""

from __future__ import annotations

import time

import torch

PEAK_BF16 = {"B200": 2.25e15, "GB200": 2.5e15, "H100": 989e12, "H200": 989e12, "A100": 312e12}


def device_peak_flops(device: torch.device) -> float:
    if device.type != "cuda":
        return 1e12
    name = torch.cuda.get_device_name(device)
    for k, v in PEAK_BF16.items():
        if k in name:
            return v
    return 2.25e15


def _deepseek_v4_params(cfg) -> int:
    """DeepSeek-V4: attention projections, compressor projections, the two
    hyper-connection maps, active + shared experts and the router per layer."""
    H, nh, D, hc = cfg.hidden_size, cfg.num_attention_heads, cfg.head_dim, cfg.hc_mult
    attn = H * cfg.q_lora_rank + cfg.q_lora_rank * nh * D + H * D + nh * D * cfg.o_lora_rank \
        + cfg.o_groups * cfg.o_lora_rank * H
    hc_maps = 2 * (2 + hc) * hc * hc * H
    moe = (cfg.num_experts_per_tok + cfg.n_shared_experts) * 3 * H * cfg.moe_intermediate_size \
        + cfg.n_routed_experts * H
    total = 0
    for t in cfg.layer_types:
        comp = 0 if t == "sliding_attention" else 2 * (2 if t == "compressed_sparse_attention" else 1) * D * H
        total += attn + comp + hc_maps + moe
    return total + cfg.vocab_size * H


def matmul_params(cfg) -> int:
    """Parameters that take part in matmuls for one token (active experts only)."""
    if hasattr(cfg, "hc_mult"):
        return _deepseek_v4_params(cfg)
    H, I = cfg.hidden_size, cfg.intermediate_size
    attn = H * cfg.qkv_dim + cfg.q_dim * H
    total = 0
    for i in range(cfg.num_layers):
        if cfg.layer_is_moe(i):
            mlp = cfg.num_experts_per_tok * 3 * H * cfg.moe_intermediate_size + cfg.num_experts * H
        else:
            mlp = 3 * H * I
        total += attn + mlp
    return total + cfg.vocab_size * H  # LM head


def flops_per_token(cfg, seq_len: int, lora_params: int | None = None) -> float:
    n = matmul_params(cfg)
    if hasattr(cfg, "hc_mult"):  # each query reads its window plus at most index_topk entries
        keys = min(seq_len, cfg.sliding_window + cfg.index_topk)
        attn = 12 * cfg.num_hidden_layers * cfg.num_attention_heads * cfg.head_dim * keys
    else:
        attn = 12 * cfg.num_layers * cfg.q_dim * seq_len
    if lora_params:
        return 4 * n + 6 * lora_params + attn
    return 6 * n + attn


class PerfTracker:
    def __init__(self, cfg, device, lora_rank=None, lora_params=None):
        self.cfg = cfg
        self.device = device
        self.peak = device_peak_flops(device)
        self.lora_params = lora_params
        self.seq_len = 4096

    def step_metrics(self, global_tokens: int, seconds: float, seq_len: int | None = None) -> dict[str, float]:
        seq_len = seq_len or self.seq_len
        tps = global_tokens / max(seconds, 1e-9)
        ws = int(torch.distributed.get_world_size()) if torch.distributed.is_initialized() else 1
        fl = flops_per_token(self.cfg, seq_len, self.lora_params)
        m = {
            "perf/tokens_per_second": tps,
            "perf/step_tokens_per_second": tps,
            "perf/throughput": tps,
            "perf/step_seconds": seconds,
            "perf/mfu": tps * fl / (self.peak * ws),
        }
        if self.device.type == "cuda":
            m["perf/peak_memory_gib"] = torch.cuda.max_memory_allocated(self.device) / 2**30
        return m
