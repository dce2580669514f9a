"""Throughput / MFU accounting.

FLOPs per trained token = 6 * N_active_matmul + 12 * L * H * S (attention
scores, H the hidden size), the formula of the reference
(trainer/perf.py:35-202); with LoRA the frozen base contributes 4 * N (no
weight gradient), other trainable tensors 2 * n and adapters 6 * N_lora.
``perf/mfu`` is in percent of the dense bf16/fp16 peak of the device
(B200: 2.25e15, trainer/perf.py:233-284) and is left out on hardware without
a known peak (CPU included).  DeepSeek-V4 counts its own projections and
bounds the attention term by the keys a query can see (sliding window plus
the indexer's top-k) instead of the whole sequence.
"""

from __future__ import annotations

import time

import torch

def peak_flops_per_second(device_name: str, dtype: torch.dtype = torch.bfloat16) -> float | None:
    """Dense (non-sparse) bf16/fp16 tensor peak of the named accelerator."""
    if dtype not in (torch.bfloat16, torch.float16):
        return None
    n = device_name.upper()
    if "GB200" in n or "GB300" in n:
        return 2.5e15
    if "B200" in n or "B300" in n:
        return 2.25e15
    if "H100" in n or "H200" in n:
        return 835e12 if "NVL" in n else 756e12 if "PCIE" in n else 989e12
    if "A100" in n:
        return 312e12
    if "MI300X" in n or "MI325X" in n:
        return 1307.4e12
    return None


def device_peak_flops(device: torch.device, dtype: torch.dtype = torch.bfloat16) -> float | None:
    if device.type != "cuda":
        return None
    return peak_flops_per_second(torch.cuda.get_device_name(device), dtype)


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


def attention_flops_per_token(cfg, seq_len: int) -> int:
    if seq_len < 1:
        raise ValueError("seq_len must be positive.")
    if hasattr(cfg, "hc_mult"):  # each query reads its window plus at most index_topk entries
        keys = min(seq_len, cfg.sliding_window + cfg.index_topk)
        return 12 * cfg.num_hidden_layers * cfg.num_attention_heads * cfg.head_dim * keys
    return 12 * cfg.num_layers * cfg.hidden_size * seq_len


def flops_per_token(cfg, seq_len: int, lora_params: int | None = None, other_trainable: int = 0) -> float:
    n = matmul_params(cfg)
    attn = attention_flops_per_token(cfg, seq_len)
    if lora_params:
        return 4 * n + 2 * other_trainable + 6 * lora_params + attn
    return 6 * n + attn


def training_flop_metrics(*, flops_per_token: float | None, model_tokens: float, elapsed_seconds: float,
                          world_size: int, peak: float | None) -> dict[str, float]:
    """``perf/model_flops_per_token`` always; the per-GPU peak and percent MFU
    when the peak is known and the step did work."""
    if flops_per_token is None:
        return {}
    m = {"perf/model_flops_per_token": float(flops_per_token)}
    if peak is None or model_tokens <= 0 or elapsed_seconds <= 0 or world_size < 1:
        return m
    m["perf/peak_flops_per_second_per_gpu"] = peak
    m["perf/mfu"] = 100.0 * flops_per_token * model_tokens / elapsed_seconds / peak / world_size
    return m


class PerfTracker:
    def __init__(self, cfg, device, lora_rank=None, lora_params=None, dtype: torch.dtype = torch.bfloat16):
        self.cfg = cfg
        self.device = device
        self.peak = device_peak_flops(device, dtype)
        self.lora_params = lora_params
        self.seq_len = 4096

    def step_metrics(self, global_tokens: int, seconds: float, seq_len: int | None = None) -> dict[str, float]:
        seq_len = seq_len or self.seq_len
        tps = global_tokens / max(seconds, 1e-9)
        ws = int(torch.distributed.get_world_size()) if torch.distributed.is_initialized() else 1
        m = {
            "perf/tokens_per_second": tps,
            "perf/step_tokens_per_second": tps,
            "perf/throughput": tps,
            "perf/step_seconds": seconds,
        }
        m.update(training_flop_metrics(flops_per_token=flops_per_token(self.cfg, seq_len, self.lora_params),
                                       model_tokens=global_tokens, elapsed_seconds=seconds, world_size=ws,
                                       peak=self.peak))
        if self.device.type == "cuda":
            m["perf/peak_memory_gib"] = torch.cuda.max_memory_allocated(self.device) / 2**30
        return m
