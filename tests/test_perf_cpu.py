"""FLOP / MFU accounting against the values the reference's own tests pin
(tests/test_perf.py of the reference: a 2-layer dense toy, a MoE toy, LoRA
cost, the peak table and percent MFU)."""

import pytest
import torch

from wavelet_b200.models.config import ArchConfig
from wavelet_b200.trainer.perf import (PerfTracker, attention_flops_per_token, flops_per_token, matmul_params,
                                       peak_flops_per_second, training_flop_metrics)

DENSE = ArchConfig(arch="qwen3", vocab_size=32, hidden_size=8, intermediate_size=16, num_layers=2, num_heads=2,
                   num_kv_heads=1, head_dim=4)


def test_dense_estimate():
    assert matmul_params(DENSE) == 1_408
    assert attention_flops_per_token(DENSE, 10) == 1_920
    assert flops_per_token(DENSE, 10) == 10_368
    assert flops_per_token(DENSE, 20) == 12_288
    with pytest.raises(ValueError, match="seq_len must be positive"):
        flops_per_token(DENSE, 0)


def test_moe_counts_active_experts_and_router():
    # 4 layers, the first dense (mlp_only_layers), top-2 of 8 experts of width 12
    moe = ArchConfig(arch="qwen3_moe", vocab_size=32, hidden_size=8, intermediate_size=16, num_layers=4,
                     num_heads=2, num_kv_heads=1, head_dim=4, num_experts=8, num_experts_per_tok=2,
                     moe_intermediate_size=12, mlp_only_layers=(0,))
    # the reference's 4_192 includes a 12-wide shared expert per sparse layer (3 * 288); Qwen3-MoE has none
    assert matmul_params(moe) == 4_192 - 3 * 3 * 12 * 8


def test_lora_uses_frozen_base_backward_cost():
    assert flops_per_token(DENSE, 10, lora_params=7) == 7_594
    assert flops_per_token(DENSE, 10, lora_params=7, other_trainable=5) == 7_594 + 10


@pytest.mark.parametrize(("name", "peak"), [
    ("NVIDIA A100-SXM4-80GB", 312e12), ("NVIDIA H100 PCIe", 756e12), ("NVIDIA H100 NVL", 835e12),
    ("NVIDIA H200", 989e12), ("NVIDIA B200", 2.25e15), ("NVIDIA GB200", 2.5e15), ("AMD Instinct MI325X", 1307.4e12),
])
def test_peak_table(name, peak):
    assert peak_flops_per_second(name, torch.bfloat16) == peak
    assert peak_flops_per_second(name, torch.float32) is None


def test_percent_mfu_and_unknown_hardware():
    m = training_flop_metrics(flops_per_token=1_000, model_tokens=2_000, elapsed_seconds=0.5, world_size=2,
                              peak=peak_flops_per_second("NVIDIA A100"))
    assert m["perf/model_flops_per_token"] == 1_000
    assert m["perf/peak_flops_per_second_per_gpu"] == 312e12
    assert m["perf/mfu"] == pytest.approx(100 * 4e6 / (2 * 312e12))
    assert training_flop_metrics(flops_per_token=1_000, model_tokens=2_000, elapsed_seconds=0.5, world_size=1,
                                 peak=peak_flops_per_second("Unknown Accelerator")) == {"perf/model_flops_per_token": 1_000.0}


def test_tracker_on_cpu_reports_throughput_without_mfu():
    t = PerfTracker(DENSE, torch.device("cpu"))
    m = t.step_metrics(1000, 0.5, seq_len=10)
    assert m["perf/tokens_per_second"] == pytest.approx(2000.0)
    assert m["perf/model_flops_per_token"] == 10_368
    assert "perf/mfu" not in m
