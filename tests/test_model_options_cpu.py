"""Model-section options that used to be accepted without effect."""

import pytest
import torch

from wavelet_b200.configs.config import FSDPConfig, ModelConfig
from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper
from wavelet_b200.trainer.engine import Engine
from wavelet_b200.trainer.model_options import apply_model_options


def _moe_preset():
    return PRESETS["tiny-moe"]


def test_freeze_moe_router_keeps_router_fixed_under_decay():
    from wavelet_b200.data.fake import synthetic_sft_microbatches

    cfg = _moe_preset()
    m = build_model(cfg, "cpu", torch.float32, seed=3)
    m.fused_cpu = True
    apply_model_options(m, ModelConfig(freeze_moe_router=True))
    routers = [n for n in m.flat.names() if n.endswith(".router_w")]
    before = {n: m.flat.view(n).clone() for n in m.flat.names()}
    eng = Engine(m, AdamWHyper(lr=1e-2, weight_decay=0.1, max_grad_norm=1.0))
    (b,) = synthetic_sft_microbatches(1, 32, cfg.vocab_size, seed=1)
    eng.sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    eng.optimizer_step(1e-2)
    for n in routers:
        assert torch.equal(m.flat.view(n), before[n]), n
    moved = [n for n in m.flat.names() if n not in routers and not torch.equal(m.flat.view(n), before[n])]
    assert moved  # everything else trains


def test_freeze_moe_router_on_dense_model_is_an_error():
    m = build_model(PRESETS["tiny"], "cpu", torch.float32, seed=3)
    with pytest.raises(ValueError, match="freeze_moe_router"):
        apply_model_options(m, ModelConfig(freeze_moe_router=True))


def test_router_dtype_and_matmul_precision_and_notes():
    cfg = _moe_preset()
    m = build_model(cfg, "cpu", torch.float32, seed=3)
    old = torch.get_float32_matmul_precision()
    try:
        apply_model_options(m, ModelConfig(moe_router_dtype="float32", matmul_precision="medium"))
        assert torch.get_float32_matmul_precision() == "medium"
        assert all(not l.moe.router_logits_bf16 for l in m.layers if l.moe is not None)
        notes = apply_model_options(m, ModelConfig(moe_router_dtype="none", meta_device_init=True),
                                    FSDPConfig(reshard_after_forward=False, impl="fsdp2"))
        assert all(l.moe.router_logits_bf16 for l in m.layers if l.moe is not None)
        assert any("meta_device_init" in n for n in notes)
        assert any("reshard_after_forward" in n for n in notes)
    finally:
        torch.set_float32_matmul_precision(old)
