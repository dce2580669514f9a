"""LoRA / QLoRA plumbing on the CPU float32 path."""

from types import SimpleNamespace

import torch

from wavelet_b200.data.fake import synthetic_sft_microbatches
from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.lora import merge_adapter_into
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper
from wavelet_b200.trainer.engine import Engine

LORA = SimpleNamespace(rank=4, alpha=8.0, dropout=0.0,
                       target_modules=["q_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"])


def _hidden(m, b):
    ctx = m.batch_ctx(b.position_ids, b.cu_seqlens, b.max_seqlen)
    return m.hidden(b.input_ids, ctx)


def test_lora_starts_at_base_and_trains_only_adapters(tmp_path):
    cfg = PRESETS["tiny"]
    base = build_model(cfg, "cpu", torch.float32, seed=2)
    m = build_model(cfg, "cpu", torch.float32, seed=2, lora=LORA)
    assert m.flat.grad is None and m.lora is not None
    (b,) = synthetic_sft_microbatches(1, 64, cfg.vocab_size, seed=0, seqs_per_micro=2)
    torch.testing.assert_close(_hidden(m, b).detach(), _hidden(base, b).detach())
    base_w = m.flat.compute.detach().clone()
    eng = Engine(m, AdamWHyper(lr=1e-2))
    scale = 1.0 / float(b.loss_mask.sum())
    losses = []
    for _ in range(6):
        losses.append(eng.sft_micro_step(b, scale).item())
        eng.optimizer_step(1e-2)
    assert losses[-1] < losses[0], losses
    assert torch.equal(m.flat.compute.detach(), base_w)  # base frozen
    # off-diagonal blocks of the stacked B and the padding stay exactly zero
    lay = m.lora.layouts["qkv"]
    B = m.lora.flat.view("l0.qkv.B")
    q_lo, q_hi = 0, cfg.q_dim
    assert torch.count_nonzero(B[q_lo:q_hi, LORA.rank:]) == 0
    assert torch.count_nonzero(B[cfg.q_dim : cfg.q_dim + cfg.kv_dim]) == 0  # k_proj not targeted
    assert lay.kp == 64
    # PEFT export -> merge into a dense copy reproduces the adapted model
    m.lora.save_adapter(tmp_path / "adapter")
    dense = build_model(cfg, "cpu", torch.float32, seed=2)
    merge_adapter_into(dense, tmp_path / "adapter")
    torch.testing.assert_close(_hidden(dense, b).detach(), _hidden(m, b).detach(), rtol=1e-4, atol=1e-4)


def test_qlora_base_is_dequantized_nf4():
    cfg = PRESETS["tiny"]
    q = build_model(cfg, "cpu", torch.float32, seed=4, lora=LORA, load_in_4bit=True)
    dense = build_model(cfg, "cpu", torch.float32, seed=4)
    assert set(q.quant) == {f"l{i}.{w}" for i in range(cfg.num_layers) for w in ("qkv_w", "o_w", "gu_w", "down_w")}
    for name, nf in q.quant.items():
        w = dense.flat.view(name)
        err = (nf.dequantize(torch.float32) - w).abs().max().item()
        assert err <= 0.5 * w.abs().max().item()
    # same random init for the non-quantised tensors
    torch.testing.assert_close(q.flat.view("embed"), dense.flat.view("embed"))
    (b,) = synthetic_sft_microbatches(1, 64, cfg.vocab_size, seed=0, seqs_per_micro=2)
    eng = Engine(q, AdamWHyper(lr=1e-2))
    l0 = eng.sft_micro_step(b, 1.0 / float(b.loss_mask.sum())).item()
    eng.optimizer_step(1e-2)
    assert l0 > 0
