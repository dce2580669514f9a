"""Eager DeepSeek-V4: all three attention types with packed-document
isolation, hyper-connections, hash / top-k routing, native checkpoints with
fp32-sensitive tensors, and conversion from / to the published layout
(including FP8 and MXFP4 dequantization)."""

import pytest
import torch

from wavelet_b200.models.deepseek_v4 import DeepseekV4Config, DeepseekV4ForCausalLM
from wavelet_b200.models.deepseek_v4.attention import Attention, PackedLayout
from wavelet_b200.models.deepseek_v4.convert import (convert_checkpoint, dequantize, native_to_raw, raw_to_native,
                                                     unpack_mxfp4)
from wavelet_b200.models.deepseek_v4.layers import DualRotary, sinkhorn


def _cfg(**over):
    kw = dict(vocab_size=16, hidden_size=8, num_hidden_layers=3, num_attention_heads=2, head_dim=4, q_lora_rank=4,
              partial_rotary_factor=1.0,
              layer_types=["sliding_attention", "compressed_sparse_attention", "heavily_compressed_attention"],
              compress_rates={"compressed_sparse_attention": 2, "heavily_compressed_attention": 4},
              sliding_window=4, o_groups=2, o_lora_rank=2, index_n_heads=2, index_head_dim=4, index_topk=2,
              moe_intermediate_size=8, n_routed_experts=2, num_experts_per_tok=1, num_hash_layers=1, hc_mult=2,
              max_position_embeddings=16)
    kw.update(over)
    return DeepseekV4Config(**kw)


IDS = torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8]])


def test_forward_backward_and_native_roundtrip(tmp_path):
    torch.manual_seed(11)
    m = DeepseekV4ForCausalLM(_cfg()).eval()
    with torch.no_grad():
        ref = m(IDS).logits
    assert ref.shape == (1, 8, 16)
    m.save_pretrained(tmp_path)
    back = DeepseekV4ForCausalLM.from_pretrained(tmp_path).eval()
    assert back.config.wavelet_checkpoint_format == "deepseek_v4_native_v1"
    with torch.no_grad():
        torch.testing.assert_close(back(IDS).logits, ref, atol=1e-6, rtol=1e-6)
    t = DeepseekV4ForCausalLM(_cfg())
    loss = t(IDS, labels=IDS).loss
    loss.backward()
    assert torch.isfinite(loss) and t.model.embed_tokens.weight.grad is not None
    # the indexer is selection only: no gradients, not trainable
    ix = t.model.layers[1].self_attn.compressor.indexer
    assert all(not p.requires_grad for p in ix.parameters())


@pytest.mark.parametrize("kind", ["sliding_attention", "compressed_sparse_attention", "heavily_compressed_attention"])
def test_packed_documents_are_isolated(kind):
    torch.manual_seed(7)
    cfg = _cfg(num_hidden_layers=1, layer_types=[kind], num_hash_layers=0)
    rot = DualRotary(cfg)
    att = Attention(cfg, 0)
    h = torch.randn(8, cfg.hidden_size, requires_grad=True)
    both = att(h, PackedLayout.build(rot, torch.tensor([3, 5]), torch.float32, "cpu"))
    both.square().mean().backward()
    assert torch.isfinite(h.grad).all()
    with torch.no_grad():
        a = att(h[:3], PackedLayout.build(rot, torch.tensor([3]), torch.float32, "cpu"))
        b = att(h[3:], PackedLayout.build(rot, torch.tensor([5]), torch.float32, "cpu"))
    torch.testing.assert_close(both.detach(), torch.cat([a, b]), atol=1e-5, rtol=1e-5)


def test_window_and_entry_layout():
    cfg = _cfg()
    lay = PackedLayout.build(DualRotary(cfg), torch.tensor([3, 9]), torch.float32, "cpu")
    assert lay.positions.tolist() == [0, 1, 2] + list(range(9))
    # token 11 (position 8 of document 2) sees tokens 8..11; token 4 (position 1) sees 3, 4
    assert lay.window[11].tolist() == [8, 9, 10, 11]
    assert lay.window[4].tolist()[:2] == [3, 4] and set(lay.window[4].tolist()[2:]) == {-1}
    el = lay.entries[4]  # rate 4: document 1 has none, document 2 has entries at tokens 3..6 and 7..10
    assert el.tokens.tolist() == [[3, 4, 5, 6], [7, 8, 9, 10]] and el.doc_first.tolist() == [0, 0]


def test_sinkhorn_is_doubly_stochastic_and_mhc_gates():
    m = sinkhorn(torch.randn(5, 4, 4) * 3, 20, 1e-6)
    # the last Sinkhorn half-step normalises columns exactly; rows converge
    torch.testing.assert_close(m.sum(-2), torch.ones(5, 4), atol=1e-4, rtol=0)
    torch.testing.assert_close(m.sum(-1), torch.ones(5, 4), atol=2e-2, rtol=0)
    torch.manual_seed(0)
    mdl = DeepseekV4ForCausalLM(_cfg())
    post, comb, x = mdl.model.layers[0].attn_hc(torch.randn(6, 2, 8))
    assert ((post >= 0) & (post <= 2)).all() and x.shape == (6, 8) and comb.shape == (6, 2, 2)


def test_hash_and_topk_routing():
    torch.manual_seed(3)
    mdl = DeepseekV4ForCausalLM(_cfg(n_routed_experts=4, num_experts_per_tok=2))
    moe0, moe1 = mdl.model.layers[0].mlp, mdl.model.layers[1].mlp
    assert moe0.hashed and not moe1.hashed
    moe0.router.tid2eid.copy_(torch.tensor([[1, 3]] * 16))
    x = torch.randn(5, 8)
    w, chosen = moe0.router(x, moe0.router.tid2eid[torch.arange(5)])
    assert chosen.tolist() == [[1, 3]] * 5
    torch.testing.assert_close(w.sum(-1), torch.full((5,), mdl.config.routed_scaling_factor))
    # a large selection bias wins the top-k without changing the weights' formula
    moe1.router.selection_bias.copy_(torch.tensor([0.0, 0.0, 100.0, 100.0]))
    _, chosen = moe1.router(x)
    assert sorted(chosen[0].tolist()) == [2, 3]
    moe1.train()
    moe1(x)
    assert moe1.tokens_per_expert.sum() == 10
    moe1.balance_(0.5)
    assert moe1.router.selection_bias[2] < 100.0 and moe1.tokens_per_expert.sum() == 0


def test_bf16_keeps_sensitive_tensors_fp32(tmp_path):
    m = DeepseekV4ForCausalLM(_cfg())
    with torch.no_grad():
        m.model.layers[0].self_attn.sinks.fill_(0.123456789)
        m.model.layers[1].mlp.router.selection_bias.fill_(0.314159265)
    m.save_pretrained(tmp_path)
    b = DeepseekV4ForCausalLM.from_pretrained(tmp_path, dtype=torch.bfloat16)
    assert b.model.layers[0].self_attn.sinks.dtype == torch.float32
    assert b.model.layers[0].self_attn.sinks[0].item() == torch.tensor(0.123456789).item()  # exact fp32 value
    assert b.model.layers[1].mlp.router.selection_bias.dtype == torch.float32
    assert b.model.layers[0].attn_hc.fn.dtype == torch.float32 and b.lm_head.weight.dtype == torch.bfloat16
    assert DeepseekV4ForCausalLM.keep_in_fp32_for_weight_transfer("model.layers.1.self_attn.compressor.position_bias")
    assert not DeepseekV4ForCausalLM.keep_in_fp32_for_weight_transfer("lm_head.weight")
    out = b(IDS, labels=IDS)
    out.loss.backward()
    assert torch.isfinite(out.loss)


def test_raw_native_conversion(tmp_path):
    torch.manual_seed(5)
    m = DeepseekV4ForCausalLM(_cfg()).eval()
    native = m.state_dict()
    raw = native_to_raw(native)
    assert "layers.0.attn.attn_sink" in raw and "layers.1.ffn.experts.1.w2.weight" in raw
    assert "layers.1.attn.indexer.compressor.ape" in raw
    back = raw_to_native(raw)
    assert set(back) == set(native)
    for k, v in native.items():
        torch.testing.assert_close(back[k], v)
    # full directory round trip preserves the logits
    with torch.no_grad():
        ref = m(IDS).logits
    m.save_pretrained(tmp_path / "native")
    convert_checkpoint(tmp_path / "native", tmp_path / "raw", to_raw=True)
    with pytest.raises(ValueError, match="converted native checkpoint"):
        DeepseekV4ForCausalLM.from_pretrained(tmp_path / "raw")
    convert_checkpoint(tmp_path / "raw", tmp_path / "again")
    with torch.no_grad():
        torch.testing.assert_close(DeepseekV4ForCausalLM.from_pretrained(tmp_path / "again").eval()(IDS).logits, ref,
                                   atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("corruption", ["missing", "shape"])
def test_converter_rejects_corrupt_checkpoints(tmp_path, corruption):
    from safetensors.torch import load_file, save_file

    DeepseekV4ForCausalLM(_cfg()).save_pretrained(tmp_path / "src")
    w = load_file(str(tmp_path / "src" / "model.safetensors"))
    if corruption == "missing":
        del w["model.embed_tokens.weight"]
    else:
        w["model.embed_tokens.weight"] = w["model.embed_tokens.weight"][:1]
    save_file(w, str(tmp_path / "src" / "model.safetensors"))
    with pytest.raises(ValueError, match="missing|shape"):
        convert_checkpoint(tmp_path / "src", tmp_path / "dst", to_raw=True)
    assert not (tmp_path / "dst").exists()


def test_dequantize_fp8_and_mxfp4():
    w8 = torch.tensor([[1.0, -2.0, 0.5, 4.0]] * 2).to(torch.float8_e4m3fn)
    s = torch.tensor([[2.0, 0.5]])
    torch.testing.assert_close(dequantize(w8, s).float(), torch.tensor([[2.0, -4.0, 0.25, 2.0]] * 2))
    packed = torch.tensor([[0x21, 0xF8]], dtype=torch.uint8).view(torch.int8)  # codes 1,2 | 8,15
    assert unpack_mxfp4(packed).tolist() == [[0.5, 1.0, -0.0, -6.0]]
    torch.testing.assert_close(dequantize(packed, torch.tensor([[4.0]])).float(), torch.tensor([[2.0, 4.0, 0.0, -24.0]]))
    state = {"layers.0.attn.wq_a.weight": w8}
    with pytest.raises(ValueError, match="scale"):
        raw_to_native(state)


def test_position_validation():
    m = DeepseekV4ForCausalLM(_cfg())
    with pytest.raises(ValueError):
        m(IDS, position_ids=torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8]]))
    with pytest.raises(ValueError):
        m(IDS, position_ids=torch.tensor([[0, 1, 2, 4, 5, 6, 7, 8]]))
    # two packed documents via restarting positions
    out = m(IDS, position_ids=torch.tensor([[0, 1, 2, 0, 1, 2, 3, 4]]))
    assert out.logits.shape == (1, 8, 16)


def test_legacy_compress_ratios_and_yarn():
    cfg = DeepseekV4Config(num_hidden_layers=3, compress_ratios=[0, 4, 128],
                           rope_scaling={"type": "yarn", "factor": 16.0, "original_max_position_embeddings": 65536})
    assert cfg.layer_types == ["sliding_attention", "compressed_sparse_attention", "heavily_compressed_attention"]
    assert cfg.rope_parameters["compress"]["rope_type"] == "yarn"
    assert cfg.rope_parameters["main"]["rope_type"] == "default"
    rot = DualRotary(cfg)
    assert getattr(rot, "compress_inv_freq").shape == (32,)
    # long wavelengths are interpolated by the factor, short ones kept
    base = 1.0 / 160000.0 ** (torch.arange(0, 64, 2).double() / 64)
    assert torch.allclose(rot.compress_inv_freq[0].double(), base[0], rtol=1e-5)
    assert torch.allclose(rot.compress_inv_freq[-1].double(), base[-1] / 16.0, rtol=1e-5)
