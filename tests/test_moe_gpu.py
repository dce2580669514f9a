"""MoE block on the GPU (grouped tcgen05 expert GEMMs, hand-written backward)
against a float32 autograd reference that uses the same expert choices (the
top-k of near-tied bf16 router logits may legitimately differ from fp32)."""

import pytest
import torch
import torch.nn.functional as F

from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.moe import MoEBlock
from wavelet_b200.models.qwen import build_model

pytestmark = pytest.mark.gpu


def _ref(x2, P, topi, cfg):
    x = x2.float().requires_grad_(True)
    Wn = P["post_norm"].float().requires_grad_(True)
    Wr = P["router_w"].float().requires_grad_(True)
    Wg = P["exp_gu_w"].float().requires_grad_(True)
    Wd = P["exp_down_w"].float().requires_grad_(True)
    h = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * Wn
    probs = torch.softmax(h @ Wr.t(), -1)
    w = probs.gather(1, topi)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    out = x.clone()
    Ie = cfg.moe_intermediate_size
    for slot in range(topi.shape[1]):
        for e in range(cfg.num_experts):
            tok = (topi[:, slot] == e).nonzero().flatten()
            if tok.numel() == 0:
                continue
            gu = h[tok] @ Wg[e].t()
            y = (F.silu(gu[:, :Ie]) * gu[:, Ie:]) @ Wd[e].t()
            out = out.index_add(0, tok, y * w[tok, slot : slot + 1])
    return out, (x, Wn, Wr, Wg, Wd)


def test_moe_block_matches_reference(cuda_ext):
    torch.manual_seed(0)
    cfg = PRESETS["tiny-moe-gpu"]
    m = build_model(cfg, "cuda", torch.bfloat16, seed=1)
    layer = m.layers[0]
    P, G = layer.P, layer.G
    blk = MoEBlock(cfg, 0)
    T = 300
    x2 = (torch.randn(T, cfg.hidden_size, device="cuda")).to(torch.bfloat16)
    out, cache = blk.forward(x2, P, save=True)
    dout = torch.randn(T, cfg.hidden_size, device="cuda").to(torch.bfloat16)
    m.flat.zero_grad()
    dx = blk.backward(dout, x2, cache, P, G)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    ref_out, leaves = _ref(x2, P, cache["topi"], cfg)
    torch.testing.assert_close(out.float(), ref_out.detach(), rtol=3e-2, atol=3e-2)
    ref_out.backward(dout.float())
    x, Wn, Wr, Wg, Wd = leaves
    for got, want, name in ((dx.float(), x.grad, "dx"), (G["post_norm"], Wn.grad, "post_norm"),
                            (G["router_w"], Wr.grad, "router"), (G["exp_gu_w"], Wg.grad, "gu"),
                            (G["exp_down_w"], Wd.grad, "down")):
        cos = F.cosine_similarity(got.flatten().float(), want.flatten(), dim=0).item()
        rel = ((got.float() - want).norm() / (want.norm() + 1e-12)).item()
        assert cos > 0.99 and rel < 0.1, (name, cos, rel)
