"""Qwen3-MoE sparse MLP block: router, top-k routing, expert SwiGLU FFNs.

GPU path (``MoEBlock``), inside the recompute-based decoder layer:

    h2 = rmsnorm(x2)                         logits = h2 Wr^T            (fp32)
    p  = softmax(logits); (w, e) = topk(p)   w /= sum(w) if norm_topk_prob
    token copies are laid out expert-by-expert in a buffer whose expert
    segments are padded to 128 rows, so every 128-row GEMM tile belongs to one
    expert; the expert FFNs run as grouped tcgen05 GEMMs (M-grouped: the tile's
    expert selects its weight block) and the weight gradients as K-grouped
    GEMMs over each expert's token segment, accumulated in fp32 straight into
    the flat gradient buffer.
    out = x2 + sum_k w_k * expert_{e_k}(h2)

Auxiliary load-balance loss (Switch form, ``router_aux_loss_coef``):
    L_aux = E * sum_e f_e * P_e,  f_e = share of the T*k assignments routed to
    e, P_e = mean router probability of e; its gradient (f_e treated as a
    constant) is injected into the router gradient in the block's backward,
    scaled by ``aux_loss_scale`` (set by the trainer per micro-batch).

``moe_reference`` is the float32 eager formulation (the CPU path and the
oracle), matching HF ``Qwen3MoeSparseMoeBlock`` used by the reference
(trainer/moe.py:241-272, routing metrics :387-436).

Expert parallelism (EP) exchanges token copies with NCCL all-to-all
(``ep_group``); the counts are exchanged first so every rank knows its
receive layout (trainer/moe.py:174-233).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref

PAD = 128


def moe_reference(h: torch.Tensor, router_w: torch.Tensor, gu_w: torch.Tensor, down_w: torch.Tensor, cfg):
    """Returns (out [T, H], aux_loss scalar, stats)."""
    T = h.shape[0]
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    logits = h.float() @ router_w.float().t()
    probs = torch.softmax(logits, -1)
    topv, topi = torch.topk(probs, k, dim=-1)
    if cfg.norm_topk_prob:
        topv = topv / topv.sum(-1, keepdim=True)
    out = torch.zeros(T, h.shape[1], dtype=torch.float32, device=h.device)
    for e in range(E):
        sel = (topi == e)
        tok = sel.any(-1).nonzero().flatten()
        if tok.numel() == 0:
            continue
        w = (topv * sel).sum(-1)[tok]
        y = ref.swiglu(h[tok].float() @ gu_w[e].float().t()) @ down_w[e].float().t()
        out.index_add_(0, tok, y * w[:, None])
    counts = torch.bincount(topi.flatten(), minlength=E).float()
    f = counts / (T * k)
    P = probs.mean(0)
    aux = E * (f * P).sum()
    return out.to(h.dtype), aux, {"counts": counts}


class Routing:
    """Padded expert layout of the T*k token copies of a micro-batch."""

    def __init__(self, topi: torch.Tensor, E: int, pad: int = PAD):
        T, k = topi.shape
        dev = topi.device
        flat = topi.reshape(-1)
        counts = torch.bincount(flat, minlength=E)
        cl = counts.tolist()  # host sync: the padded layout sizes the grouped GEMM grid
        padded = [(c + pad - 1) // pad * pad for c in cl]
        starts = [0] * E
        acc = 0
        for e in range(E):
            starts[e] = acc
            acc += padded[e]
        self.R = max(acc, pad)
        self.counts = counts
        order = torch.argsort(flat, stable=True)
        rank_in = torch.empty_like(order)
        cum = torch.zeros(E + 1, dtype=torch.long, device=dev)
        cum[1:] = counts.cumsum(0)
        sorted_e = flat[order]
        rank_in[order] = torch.arange(flat.numel(), device=dev) - cum[sorted_e]
        start_t = torch.tensor(starts, dtype=torch.long, device=dev)
        self.pos = start_t[flat] + rank_in  # row of each (token, slot) copy in the padded buffer
        self.tok = torch.arange(T, device=dev).repeat_interleave(k)
        tiles = []
        for e in range(E):
            tiles += [e] * (padded[e] // pad)
        if not tiles:
            tiles = [0]
        self.tile_group = torch.tensor(tiles, dtype=torch.int32, device=dev)
        self.k_start = torch.tensor(starts, dtype=torch.int32, device=dev)
        self.k_len = torch.tensor(padded, dtype=torch.int32, device=dev)
        self.E = E


class MoEBlock:
    def __init__(self, cfg, layer_idx: int):
        self.cfg = cfg
        self.layer = layer_idx
        self.ep_group = None
        self.aux_loss_scale = 0.0
        self.last_aux = None
        self.last_counts = None

    # ------------------------------------------------------------ shared
    def _route(self, h2, P):
        cfg = self.cfg
        logits = ops.gemm(h2, P["router_w"], epi=ops.EPI_F32)
        probs = torch.softmax(logits, -1)
        topv, topi = torch.topk(probs, cfg.num_experts_per_tok, dim=-1)
        s = topv.sum(-1, keepdim=True)
        w = topv / s if cfg.norm_topk_prob else topv
        return probs, topv, topi, s, w

    def _experts(self, h2, P, rt: Routing):
        cfg = self.cfg
        E, H, Ie = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
        xs = torch.zeros(rt.R, H, device=h2.device, dtype=h2.dtype)
        xs.index_copy_(0, rt.pos, h2.index_select(0, rt.tok))
        m = ops.ext()
        gu = torch.empty(rt.R, 2 * Ie, device=h2.device, dtype=h2.dtype)
        m.gemm_grouped(xs, False, P["exp_gu_w"].view(E * 2 * Ie, H), False, gu, 1, rt.R, 2 * Ie, H, rt.tile_group,
                       2 * Ie, E * 2 * Ie, None, None, E, ops.EPI_BF16, 1.0)
        a = ops.swiglu_fwd(gu)
        y = torch.empty(rt.R, H, device=h2.device, dtype=h2.dtype)
        m.gemm_grouped(a, False, P["exp_down_w"].view(E * H, Ie), False, y, 1, rt.R, H, Ie, rt.tile_group, H, E * H,
                       None, None, E, ops.EPI_BF16, 1.0)
        return xs, gu, a, y

    # ------------------------------------------------------------ forward
    def forward(self, x2, P, save: bool):
        cfg = self.cfg
        T = x2.shape[0]
        k = cfg.num_experts_per_tok
        h2, rstd2, _ = ops.rmsnorm_fwd(x2, P["post_norm"], cfg.rms_eps)
        probs, topv, topi, s, w = self._route(h2, P)
        rt = Routing(topi, cfg.num_experts)
        xs, gu, a, y = self._experts(h2, P, rt)
        contrib = y.index_select(0, rt.pos).float() * w.reshape(-1, 1)
        out = (x2.float() + contrib.view(T, k, -1).sum(1)).to(x2.dtype)
        f = rt.counts.float() / (T * k)
        self.last_aux = float(cfg.num_experts * (f * probs.mean(0)).sum())
        self.last_counts = rt.counts
        cache = None
        if save:
            cache = dict(h2=h2, rstd2=rstd2, probs=probs, topv=topv, topi=topi, s=s, w=w, rt=rt, xs=xs, gu=gu, a=a, y=y, f=f)
        return out, cache

    # ------------------------------------------------------------ backward
    def backward(self, dout, x2, c, P, G):
        cfg = self.cfg
        E, H, Ie, k = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts_per_tok
        T = x2.shape[0]
        rt: Routing = c["rt"]
        m = ops.ext()
        dout_rows = dout.index_select(0, rt.tok)  # [T*k, H]
        w = c["w"].reshape(-1, 1)
        dy = torch.zeros(rt.R, H, device=dout.device, dtype=dout.dtype)
        dy.index_copy_(0, rt.pos, (dout_rows.float() * w).to(dout.dtype))
        dw = (dout_rows.float() * c["y"].index_select(0, rt.pos).float()).sum(-1).view(T, k)
        # down projection
        da = torch.empty(rt.R, Ie, device=dout.device, dtype=dout.dtype)
        m.gemm_grouped(dy, False, P["exp_down_w"].view(E * H, Ie), True, da, 1, rt.R, Ie, H, rt.tile_group, H, E * H,
                       None, None, E, ops.EPI_BF16, 1.0)
        if G.get("exp_down_w") is not None:
            m.gemm_grouped(dy, True, c["a"], True, G["exp_down_w"].view(E * H, Ie), 2, H, Ie, rt.R, None, 0, 0,
                           rt.k_start, rt.k_len, E, ops.EPI_F32_ACC, 1.0)
        dgu = ops.swiglu_bwd(c["gu"], da)
        del da
        if G.get("exp_gu_w") is not None:
            m.gemm_grouped(dgu, True, c["xs"], True, G["exp_gu_w"].view(E * 2 * Ie, H), 2, 2 * Ie, H, rt.R, None, 0,
                           0, rt.k_start, rt.k_len, E, ops.EPI_F32_ACC, 1.0)
        dxs = torch.empty(rt.R, H, device=dout.device, dtype=dout.dtype)
        m.gemm_grouped(dgu, False, P["exp_gu_w"].view(E * 2 * Ie, H), True, dxs, 1, rt.R, H, 2 * Ie, rt.tile_group,
                       2 * Ie, E * 2 * Ie, None, None, E, ops.EPI_BF16, 1.0)
        del dgu
        dh2 = torch.zeros(T, H, device=dout.device, dtype=torch.float32)
        dh2.index_add_(0, rt.tok, dxs.index_select(0, rt.pos).float())
        # router: top-k weights (optionally renormalised) and the aux loss
        if cfg.norm_topk_prob:
            wv = c["w"]
            dv = (dw - (dw * wv).sum(-1, keepdim=True)) / c["s"]
        else:
            dv = dw
        probs = c["probs"]
        dprobs = torch.zeros_like(probs).scatter_(1, c["topi"], dv)
        if self.aux_loss_scale:
            dprobs += self.aux_loss_scale * cfg.num_experts * c["f"][None, :] / T
        dlogits = probs * (dprobs - (dprobs * probs).sum(-1, keepdim=True))
        dl16 = dlogits.to(dout.dtype).contiguous()
        if G.get("router_w") is not None:
            ops.gemm(dl16, c["h2"], a_mn=True, b_mn=True, out=G["router_w"], epi=ops.EPI_F32_ACC)
        dh2 += ops.gemm(dl16, P["router_w"], b_mn=True).float()
        return ops.rmsnorm_bwd(x2, P["post_norm"], c["rstd2"], dh2.to(dout.dtype), dres=dout, dw=G.get("post_norm"))

    # ------------------------------------------------------------ generator
    @torch.no_grad()
    def infer(self, h2, x, P):
        cfg = self.cfg
        T = h2.shape[0]
        k = cfg.num_experts_per_tok
        if not h2.is_cuda:
            out, _, _ = moe_reference(h2, P["router_w"], P["exp_gu_w"], P["exp_down_w"], cfg)
            return x + out
        probs, topv, topi, s, w = self._route(h2, P)
        rt = Routing(topi, cfg.num_experts)
        _, _, _, y = self._experts(h2, P, rt)
        contrib = y.index_select(0, rt.pos).float() * w.reshape(-1, 1)
        return (x.float() + contrib.view(T, k, -1).sum(1)).to(x.dtype)
