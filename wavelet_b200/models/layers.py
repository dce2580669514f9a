"""Decoder-layer forward/backward on the GPU kernels, with full recompute.

One decoder layer is a single autograd node (``DecoderLayerFn``).  Its forward
keeps only the layer input; its backward recomputes the layer and runs the
hand-written backward, writing every weight gradient directly into the fp32
flat gradient buffer:

    h1  = rmsnorm(x)                     qkv = h1 Wqkv^T (+ b)
    q,k = rope(qk_norm(q, k))            att = attention(q, k, v)
    x2  = x + att Wo^T   (residual fused in the GEMM epilogue)
    h2  = rmsnorm(x2)                    gu  = h2 Wgu^T
    a   = silu(g) * u                    out = x2 + a Wd^T (residual fused)

This is the activation-checkpointed Qwen2/Qwen3 decoder layer that the
reference runs as HF modules under ``checkpoint_wrapper``
(trainer/model.py:1341-1429) with Liger/FA kernels; here it is a fixed kernel
sequence: 7 GEMMs forward (3 attention + 2 MLP... counted per weight), every
one of them on the tcgen05 GEMM.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from .. import ops
from ..ops.attention import attention_bwd, attention_fwd
from .config import ArchConfig


@dataclass
class BatchCtx:
    """Per-micro-batch metadata shared by every layer."""

    pos: torch.Tensor  # int32 [T]
    cu_seqlens: torch.Tensor  # int32 [n+1]
    max_seqlen: int
    inv_freq: torch.Tensor  # fp32 [head_dim/2]


def _dense_mlp_fwd(x2, P, c, save):
    h2, rstd2, _ = ops.rmsnorm_fwd(x2, P["post_norm"], c.rms_eps)
    gu = ops.gemm(h2, P["gu_w"])
    a = ops.swiglu_fwd(gu)
    out = ops.gemm(a, P["down_w"], res=x2)
    return out, (dict(h2=h2, rstd2=rstd2, gu=gu, a=a) if save else None)


def layer_fwd(x: torch.Tensor, P: dict[str, torch.Tensor], cfg: ArchConfig, b: BatchCtx, save: bool,
              moe: Any = None):
    T = x.shape[0]
    nq, nk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    h1, rstd1, _ = ops.rmsnorm_fwd(x, P["in_norm"], cfg.rms_eps)
    qkv = ops.gemm(h1, P["qkv_w"], bias=P.get("qkv_b"))
    qkv_pre = qkv.clone() if (save and cfg.qk_norm) else None
    rstd_qk = ops.qk_norm_rope_(qkv, nq, nk, b.pos, b.inv_freq, P.get("q_norm"), P.get("k_norm"), cfg.rms_eps)
    q = qkv[:, : nq * hd].view(T, nq, hd)
    k = qkv[:, nq * hd : (nq + nk) * hd].view(T, nk, hd)
    v = qkv[:, (nq + nk) * hd :].view(T, nk, hd)
    att, lse = attention_fwd(q, k, v, b.cu_seqlens, b.max_seqlen, True)
    att2 = att.view(T, nq * hd)
    x2 = ops.gemm(att2, P["o_w"], res=x)
    if moe is None:
        out, mc = _dense_mlp_fwd(x2, P, cfg, save)
    else:
        out, mc = moe.forward(x2, P, save)
    cache = None
    if save:
        cache = dict(h1=h1, rstd1=rstd1, qkv=qkv, qkv_pre=qkv_pre, rstd_qk=rstd_qk, att=att, lse=lse, x2=x2, mlp=mc)
    return out, cache


def layer_bwd(dout: torch.Tensor, x: torch.Tensor, c: dict, P: dict[str, torch.Tensor],
              G: dict[str, torch.Tensor], cfg: ArchConfig, b: BatchCtx, moe: Any = None):
    T = x.shape[0]
    nq, nk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    dout = dout.contiguous()
    mc = c["mlp"]
    if moe is None:
        # out = x2 + a Wd^T
        da = ops.gemm(dout, P["down_w"], b_mn=True)
        ops.gemm(dout, mc["a"], a_mn=True, b_mn=True, out=G["down_w"], epi=ops.EPI_F32_ACC)
        dgu = ops.swiglu_bwd(mc["gu"], da)
        del da
        ops.gemm(dgu, mc["h2"], a_mn=True, b_mn=True, out=G["gu_w"], epi=ops.EPI_F32_ACC)
        dh2 = ops.gemm(dgu, P["gu_w"], b_mn=True)
        del dgu
        dx2 = ops.rmsnorm_bwd(c["x2"], P["post_norm"], mc["rstd2"], dh2, dres=dout, dw=G["post_norm"])
        del dh2
    else:
        dx2 = moe.backward(dout, c["x2"], mc, P, G)
    # x2 = x + att Wo^T
    datt = ops.gemm(dx2, P["o_w"], b_mn=True)
    ops.gemm(dx2, c["att"].view(T, nq * hd), a_mn=True, b_mn=True, out=G["o_w"], epi=ops.EPI_F32_ACC)
    qkv = c["qkv"]
    q = qkv[:, : nq * hd].view(T, nq, hd)
    k = qkv[:, nq * hd : (nq + nk) * hd].view(T, nk, hd)
    v = qkv[:, (nq + nk) * hd :].view(T, nk, hd)
    dq, dk, dv = attention_bwd(datt.view(T, nq, hd), q, k, v, c["att"], c["lse"], b.cu_seqlens, b.max_seqlen, True)
    del datt
    dqkv = torch.cat([dq.reshape(T, -1), dk.reshape(T, -1), dv.reshape(T, -1)], 1)
    del dq, dk, dv
    qkv_pre = c["qkv_pre"] if c["qkv_pre"] is not None else qkv
    ops.ext().qk_norm_rope_bwd(
        dqkv, qkv_pre, nq, nk, b.pos, b.inv_freq, P.get("q_norm"), P.get("k_norm"), c["rstd_qk"],
        G.get("q_norm"), G.get("k_norm"),
    )
    if "qkv_b" in P:
        G["qkv_b"].add_(dqkv.float().sum(0))
    ops.gemm(dqkv, c["h1"], a_mn=True, b_mn=True, out=G["qkv_w"], epi=ops.EPI_F32_ACC)
    dh1 = ops.gemm(dqkv, P["qkv_w"], b_mn=True)
    del dqkv
    dx = ops.rmsnorm_bwd(x, P["in_norm"], c["rstd1"], dh1, dres=dx2, dw=G["in_norm"])
    return dx


class DecoderLayerFn(torch.autograd.Function):
    """Activation-checkpointed decoder layer: saves x, recomputes in backward."""

    @staticmethod
    def forward(ctx, x, anchor, layer):
        with torch.no_grad():
            out, _ = layer_fwd(x, layer.P, layer.cfg, layer.batch, save=False, moe=layer.moe)
        ctx.save_for_backward(x)
        ctx.layer = layer
        return out

    @staticmethod
    def backward(ctx, dout):
        (x,) = ctx.saved_tensors
        layer = ctx.layer
        with torch.no_grad():
            _, cache = layer_fwd(x, layer.P, layer.cfg, layer.batch, save=True, moe=layer.moe)
            dx = layer_bwd(dout, x, cache, layer.P, layer.G, layer.cfg, layer.batch, moe=layer.moe)
        return dx, None, None


class EmbeddingFn(torch.autograd.Function):
    """Row gather whose backward scatter-adds straight into the fp32 grad."""

    @staticmethod
    def forward(ctx, ids, anchor, table, gtable):
        ctx.save_for_backward(ids)
        ctx.gtable = gtable
        return ops.embedding_fwd(table, ids)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        if ctx.gtable is not None:
            ops.embedding_bwd_(dy, ids, ctx.gtable)
        return None, None, None, None


class FinalNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, gw, eps):
        y, rstd, _ = ops.rmsnorm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        ctx.gw = gw
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx = ops.rmsnorm_bwd(x, w, rstd, dy, dw=ctx.gw)
        return dx, None, None, None
