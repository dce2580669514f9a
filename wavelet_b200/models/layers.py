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
from ..utils import nvtx
from ..ops.attention import attention_bwd, attention_fwd
from ..parallel.context_parallel import attention_bwd as cp_attention_bwd
from ..parallel.context_parallel import attention_fwd as cp_attention_fwd
from .config import ArchConfig


@dataclass
class BatchCtx:
    """Per-micro-batch metadata shared by every layer."""

    pos: torch.Tensor  # int32 [T]
    cu_seqlens: torch.Tensor  # int32 [n+1]
    max_seqlen: int
    inv_freq: torch.Tensor  # fp32 [head_dim/2]
    cp: Any = None  # parallel.context_parallel.CPPlan: attention over the CP group's full sequences
    mm: Any = None  # processor fields of the row's images (vision-language models)


def _lin(x, w, ad, bias=None, res=None):
    """y = x W^T (+ bias + res) (+ s (x A^T) B^T with an adapter) -> (y, u)."""
    if ad is None:
        return ops.gemm(x, w, bias=bias, res=res), None
    u = ops.gemm(x, ad.A, alpha=ad.scale)
    return ops.gemm(x, w, bias=bias, res=res, a2=u, b2=ad.B), u


def _fused_tp(tp, w, ad) -> bool:
    # the fused GEMM -> all-reduce covers plain bf16 weights (no adapter / NF4)
    return tp is not None and tp.fabric is not None and ad is None and isinstance(w, torch.Tensor)


def _lin_rowpar(x, w, ad, res, tp):
    """Row-parallel linear summed over the TP ranks (+ res): one fused
    GEMM -> all-reduce over peer memory when the TP group has a fabric, else
    the GEMM (residual on TP rank 0 only) and an NCCL all-reduce."""
    if _fused_tp(tp, w, ad):
        return tp.fabric.gemm_allreduce(x, w, res=res), None
    y, u = _lin(x, w, ad, res=_res(res, tp))
    return _tp_reduce(y, tp), u


def _lin_bwd(dy, x, u, w, gw, ad, tp=None):
    """dx of ``_lin``; accumulates dW into ``gw`` (None: frozen) and the
    adapter gradients (block-diagonal dB, dA) when ``ad`` is given.  With
    ``tp`` (column-parallel weight) dx is summed over the TP ranks."""
    if gw is not None:
        ops.gemm(dy, x, a_mn=True, b_mn=True, out=gw, epi=ops.EPI_F32_ACC)
    if _fused_tp(tp, w, ad):
        return tp.fabric.gemm_allreduce(dy, w, b_mn=True)
    if ad is None:
        return _tp_reduce(ops.gemm(dy, w, b_mn=True), tp)
    if ad.GB is not None:
        ad.add_b_grad(ops.gemm(dy, u, a_mn=True, b_mn=True, epi=ops.EPI_F32))
    g = ops.gemm(dy, ad.B, b_mn=True, alpha=ad.scale)
    if ad.GA is not None:
        ops.gemm(g, x, a_mn=True, b_mn=True, out=ad.GA, epi=ops.EPI_F32_ACC)
    return _tp_reduce(ops.gemm(dy, w, b_mn=True, a2=g, b2=ad.A), tp)


def _tp_reduce(t, tp):
    """Sum the row-parallel partial products of the TP ranks (in place)."""
    if tp is not None:
        import torch.distributed as dist

        dist.all_reduce(t, group=tp.group)
    return t


def _res(x, tp):
    # under TP the residual joins the partial sums on one rank only
    return x if tp is None or tp.rank == 0 else None


def _dense_mlp_fwd(x2, P, c, save, lora, tp=None):
    h2, rstd2, _ = ops.rmsnorm_fwd(x2, P["post_norm"], c.rms_eps)
    gu, u_gu = _lin(h2, P["gu_w"], lora.get("gu"))
    a = ops.swiglu_fwd(gu)
    out, u_dn = _lin_rowpar(a, P["down_w"], lora.get("down"), x2, tp)
    return out, (dict(h2=h2, rstd2=rstd2, gu=gu, a=a, u_gu=u_gu, u_dn=u_dn) if save else None)


_NO_LORA: dict = {}


def layer_fwd(x: torch.Tensor, P: dict, cfg: ArchConfig, b: BatchCtx, save: bool,
              moe: Any = None, lora: dict | None = None, tp: Any = None):
    lora = lora or _NO_LORA
    T = x.shape[0]
    nq, nk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    h1, rstd1, _ = ops.rmsnorm_fwd(x, P["in_norm"], cfg.rms_eps)
    qkv, u_qkv = _lin(h1, P["qkv_w"], lora.get("qkv"), bias=P.get("qkv_b"))
    qkv_pre = qkv.clone() if (save and cfg.qk_norm) else None
    rstd_qk = ops.qk_norm_rope_(qkv, nq, nk, b.pos, b.inv_freq, P.get("q_norm"), P.get("k_norm"), cfg.rms_eps)
    q = qkv[:, : nq * hd].view(T, nq, hd)
    k = qkv[:, nq * hd : (nq + nk) * hd].view(T, nk, hd)
    v = qkv[:, (nq + nk) * hd :].view(T, nk, hd)
    if b.cp is not None:
        att, lse = cp_attention_fwd(q, k, v, b.cp)
    else:
        att, lse = attention_fwd(q, k, v, b.cu_seqlens, b.max_seqlen, True)
    att2 = att.view(T, nq * hd)
    x2, u_o = _lin_rowpar(att2, P["o_w"], lora.get("o"), x, tp)
    if moe is None:
        out, mc = _dense_mlp_fwd(x2, P, cfg, save, lora, tp)
    else:
        out, mc = moe.forward(x2, P, save)
    cache = None
    if save:
        cache = dict(h1=h1, rstd1=rstd1, qkv=qkv, qkv_pre=qkv_pre, rstd_qk=rstd_qk, att=att, lse=lse, x2=x2, mlp=mc,
                     u_qkv=u_qkv, u_o=u_o)
    return out, cache


def layer_bwd(dout: torch.Tensor, x: torch.Tensor, c: dict, P: dict, G: dict, cfg: ArchConfig, b: BatchCtx,
              moe: Any = None, lora: dict | None = None, tp: Any = None):
    lora = lora or _NO_LORA
    T = x.shape[0]
    nq, nk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    dout = dout.contiguous()
    mc = c["mlp"]
    if moe is None:
        # out = x2 + a Wd^T
        da = _lin_bwd(dout, mc["a"], mc["u_dn"], P["down_w"], G.get("down_w"), lora.get("down"))
        dgu = ops.swiglu_bwd(mc["gu"], da)
        del da
        dh2 = _lin_bwd(dgu, mc["h2"], mc["u_gu"], P["gu_w"], G.get("gu_w"), lora.get("gu"), tp)
        del dgu
        dx2 = ops.rmsnorm_bwd(c["x2"], P["post_norm"], mc["rstd2"], dh2, dres=dout, dw=G.get("post_norm"))
        del dh2
    else:
        dx2 = moe.backward(dout, c["x2"], mc, P, G)
    # x2 = x + att Wo^T
    datt = _lin_bwd(dx2, c["att"].view(T, nq * hd), c["u_o"], P["o_w"], G.get("o_w"), lora.get("o"))
    qkv = c["qkv"]
    q = qkv[:, : nq * hd].view(T, nq, hd)
    k = qkv[:, nq * hd : (nq + nk) * hd].view(T, nk, hd)
    v = qkv[:, (nq + nk) * hd :].view(T, nk, hd)
    if b.cp is not None:
        dq, dk, dv = cp_attention_bwd(datt.view(T, nq, hd), q, k, v, c["att"], c["lse"], b.cp)
    else:
        dq, dk, dv = attention_bwd(datt.view(T, nq, hd), q, k, v, c["att"], c["lse"], b.cu_seqlens, b.max_seqlen,
                                   True)
    del datt
    dqkv = torch.cat([dq.reshape(T, -1), dk.reshape(T, -1), dv.reshape(T, -1)], 1)
    del dq, dk, dv
    qkv_pre = c["qkv_pre"] if c["qkv_pre"] is not None else qkv
    ops.qk_norm_rope_bwd_(dqkv, qkv_pre, nq, nk, b.pos, b.inv_freq, P.get("q_norm"), P.get("k_norm"), c["rstd_qk"],
                          G.get("q_norm"), G.get("k_norm"), cfg.rms_eps)
    if G.get("qkv_b") is not None:
        G["qkv_b"].add_(dqkv.sum(0, dtype=torch.float32))  # reduce in fp32, no fp32 copy of dqkv
    dh1 = _lin_bwd(dqkv, c["h1"], c["u_qkv"], P["qkv_w"], G.get("qkv_w"), lora.get("qkv"), tp)
    del dqkv
    dx = ops.rmsnorm_bwd(x, P["in_norm"], c["rstd1"], dh1, dres=dx2, dw=G.get("in_norm"))
    return dx


class ActivationOffload:
    """Keeps every decoder layer's saved input in pinned host memory between
    forward and backward (``model.smart_gc``; reference kernels/smart_gc.py
    offloads checkpoint inputs over 2 MB to pinned CPU).  The device-to-host
    copy runs on a side stream ordered after the producing kernels; the
    backward copies the input back before recomputing the layer.  Only the
    per-layer inputs are kept (the layer itself is recomputed), so device
    activation memory no longer grows with depth."""

    def __init__(self, min_bytes: int = 2 << 20):
        self.min_bytes = min_bytes
        self.stream = None

    def save(self, x: torch.Tensor):
        if not x.is_cuda or x.numel() * x.element_size() < self.min_bytes:
            return x, None
        if self.stream is None:
            self.stream = torch.cuda.Stream(x.device)
        host = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        self.stream.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(self.stream):
            host.copy_(x, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        x.record_stream(self.stream)  # keep x alive until the copy has read it
        return host, ev

    @staticmethod
    def restore(saved, ev, device) -> torch.Tensor:
        if ev is None:
            return saved
        ev.synchronize()
        return saved.to(device, non_blocking=True)


class DecoderLayerFn(torch.autograd.Function):
    """One decoder layer as one autograd node.  With ``layer.recompute``
    (activation checkpointing, the default) only the input is saved and the
    backward recomputes the layer; otherwise the forward keeps the layer's
    activations and the backward uses them directly (one GEMM pass fewer,
    about 0.66 GB per layer per 4096 tokens at the 7B shape)."""

    @staticmethod
    def forward(ctx, x, anchor, layer):
        keep = not getattr(layer, "recompute", True)
        z = getattr(layer, "zero3", None)
        if z is not None:
            z.stage_forward(layer.index)  # ZeRO-3: gather this layer's weights
        with torch.no_grad(), nvtx.range(f"layer{layer.index}.fwd"):
            out, cache = layer_fwd(x, layer.P, layer.cfg, layer.batch, save=keep, moe=layer.moe, lora=layer.lora,
                                   tp=layer.tp)
        ctx.cache = cache  # kept activations: the backward skips the recompute
        off = getattr(layer, "offload", None) if not keep else None
        if off is not None:
            ctx.host, ctx.ev = off.save(x)
            ctx.device = x.device
            ctx.save_for_backward()
        else:
            ctx.host = None
            ctx.save_for_backward(x)
        ctx.layer = layer
        return out

    @staticmethod
    def backward(ctx, dout):
        if ctx.host is not None:
            x = ActivationOffload.restore(ctx.host, ctx.ev, ctx.device)
            ctx.host = None
        else:
            (x,) = ctx.saved_tensors
        layer = ctx.layer
        z = getattr(layer, "zero3", None)
        if z is not None:
            z.stage_backward(layer.index)  # weights again, gradients into a zeroed staging slot
        with torch.no_grad(), nvtx.range(f"layer{layer.index}.bwd"):
            cache, ctx.cache = ctx.cache, None
            if cache is None:
                _, cache = layer_fwd(x, layer.P, layer.cfg, layer.batch, save=True, moe=layer.moe, lora=layer.lora,
                                     tp=layer.tp)
            dx = layer_bwd(dout, x, cache, layer.P, layer.G, layer.cfg, layer.batch, moe=layer.moe, lora=layer.lora,
                           tp=layer.tp)
        if z is not None:
            z.end_backward_layer(layer.index)
        return dx, None, None


class EmbeddingFn(torch.autograd.Function):
    """Row gather whose backward scatter-adds straight into the fp32 grad."""

    @staticmethod
    def forward(ctx, ids, anchor, table, gtable, zero3=None):
        ctx.save_for_backward(ids)
        ctx.gtable = gtable
        ctx.zero3 = zero3
        return ops.embedding_fwd(table, ids)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        if ctx.gtable is not None:
            ops.embedding_bwd_(dy, ids, ctx.gtable)
        if ctx.zero3 is not None:  # the last node of the backward: reduce the remaining gradients
            ctx.zero3.finish_backward()
        return None, None, None, None, None


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
