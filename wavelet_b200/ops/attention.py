"""Packed variable-length causal attention (training forward/backward).

Layout: q [T, Hq, 128], k/v [T, Hk, 128] bf16 with sequences packed along T
and delimited by ``cu_seqlens`` (int32 [n+1]); GQA with Hq % Hk == 0.  This is
the varlen attention the reference reaches through FA2/FA3/SDPA with packed
``position_ids`` (trainer/rl.py:189-229, trainer/model.py:315-360).

CUDA tensors run the extension's sm_100a attention kernels (``attn_fwd`` /
``attn_bwd``); CPU tensors use the float32 reference in ``ops.reference``.

Separate key sequences (``cu_seqlens_k``, context parallelism): sequence i's
keys are k[cu_seqlens_k[i]:cu_seqlens_k[i+1]] and its queries are the LAST
positions of those keys, so query j sees keys <= j + (Lk - Lq).  On CUDA,
Lk - Lq must be a non-negative multiple of 128 for every sequence.
"""

from __future__ import annotations

import math

import torch

from . import reference as ref
from ._ext import load as _load_ext


def native_attention() -> bool:
    try:
        return hasattr(_load_ext(), "attn_fwd")
    except Exception:
        return False


def attention_fwd(q, k, v, cu_seqlens, max_seqlen: int, causal: bool = True, scale: float | None = None,
                  cu_seqlens_k=None, max_seqlen_k: int = 0):
    """Returns (out [T, Hq, D], lse [Hq, T] fp32)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not q.is_cuda:
        out = ref.attention(q, k, v, cu_seqlens, causal, scale, cu_seqlens_k)
        return out, None
    m = _load_ext()
    out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    lse = torch.empty(q.shape[1], q.shape[0], device=q.device, dtype=torch.float32)
    m.attn_fwd(q, k, v, cu_seqlens, int(max_seqlen), bool(causal), float(scale), out, lse, cu_seqlens_k,
               int(max_seqlen_k))
    return out, lse


def attention_bwd(do, q, k, v, out, lse, cu_seqlens, max_seqlen: int, causal: bool = True, scale: float | None = None,
                  cu_seqlens_k=None, max_seqlen_k: int = 0):
    """Returns (dq, dk, dv)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not q.is_cuda:  # CPU: autograd through the reference attention
        with torch.enable_grad():
            qq, kk, vv = (t.detach().float().requires_grad_(True) for t in (q, k, v))
            o = ref.attention(qq, kk, vv, cu_seqlens, causal, scale, cu_seqlens_k)
            dq, dk, dv = torch.autograd.grad(o, (qq, kk, vv), do.float())
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)
    m = _load_ext()
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
    dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
    m.attn_bwd(do.contiguous(), q, k, v, out, lse, cu_seqlens, int(max_seqlen), bool(causal), float(scale), dq, dk, dv,
               cu_seqlens_k, int(max_seqlen_k))
    return dq, dk, dv


class AttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_seqlen, causal, scale):
        out, lse = attention_fwd(q, k, v, cu_seqlens, max_seqlen, causal, scale)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens)
        ctx.cfg = (max_seqlen, causal, scale)
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse, cu = ctx.saved_tensors
        max_seqlen, causal, scale = ctx.cfg
        dq, dk, dv = attention_bwd(do, q, k, v, out, lse, cu, max_seqlen, causal, scale)
        return dq, dk, dv, None, None, None, None


def attention(q, k, v, cu_seqlens, max_seqlen, causal=True, scale=None):
    if not q.is_cuda:
        return ref.attention(q, k, v, cu_seqlens, causal, scale)
    return AttentionFn.apply(q, k, v, cu_seqlens, max_seqlen, causal, scale)
