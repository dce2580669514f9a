"""Plain PyTorch implementations of every fused op.

They serve two purposes: the CPU execution path (the CPU/gloo plumbing
configuration runs the whole framework in float32 on the host) and the float32
oracle that the GPU kernels are tested against.  Semantics follow the
reference's eager paths (HF Qwen2/Qwen3 modules used by trainer/model.py,
kernels/swiglu.py:12-83, trainer/losses.py:600-1004).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))


def apply_rope(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate-half rotary embedding; x is [T, heads, head_dim]."""
    ang = pos.float()[:, None] * inv_freq[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    rot = torch.cat([-x2, x1], -1)
    return (x.float() * cos + rot.float() * sin).to(x.dtype)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    g, u = gu.chunk(2, dim=-1)
    return (F.silu(g.float()) * u.float()).to(gu.dtype)


def attention(q, k, v, cu_seqlens: torch.Tensor, causal: bool = True, scale: float | None = None,
              cu_seqlens_k: torch.Tensor | None = None):
    """Packed variable-length attention.

    q: [T, hq, d], k/v: [T, hk, d]; cu_seqlens: int32 [n+1] sequence
    boundaries.  GQA by head repetition.  Returns [T, hq, d].  With
    ``cu_seqlens_k`` the keys of sequence i are k[cu_seqlens_k[i]:
    cu_seqlens_k[i+1]] and its queries are the last positions of that key
    sequence (causal mask aligned bottom-right).
    """
    T, hq, d = q.shape
    hk = k.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    out = torch.zeros_like(q)
    bounds = cu_seqlens.tolist()
    kb = cu_seqlens_k.tolist() if cu_seqlens_k is not None else bounds
    rep = hq // hk
    for s, e, ks0, ke in zip(bounds[:-1], bounds[1:], kb[:-1], kb[1:]):
        if e <= s:
            continue
        qs = q[s:e].transpose(0, 1).float()
        ks = k[ks0:ke].transpose(0, 1).float().repeat_interleave(rep, 0)
        vs = v[ks0:ke].transpose(0, 1).float().repeat_interleave(rep, 0)
        att = (qs @ ks.transpose(-1, -2)) * scale
        if causal:
            Lq, Lk = e - s, ke - ks0
            mask = torch.ones(Lq, Lk, dtype=torch.bool, device=q.device).tril(Lk - Lq)
            att = att.masked_fill(~mask, float("-inf"))
        p = att.softmax(-1)
        out[s:e] = (p @ vs).transpose(0, 1).to(q.dtype)
    return out


def logprob_entropy(logits: torch.Tensor, target: torch.Tensor, temperature: float = 1.0):
    z = logits.float() / temperature
    logp = torch.log_softmax(z, -1)
    lp = logp.gather(-1, target.clamp_min(0)[..., None])[..., 0]
    ent = -(logp.exp() * logp).sum(-1)
    return lp, ent
