"""Chunked LM head: per-token log-prob / entropy / cross-entropy without ever
materialising the full [T, V] logits.

Tokens are processed in chunks of ``chunk`` rows.  For each chunk the logits
z = h W^T are produced by the tcgen05 GEMM into a reusable bf16 scratch
buffer, reduced row-wise by ``softmax_stats`` (lse, target log-prob, entropy
at temperature tau), and — for the backward — overwritten in place by
``softmax_grad`` with dL/dz before two more GEMMs produce dL/dh (dgrad) and
accumulate dL/dW into the fp32 gradient buffer (wgrad, fp32-accumulate
epilogue).

Parity: trainer/losses.py:600-1004 (ChunkedLogprobLmHead,
_ChunkedLogprobFn: token x 8192-vocab chunking with online softmax and a
hand-written backward that recomputes logits) and the SFT chunked CE at
trainer/trainer.py:1520-1583.
"""

from __future__ import annotations

import torch

from . import EPI_F32_ACC, ext, gemm
from . import reference as ref

DEFAULT_CHUNK = 4096


def _chunks(T: int, chunk: int):
    for s in range(0, T, chunk):
        yield s, min(T, s + chunk)


def sft_loss_and_grad(h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor, weights: torch.Tensor,
                      gW: torch.Tensor | None, chunk: int = DEFAULT_CHUNK):
    """Fused forward + backward of sum_t weights[t] * CE(h_t W^T, targets[t]).

    Returns (loss_sum fp32 scalar tensor, dh [T, H] bf16).  ``weights`` holds the
    per-token loss scale (mask / normaliser); dW is accumulated into ``gW``.
    Tokens with target < 0 contribute nothing.
    """
    T, H = h.shape
    V = W.shape[0]
    dev = h.device
    if not h.is_cuda:
        hh = h.detach().float().requires_grad_(True)
        Wf = W.detach().float().requires_grad_(True)
        z = hh @ Wf.t()
        lp = torch.log_softmax(z, -1).gather(-1, targets.clamp_min(0)[:, None])[:, 0]
        valid = (targets >= 0).float()
        loss = -(lp * weights * valid).sum()
        loss.backward()
        if gW is not None:
            gW.add_(Wf.grad)
        return loss.detach(), hh.grad.to(h.dtype)
    m = ext()
    h = h.contiguous()
    dh = torch.empty_like(h)
    loss = torch.zeros((), device=dev, dtype=torch.float32)
    zbuf = torch.empty(min(chunk, T), V, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(min(chunk, T), device=dev, dtype=torch.float32)
    lp = torch.empty_like(lse)
    tgt_all = targets.to(torch.int64).contiguous()
    w_all = (weights * (targets >= 0)).float().contiguous()
    for s, e in _chunks(T, chunk):
        n = e - s
        z = zbuf[:n]
        gemm(h[s:e], W, out=z)
        tgt = tgt_all[s:e]
        m.softmax_stats(z, tgt, 1.0, lse[:n], lp[:n], None)
        wv = w_all[s:e]
        loss -= (lp[:n] * wv).sum()
        dlp = -wv
        m.softmax_grad(z, tgt, 1.0, lse[:n], None, dlp, None)
        gemm(z, W, b_mn=True, out=dh[s:e])
        if gW is not None:
            gemm(z, h[s:e], a_mn=True, b_mn=True, out=gW, epi=EPI_F32_ACC)
    return loss, dh


class ChunkedLogprobFn(torch.autograd.Function):
    """(h, W, targets, tau) -> (logprob [T], entropy [T]) with recompute backward."""

    @staticmethod
    def forward(ctx, h, anchor, W, gW, targets, temperature, chunk, want_entropy):
        T, H = h.shape
        V = W.shape[0]
        h = h.contiguous()
        m = ext()
        lp = torch.empty(T, device=h.device, dtype=torch.float32)
        ent = torch.empty(T, device=h.device, dtype=torch.float32)
        lse = torch.empty(T, device=h.device, dtype=torch.float32)
        zbuf = torch.empty(min(chunk, T), V, device=h.device, dtype=torch.bfloat16)
        tgt = targets.to(torch.int64).contiguous()
        for s, e in _chunks(T, chunk):
            z = zbuf[: e - s]
            gemm(h[s:e], W, out=z)
            m.softmax_stats(z, tgt[s:e], 1.0 / temperature, lse[s:e], lp[s:e], ent[s:e] if want_entropy else None)
        if not want_entropy:
            ent.zero_()
        ctx.save_for_backward(h, W, tgt, lse, ent)
        ctx.gW = gW
        ctx.cfg = (temperature, chunk, want_entropy)
        return lp, ent

    @staticmethod
    def backward(ctx, dlp, dent):
        h, W, tgt, lse, ent = ctx.saved_tensors
        temperature, chunk, want_entropy = ctx.cfg
        m = ext()
        T, H = h.shape
        V = W.shape[0]
        dh = torch.empty_like(h)
        zbuf = torch.empty(min(chunk, T), V, device=h.device, dtype=torch.bfloat16)
        dlp = dlp.float().contiguous() if dlp is not None else torch.zeros(T, device=h.device)
        dent = dent.float().contiguous() if (dent is not None and want_entropy) else None
        for s, e in _chunks(T, chunk):
            z = zbuf[: e - s]
            gemm(h[s:e], W, out=z)
            m.softmax_grad(z, tgt[s:e], 1.0 / temperature, lse[s:e], ent[s:e], dlp[s:e],
                           dent[s:e] if dent is not None else None)
            gemm(z, W, b_mn=True, out=dh[s:e])
            if ctx.gW is not None:
                gemm(z, h[s:e], a_mn=True, b_mn=True, out=ctx.gW, epi=EPI_F32_ACC)
        return dh, None, None, None, None, None, None, None


def logprob_entropy(h, W, targets, temperature: float = 1.0, gW=None, chunk: int = DEFAULT_CHUNK,
                    want_entropy: bool = True, anchor=None):
    """Per-token log-prob of ``targets`` and entropy at ``temperature``."""
    if not h.is_cuda:
        z = h @ W.t()
        return ref.logprob_entropy(z, targets, temperature)
    if anchor is None:
        anchor = torch.empty(0, device=h.device, requires_grad=True)
    return ChunkedLogprobFn.apply(h, anchor, W, gW, targets, temperature, chunk, want_entropy)


class _HeadLogitsCPU(torch.autograd.Function):
    """CPU logits ``h W^T`` whose weight gradient is added into the flat
    gradient view ``gW`` (the parameter views of the flat store do not take
    part in autograd), so the LM head trains on every CPU path of the model,
    the fused-kernel fallbacks (tensor / context parallel) included."""

    @staticmethod
    def forward(ctx, h, W, gW):
        ctx.save_for_backward(h, W)
        ctx.gW = gW
        return h @ W.t()

    @staticmethod
    def backward(ctx, dz):
        h, W = ctx.saved_tensors
        if ctx.gW is not None:
            ctx.gW.add_((dz.t() @ h).to(ctx.gW.dtype))
        return dz @ W, None, None


def cpu_head_logits(h: torch.Tensor, W: torch.Tensor, gW: torch.Tensor | None) -> torch.Tensor:
    return _HeadLogitsCPU.apply(h, W.detach(), gW)
