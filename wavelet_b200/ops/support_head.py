"""Log-partition over a per-token sampling support set.

When the generator sampled with top-k / top-p / min-p, the reference replays
the support set ("sampling mask") and renormalises the trainer log-prob over
it: lp = z_t / T - logsumexp_{j in S_t} z_j / T (trainer/losses.py:30-69).
``SupportLogZ`` computes the support log-partition and target logit for the
rows that carry a support set, gathering only |S_t| rows of the LM head
instead of the full vocabulary, with a hand-written backward that routes the
head-weight gradient into the fp32 flat gradient buffer.
"""

from __future__ import annotations

import torch

CHUNK_ROWS = 1024


class SupportLogZ(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, rows, ids, valid, W, gW, temperature, anchor):
        out = torch.empty(rows.numel(), device=h.device, dtype=torch.float32)
        for s in range(0, rows.numel(), CHUNK_ROWS):
            e = min(rows.numel(), s + CHUNK_ROWS)
            hr = h[rows[s:e]].float()  # [R, H]
            Wg = W[ids[s:e]].float()  # [R, K, H]
            z = torch.einsum("rh,rkh->rk", hr, Wg) / temperature
            z = z.masked_fill(~valid[s:e], float("-inf"))
            out[s:e] = torch.logsumexp(z, -1)
        ctx.save_for_backward(h, rows, ids, valid, W, out)
        ctx.gW = gW
        ctx.t = temperature
        return out

    @staticmethod
    def backward(ctx, g):
        h, rows, ids, valid, W, logz = ctx.saved_tensors
        T = ctx.t
        dh = torch.zeros(h.shape, device=h.device, dtype=torch.float32)
        gW = ctx.gW
        dW = None if gW is not None else torch.zeros(W.shape, device=W.device, dtype=torch.float32)
        for s in range(0, rows.numel(), CHUNK_ROWS):
            e = min(rows.numel(), s + CHUNK_ROWS)
            hr = h[rows[s:e]].float()
            Wg = W[ids[s:e]].float()
            z = torch.einsum("rh,rkh->rk", hr, Wg) / T
            p = torch.exp(z - logz[s:e, None]).masked_fill(~valid[s:e], 0.0) * (g[s:e, None] / T)  # [R, K]
            dh.index_add_(0, rows[s:e], torch.einsum("rk,rkh->rh", p, Wg))
            contrib = (p[:, :, None] * hr[:, None, :]).reshape(-1, hr.shape[1])
            flat_ids = ids[s:e].reshape(-1)
            (gW if gW is not None else dW).index_add_(0, flat_ids, contrib)
        return dh.to(h.dtype), None, None, None, (dW.to(W.dtype) if dW is not None else None), None, None, None

    @staticmethod
    def target_logit(h, rows, tgt, W, gW, temperature, anchor):
        return _TargetLogit.apply(h, rows, tgt[rows], W, gW, temperature, anchor)


class _TargetLogit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, rows, t, W, gW, temperature, anchor):
        hr = h[rows].float()
        wt = W[t].float()
        ctx.save_for_backward(h, rows, t, W)
        ctx.gW = gW
        ctx.T = temperature
        return (hr * wt).sum(-1) / temperature

    @staticmethod
    def backward(ctx, g):
        h, rows, t, W = ctx.saved_tensors
        T = ctx.T
        dh = torch.zeros(h.shape, device=h.device, dtype=torch.float32)
        dh.index_add_(0, rows, W[t].float() * (g[:, None] / T))
        contrib = h[rows].float() * (g[:, None] / T)
        dW = None
        if ctx.gW is not None:
            ctx.gW.index_add_(0, t, contrib)
        else:
            dW = torch.zeros(W.shape, device=W.device, dtype=torch.float32).index_add_(0, t, contrib).to(W.dtype)
        return dh.to(h.dtype), None, None, dW, None, None, None
