"""Context parallelism: one micro-batch's sequences split along the tokens
over ``cp`` ranks, attention over the full sequences.

The reference pads each row to a multiple of 2*cp and wraps SDPA in PyTorch's
experimental ring attention (trainer/context_parallel.py:114-163,
trainer/distributed.py:253-255); it rejects packed and padded masks.  Here CP
works on the packed varlen layout directly:

* every sequence of length L is padded to a multiple of 2*cp*``align`` and cut
  into 2*cp chunks of C tokens; rank r keeps chunks r and 2*cp-1-r (the
  load-balanced pairing: every rank gets the same causal work);
* the rank's local tokens are [chunk r of every sequence] then [chunk
  2*cp-1-r of every sequence] (groups A and B).  Everything outside attention
  is per token and runs unchanged on the local tokens;
* attention: K and V (small under GQA: Hk heads) are all-gathered over the CP
  group, each group's key prefixes (chunks 0..c of its sequences) are
  gathered into one packed key tensor, and the sm_100a varlen kernels run
  with separate key sequences whose queries are the last C positions
  (bottom-right causal alignment, so the kernels need (c * C) % 128 == 0:
  ``align`` = 128 on CUDA);
* backward: dQ is local; the dK / dV of the gathered keys (both groups
  accumulated in fp32) are reduce-scattered back to the chunks' owners.

Loss tokens are counted over the dp x cp ranks, and gradients are reduced
over them, like the reference's ``dp_cp`` mesh (trainer/trainer.py:1513-1518).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist


@dataclass
class CPPlan:
    group: Any
    rank: int
    size: int
    T: int  # local tokens
    TA: int  # group A rows (the rest is group B)
    cu_q: torch.Tensor  # int32 [n+1]: query chunks of one group (same lengths in A and B)
    max_q: int
    cu_k: tuple[torch.Tensor, torch.Tensor]  # key prefixes of groups A and B
    max_k: tuple[int, int]
    idx: tuple[torch.Tensor, torch.Tensor]  # rows of the all-gathered [size * T] keys, per group

    def to(self, device) -> "CPPlan":
        mv = lambda t: t.to(device, non_blocking=True)  # noqa: E731
        return CPPlan(self.group, self.rank, self.size, self.T, self.TA, mv(self.cu_q), self.max_q,
                      (mv(self.cu_k[0]), mv(self.cu_k[1])), self.max_k, (mv(self.idx[0]), mv(self.idx[1])))


def shard_batch(b, cp: int, rank: int, group, align: int = 128):
    """This rank's share of a packed batch (``trainer.engine.PackedBatch``)
    and its ``CPPlan``; host-side, once per micro-batch."""
    from ..trainer.engine import PackedBatch

    bounds = b.cu_seqlens.tolist()
    lens = [e - s for s, e in zip(bounds[:-1], bounds[1:])]
    unit = 2 * cp * align
    C = [max(1, -(-L // unit)) * unit // (2 * cp) for L in lens]
    dev = b.input_ids.device
    ca, cb = rank, 2 * cp - 1 - rank
    tok, pos, tgt, msk = [], [], [], []

    def take(s, c):
        s0, L = bounds[s], lens[s]
        p = torch.arange(c * C[s], (c + 1) * C[s], device=dev)
        real = p < L
        src = (s0 + p).clamp_max(s0 + max(L, 1) - 1)
        tok.append(torch.where(real, b.input_ids[src], torch.zeros_like(b.input_ids[src])))
        tgt.append(torch.where(real, b.targets[src], torch.full_like(b.targets[src], -100)))
        msk.append(torch.where(real, b.loss_mask[src], torch.zeros_like(b.loss_mask[src])))
        first = b.position_ids[s0] if L > 0 else torch.zeros((), dtype=b.position_ids.dtype, device=dev)
        pos.append((first + p).to(b.position_ids.dtype))

    for s in range(len(lens)):
        take(s, ca)
    for s in range(len(lens)):
        take(s, cb)
    TA = sum(C)
    T = 2 * TA
    # where chunk (s, c) lives in the all-gathered keys: rank j's local row i -> j * T + i
    off = [sum(C[:s]) for s in range(len(lens))]

    def chunk_rows(s, c):
        j, base = (c, 0) if c < cp else (2 * cp - 1 - c, TA)
        return torch.arange(j * T + base + off[s], j * T + base + off[s] + C[s], dtype=torch.int64)

    def key_group(cq):
        idx, cu = [], [0]
        for s in range(len(lens)):
            for c in range(cq + 1):
                idx.append(chunk_rows(s, c))
            cu.append(cu[-1] + (cq + 1) * C[s])
        return torch.cat(idx), torch.tensor(cu, dtype=torch.int32)

    ia, cka = key_group(ca)
    ib, ckb = key_group(cb)
    cu_q = torch.tensor([0] + [sum(C[: s + 1]) for s in range(len(lens))], dtype=torch.int32)
    mc = max(C)
    plan = CPPlan(group=group, rank=rank, size=cp, T=T, TA=TA, cu_q=cu_q, max_q=mc,
                  cu_k=(cka, ckb), max_k=((ca + 1) * mc, (cb + 1) * mc), idx=(ia, ib))
    local = PackedBatch(torch.cat(tok), torch.cat(pos), cu_q_local(C), mc, torch.cat(tgt), torch.cat(msk))
    local.cp = plan.to(dev)
    return local


def shard_index(cu_seqlens: torch.Tensor, cp: int, rank: int, align: int = 128):
    """Token map of this rank's context-parallel share (the layout of
    ``shard_batch``): for every local token its source row in the packed
    batch, whether it is a real token (not chunk padding) and its sequence.
    Any per-token tensor ``t`` of the batch maps to the local layout as
    ``torch.where(real, t[src], fill)``."""
    bounds = cu_seqlens.tolist()
    lens = [e - s_ for s_, e in zip(bounds[:-1], bounds[1:])]
    unit = 2 * cp * align
    C = [max(1, -(-L // unit)) * unit // (2 * cp) for L in lens]
    src, real, seq = [], [], []
    for c in (rank, 2 * cp - 1 - rank):
        for s_, L in enumerate(lens):
            p = torch.arange(c * C[s_], (c + 1) * C[s_])
            src.append((bounds[s_] + p).clamp_max(bounds[s_] + max(L, 1) - 1))
            real.append(p < L)
            seq.append(torch.full((C[s_],), s_, dtype=torch.long))
    return torch.cat(src), torch.cat(real), torch.cat(seq)


def cu_q_local(C: list[int]) -> torch.Tensor:
    """Sequence boundaries of the local tokens (every chunk is its own
    sequence for the per-token kernels; attention uses the plan)."""
    cu = [0]
    for c in C + C:
        cu.append(cu[-1] + c)
    return torch.tensor(cu, dtype=torch.int32)


def _all_gather(t: torch.Tensor, p: CPPlan) -> torch.Tensor:
    t = t.contiguous()
    out = torch.empty((p.size,) + tuple(t.shape), device=t.device, dtype=t.dtype)
    if t.is_cuda:
        dist.all_gather_into_tensor(out, t, group=p.group)
    else:
        dist.all_gather(list(out.unbind(0)), t, group=p.group)
    return out.view((p.size * t.shape[0],) + tuple(t.shape[1:]))


def _reduce_scatter(full: torch.Tensor, p: CPPlan) -> torch.Tensor:
    """Sum over the CP ranks of [size * T, ...] and keep this rank's T rows."""
    if full.is_cuda:
        out = torch.empty((p.T,) + tuple(full.shape[1:]), device=full.device, dtype=full.dtype)
        dist.reduce_scatter_tensor(out, full, group=p.group)
        return out
    dist.all_reduce(full, group=p.group)  # gloo has no reduce-scatter
    return full[p.rank * p.T:(p.rank + 1) * p.T].clone()


def _keys(k: torch.Tensor, v: torch.Tensor, p: CPPlan):
    kg, vg = _all_gather(k, p), _all_gather(v, p)
    return [(kg.index_select(0, p.idx[i]), vg.index_select(0, p.idx[i])) for i in range(2)]


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, p: CPPlan):
    """(out [T, Hq, 128], (lse_A, lse_B)) of the local queries over the full sequences."""
    from ..ops.attention import attention_fwd as attn

    kv = _keys(k, v, p)
    outs, lses = [], []
    for i, (q_i, (k_i, v_i)) in enumerate(zip((q[: p.TA], q[p.TA:]), kv)):
        o, lse = attn(q_i, k_i, v_i, p.cu_q, p.max_q, True, None, p.cu_k[i], p.max_k[i])
        outs.append(o)
        lses.append(lse)
    return torch.cat(outs, 0), tuple(lses)


def attention_bwd(dout, q, k, v, out, lse, p: CPPlan):
    """(dq, dk, dv) of the local tokens; dK / dV summed over every rank's queries."""
    from ..ops.attention import attention_bwd as attn_bwd

    kv = _keys(k, v, p)
    full_shape = (p.size * p.T,) + tuple(k.shape[1:])
    dkg = torch.zeros(full_shape, device=k.device, dtype=torch.float32)
    dvg = torch.zeros(full_shape, device=k.device, dtype=torch.float32)
    dqs = []
    for i, sl in enumerate((slice(0, p.TA), slice(p.TA, p.T))):
        k_i, v_i = kv[i]
        dq, dk, dv = attn_bwd(dout[sl], q[sl], k_i, v_i, out[sl], None if lse is None else lse[i], p.cu_q, p.max_q,
                              True, None, p.cu_k[i], p.max_k[i])
        dqs.append(dq)
        dkg.index_add_(0, p.idx[i], dk.float())
        dvg.index_add_(0, p.idx[i], dv.float())
    dk = _reduce_scatter(dkg, p).to(k.dtype)
    dv = _reduce_scatter(dvg, p).to(v.dtype)
    return torch.cat(dqs, 0), dk, dv
