"""Synthetic data sources (no network, no tokenizer).

``synthetic_sft_microbatches`` produces packed micro-batches of uniform random
tokens with the loss masked on a random 10-40% prompt prefix of every
sequence — the data shape of the 7B SFT benchmark.  The reference's ``fake``
SFT source (data/sft.py:195) plays the same role for its tests and benchmark.
"""

from __future__ import annotations

import torch

from ..trainer.engine import PackedBatch


def packed_from_sequences(seqs: list[torch.Tensor], loss_masks: list[torch.Tensor]) -> PackedBatch:
    """Pack token sequences end to end (``cat`` packing, no padding)."""
    ids = torch.cat(seqs).long()
    lens = [len(s) for s in seqs]
    cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lens, dtype=torch.int32).cumsum(0)
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens])
    tgt_parts, mask_parts = [], []
    for s, m in zip(seqs, loss_masks):
        t = torch.empty_like(s, dtype=torch.long)
        t[:-1] = s[1:]
        t[-1] = -100
        mm = m.float().clone()
        mm[-1] = 0.0
        tgt_parts.append(t)
        mask_parts.append(mm)
    tgt = torch.cat(tgt_parts)
    mask = torch.cat(mask_parts)
    tgt = torch.where(mask > 0, tgt, torch.full_like(tgt, -100))
    return PackedBatch(ids, pos, cu, max(lens), tgt, mask)


def synthetic_sft_microbatches(n: int, seq_len: int, vocab: int, seed: int = 0, low: int = 3,
                               prompt_frac=(0.1, 0.4), seqs_per_micro: int = 1) -> list[PackedBatch]:
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        seqs, masks = [], []
        for _ in range(seqs_per_micro):
            s = torch.randint(low, vocab, (seq_len,), generator=g)
            f = prompt_frac[0] + (prompt_frac[1] - prompt_frac[0]) * torch.rand((), generator=g).item()
            m = torch.ones(seq_len)
            m[: int(f * seq_len)] = 0.0
            seqs.append(s)
            masks.append(m)
        out.append(packed_from_sequences(seqs, masks))
    return out
