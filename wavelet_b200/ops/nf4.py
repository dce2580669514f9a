"""4-bit NormalFloat (NF4) weights for QLoRA.

NF4 (Dettmers et al., "QLoRA", 2023, section 3) maps each block of 64
consecutive weights to 4-bit codes of a 16-value table built from quantiles
of the standard normal distribution, scaled by the block's absolute maximum.
The table is asymmetric so that zero is exactly representable: 8 positive
quantiles at probabilities linspace(delta, 1/2, 9)[:-1], 7 negative ones at
linspace(delta, 1/2, 8)[:-1], plus 0, normalised to [-1, 1], with
delta = 1 - (1/(2*15) + 1/(2*16)) / 2.  It is computed here from that
construction (``statistics.NormalDist``) rather than copied.

Storage (``NF4Weight``): the row-major [rows, cols] matrix as uint8 codes,
two per byte (element 2i in the high nibble, 2i+1 in the low nibble), and
one fp32 absmax per 64 elements of a row (cols % 64 == 0).  The reference
loads its base model through bitsandbytes ``load_in_4bit`` (NF4, blocksize
64; trainer/model.py:446-468) and dequantises per call inside its LoRA
kernels (kernels/utils.py:8-86); here the tcgen05 GEMM dequantises inside
the kernel (csrc/gemm.cu, NF4 B operand).
"""

from __future__ import annotations

import dataclasses
import itertools

from dataclasses import dataclass
from functools import lru_cache
from statistics import NormalDist

import torch

BLOCK = 64


@lru_cache(maxsize=1)
def nf4_table() -> tuple[float, ...]:
    nd = NormalDist()
    delta = 1.0 - 0.5 * (1.0 / (2 * 15) + 1.0 / (2 * 16))
    pos = [nd.inv_cdf(delta + (0.5 - delta) * i / 8) for i in range(8)]
    neg = [-nd.inv_cdf(delta + (0.5 - delta) * i / 7) for i in range(7)]
    vals = sorted(pos + neg + [0.0])
    top = max(abs(v) for v in vals)
    return tuple(v / top for v in vals)


_NF4_UIDS = itertools.count()


@dataclass
class NF4Weight:
    codes: torch.Tensor  # uint8 [rows * cols / 2]
    absmax: torch.Tensor  # fp32 [rows * cols / 64]
    rows: int
    cols: int
    version: int = 0  # bumped whenever codes/absmax change (invalidates dequant caches)
    # process-unique serial for cache keys: id() is reused once an object is freed,
    # so a new weight could otherwise hit a dead weight's cached dequantisation
    uid: int = dataclasses.field(default_factory=lambda: next(_NF4_UIDS), compare=False)

    @property
    def shape(self) -> tuple[int, int]:
        return (self.rows, self.cols)

    @property
    def device(self) -> torch.device:
        return self.codes.device

    def nbytes(self) -> int:
        return self.codes.numel() + 4 * self.absmax.numel()

    def dequantize(self, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        return dequantize(self, dtype)


def _lut(device) -> torch.Tensor:
    return torch.tensor(nf4_table(), dtype=torch.float32, device=device)


@torch.no_grad()
def quantize(w: torch.Tensor, chunk_rows: int = 4096) -> NF4Weight:
    """Blockwise NF4 quantisation of a [rows, cols] matrix (nearest code)."""
    if w.dim() != 2 or w.shape[1] % BLOCK:
        raise ValueError(f"NF4 needs a 2-D weight with cols % {BLOCK} == 0, got {tuple(w.shape)}")
    rows, cols = w.shape
    lut = _lut(w.device)
    mids = (lut[1:] + lut[:-1]) / 2
    codes = torch.empty(rows * cols // 2, dtype=torch.uint8, device=w.device)
    absmax = torch.empty(rows * cols // BLOCK, dtype=torch.float32, device=w.device)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        blk = w[r0:r1].float().reshape(-1, BLOCK)
        am = blk.abs().amax(1)
        xn = blk / am.clamp_min(1e-30)[:, None]
        q = torch.bucketize(xn, mids).to(torch.uint8).reshape(-1)
        codes[r0 * cols // 2 : r1 * cols // 2] = (q[0::2] << 4) | q[1::2]
        absmax[r0 * cols // BLOCK : r1 * cols // BLOCK] = am
    return NF4Weight(codes, absmax, rows, cols)


# GEMMs with more rows than this dequantise the weight once (memory-bound
# kernel, cached) and run the dense GEMM; smaller ones (generation) dequantise
# inside the GEMM so the weight is read at 0.5 byte per element.  With M rows
# the in-kernel path repeats the dequantisation for every 128-row M tile.
FUSED_MAX_M = 256


class DequantCache:
    """Small LRU of dequantised bf16 weights.  A decoder layer's backward
    recomputes its forward and then runs the dgrad GEMMs in reverse order, so
    four entries (qkv, o, gate/up, down) let the dgrads reuse the recompute's
    dequantisation."""

    def __init__(self, capacity: int = 4):
        self.capacity = capacity
        self.entries: list[tuple[tuple[int, int], torch.Tensor]] = []
        self.pool: list[torch.Tensor] = []

    def get(self, q: NF4Weight) -> torch.Tensor:
        key = (q.uid, q.version)
        n = q.rows * q.cols
        for i, (k, t) in enumerate(self.entries):
            if k == key:
                self.entries.append(self.entries.pop(i))
                return t[:n].view(q.rows, q.cols)
        buf = None
        while len(self.entries) >= self.capacity:
            self.pool.append(self.entries.pop(0)[1])
        for i, t in enumerate(self.pool):
            if t.numel() >= n and t.device == q.device:
                buf = self.pool.pop(i)
                break
        if buf is None:
            buf = torch.empty(n, device=q.device, dtype=torch.bfloat16)
        out = buf[:n]
        from . import ext

        ext().nf4_dequant(q.codes, q.absmax, out, list(nf4_table()))
        self.entries.append((key, buf))
        return out.view(q.rows, q.cols)

    def clear(self) -> None:
        self.entries.clear()
        self.pool.clear()


_cache = DequantCache()


def dequant_cache() -> DequantCache:
    return _cache


@torch.no_grad()
def dequantize(q: NF4Weight, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    lut = _lut(q.codes.device)
    hi = (q.codes >> 4).long()
    lo = (q.codes & 15).long()
    vals = torch.stack([lut[hi], lut[lo]], 1).reshape(-1, BLOCK) * q.absmax[:, None]
    return vals.reshape(q.rows, q.cols).to(dtype)
