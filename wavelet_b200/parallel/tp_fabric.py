"""Tensor-parallel GEMM -> all-reduce fused over peer memory (one NVLink node).

Megatron-style TP (``models.qwen.tp_slicers``) without sequence parallelism
has two reduction points per block, both a GEMM followed by a collective:
the row-parallel output projections (o_proj, down_proj) in the forward and
the column-parallel input gradients (qkv, gate/up dgrad) in the backward.
The reference reaches them through DTensor / NCCL all-reduce after a cuBLAS
GEMM (trainer/model.py:1001-1034 parallelize plan).  Here the GEMM's epilogue
writes its bf16 partial tile straight into every TP rank's receive buffer
over NVLink (``kEpiPeerBF16``), so the transfer of one tile overlaps the MMA
of the next; after one barrier each rank sums the ``world`` slots it received
in rank order plus the residual (``slots_sum``).  All ranks therefore hold the
identical result without a separate all-reduce, and the residual no longer
has to ride on one rank's partial sum.

Receive buffers are double-buffered: a rank can run at most one fused GEMM
ahead of a peer (the barrier of op i separates op i+1's stores into buffer
(i+1)%2 from the peer's op i reduction of buffer i%2), so one barrier per op
suffices.  Buffers grow collectively (all TP ranks run the same shapes in the
same order).
"""

from __future__ import annotations

import torch

from .. import ops
from ..utils import nvtx
from .fabric import Fabric, SharedBuffer


class TPFabric:
    def __init__(self, fabric: Fabric, capacity: int = 1 << 20):
        self.fab = fabric
        self.world = fabric.world
        self.rank = fabric.rank
        self.capacity = 0
        self.bufs: list[SharedBuffer] = []
        self.flip = 0
        self._grow(capacity)

    def _grow(self, numel: int) -> None:
        self.capacity = (numel + 127) // 128 * 128
        self.bufs = [self.fab.alloc(self.capacity * self.world, torch.bfloat16) for _ in range(2)]

    def gemm_allreduce(self, a: torch.Tensor, w: torch.Tensor, b_mn: bool = False, alpha: float = 1.0,
                       a2: torch.Tensor | None = None, b2: torch.Tensor | None = None,
                       res: torch.Tensor | None = None) -> torch.Tensor:
        """sum over TP ranks of alpha * (a B^T (+ a2 B2^T)) (+ res), on every rank.
        ``w`` holds B(n, k) K-major [N, K] (``b_mn`` False) or MN-major [K, N]."""
        M = a.shape[0]
        N = w.shape[1] if b_mn else w.shape[0]
        n = M * N
        if n > self.capacity:
            self._grow(int(n * 1.25))  # same decision on every rank: shapes are in lockstep
        buf = self.bufs[self.flip]
        self.flip ^= 1
        m = ops.ext()
        with nvtx.range("tp.gemm_allreduce"):
            m.gemm_peer(a.contiguous(), w, b_mn, N, alpha, a2, b2, buf.ptrs, self.rank, self.rank * self.capacity, N,
                        0)
            self.fab.barrier()
            out = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
            m.slots_sum(buf.tensor, self.world, self.capacity, n, None if res is None else res.contiguous(), out)
        return out

    def check(self) -> None:
        self.fab.check()
