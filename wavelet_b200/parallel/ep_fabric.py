"""Expert-parallel dispatch / combine over peer memory (one NVLink node).

The NCCL path of ``models.moe`` moves token copies with two variable-split
all-to-alls per direction and separate gather / scatter / weighting passes.
Here every rank owns four peer-visible row buffers (fabric memory):
``xs`` (expert inputs), ``y`` (expert outputs), ``dy`` and ``dxs`` (their
gradients), each laid out exactly as the grouped GEMM wants it: rows grouped
by local expert, each expert segment padded to 128 rows, and inside a
segment the rows of source rank 0, then 1, ...

Forward of one MoE layer (all ranks in lockstep):
  1. counts: every rank all-gathers its per-expert copy counts (tiny), so all
     ranks know every destination's layout and the row of every copy;
  2. dispatch (``rows_scatter``): each rank stores its token rows straight
     into the destination rank's ``xs`` row over NVLink -> barrier;
  3. padding rows zeroed locally; grouped tcgen05 expert GEMMs on ``xs``,
     writing ``y`` -> barrier;
  4. combine (``rows_gather_sum``): each token loads its k expert outputs from
     the owning ranks and forms x2 + sum_k w_k y_k in one pass.
Backward mirrors it: ``dy`` rows (dout scaled by the routing weight) are
dispatched, the expert backward runs locally, and ``dxs`` rows are gathered
back and summed per token.  Each direction costs the bytes of the NCCL path
but no staging copies, and the gather, weighting and residual add ride on
the transfers.  Buffers hold ``capacity`` rows and grow (on every rank at
once: the decision is made on the all-gathered counts) when a layout does not
fit.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops
from ..utils import nvtx
from .fabric import Fabric

PAD = 128


@dataclass
class FabricPlan:
    R: int  # rows of this rank's padded layout
    tile_group: torch.Tensor
    k_start: torch.Tensor
    k_len: torch.Tensor
    pad_rows: torch.Tensor  # rows of the layout that receive no copy (zeroed)
    dst_rank: torch.Tensor  # int32 [T*k] rank owning each copy's expert ((token, slot) order)
    dst_row: torch.Tensor  # int64 [T*k] row of the copy in that rank's layout
    src_tok: torch.Tensor  # int64 [T*k] token of each copy
    counts: torch.Tensor  # this rank's per-expert copy counts


class FabricEP:
    def __init__(self, fabric: Fabric, group, E: int, H: int, capacity: int, dtype=torch.bfloat16):
        self.fab = fabric
        self.group = group
        self.ep = fabric.world
        self.rank = fabric.rank
        self.E = E
        self.El = E // self.ep
        self.H = H
        self.capacity = capacity
        self.bufs = {n: fabric.alloc(capacity * H, dtype) for n in ("xs", "y", "dy", "dxs")}

    def view(self, name: str, rows: int) -> torch.Tensor:
        return self.bufs[name].tensor[: rows * self.H].view(rows, self.H)

    def ptrs(self, name: str) -> list[int]:
        return self.bufs[name].ptrs

    # ------------------------------------------------------------------ plan
    def plan(self, topi: torch.Tensor) -> FabricPlan:
        T, k = topi.shape
        dev = topi.device
        e = topi.reshape(-1)
        cnt = torch.bincount(e, minlength=self.E).to(torch.int32)
        allc = torch.empty(self.ep * self.E, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allc, cnt, group=self.group)
        C = allc.view(self.ep, self.E).tolist()  # host sync: the layouts size the grouped GEMMs
        El = self.El
        seg_start = [[0] * El for _ in range(self.ep)]
        Rs = []
        for d in range(self.ep):
            acc = 0
            for el in range(El):
                seg_start[d][el] = acc
                n = sum(C[s][d * El + el] for s in range(self.ep))
                acc += (n + PAD - 1) // PAD * PAD
            Rs.append(max(acc, PAD))
        if max(Rs) > self.capacity:
            # every rank sees the same counts, so all grow together (collective handle exchange)
            self.capacity = int(max(Rs) * 1.25)
            self.bufs = {n: self.fab.alloc(self.capacity * self.H, torch.bfloat16) for n in ("xs", "y", "dy", "dxs")}
        base = []
        for ge in range(self.E):
            d, el = divmod(ge, El)
            base.append(seg_start[d][el] + sum(C[s][ge] for s in range(self.rank)))
        base_t = torch.tensor(base, dtype=torch.int64, device=dev)
        order = torch.argsort(e, stable=True)
        cum = torch.zeros(self.E + 1, dtype=torch.int64, device=dev)
        cum[1:] = cnt.to(torch.int64).cumsum(0)
        rank_in = torch.empty_like(order)
        rank_in[order] = torch.arange(e.numel(), device=dev) - cum[e[order]]
        dst_row = base_t[e] + rank_in
        dst_rank = (e // El).to(torch.int32)
        # this rank's receive layout
        me = self.rank
        tiles, kl, pads = [], [], []
        for el in range(El):
            n = sum(C[s][me * El + el] for s in range(self.ep))
            padded = (n + PAD - 1) // PAD * PAD
            tiles += [el] * (padded // PAD)
            kl.append(padded)
            pads += range(seg_start[me][el] + n, seg_start[me][el] + padded)
        if not tiles:
            tiles = [0]
        R = Rs[me]
        return FabricPlan(
            R=R, tile_group=torch.tensor(tiles, dtype=torch.int32, device=dev),
            k_start=torch.tensor(seg_start[me], dtype=torch.int32, device=dev),
            k_len=torch.tensor(kl, dtype=torch.int32, device=dev),
            pad_rows=torch.tensor(pads, dtype=torch.int64, device=dev),
            dst_rank=dst_rank, dst_row=dst_row,
            src_tok=torch.arange(T, device=dev).repeat_interleave(k), counts=cnt)

    # --------------------------------------------------------------- transfers
    def dispatch(self, name: str, src: torch.Tensor, p: FabricPlan, scale: torch.Tensor | None = None) -> torch.Tensor:
        """Rows of ``src`` (one per copy, optionally scaled) into every owner's
        ``name`` buffer; returns this rank's received [R, H] view."""
        with nvtx.range(f"ep.dispatch.{name}"):
            ops.ext().rows_scatter(src, p.src_tok, p.dst_rank, p.dst_row, scale, self.ptrs(name), self.ep, self.H)
            self.fab.barrier()
        out = self.view(name, p.R)
        if p.pad_rows.numel():
            out.index_fill_(0, p.pad_rows, 0)
        return out

    def combine(self, name: str, p: FabricPlan, k: int, w: torch.Tensor | None, res: torch.Tensor | None,
                out: torch.Tensor) -> torch.Tensor:
        """out[t] = res[t] + sum_j w[t, j] * owner_rows[copy (t, j)] (after a barrier
        that orders the owners' writes of ``name``)."""
        with nvtx.range(f"ep.combine.{name}"):
            self.fab.barrier()
            ops.ext().rows_gather_sum(self.ptrs(name), self.ep, self.H, p.dst_rank, p.dst_row,
                                      None if w is None else w.reshape(-1).float().contiguous(), k, res, out)
        return out

    def gather_copies(self, name: str, p: FabricPlan, T: int, k: int) -> torch.Tensor:
        """The [T*k, H] rows of this rank's copies (no sum)."""
        out = torch.empty(T * k, self.H, device=p.dst_row.device, dtype=torch.bfloat16)
        ops.ext().rows_gather_sum(self.ptrs(name), self.ep, self.H, p.dst_rank, p.dst_row, None, 1, None, out)
        return out

    def close(self) -> None:
        pass  # buffers belong to the fabric (freed by Fabric.close)
