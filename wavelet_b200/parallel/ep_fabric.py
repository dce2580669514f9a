"""Expert-parallel dispatch / combine over peer memory (one NVLink node).

The NCCL path of ``models.moe`` moves token copies with two variable-split
all-to-alls per direction and separate gather / scatter / weighting passes.
Here every rank owns four peer-visible row buffers (fabric memory):
``xs`` (expert inputs), ``y`` (expert outputs), ``dy`` and ``dxs`` (their
gradients), each laid out exactly as the grouped GEMM wants it: rows grouped
by local expert, each expert segment padded to 128 rows, and inside a
segment the rows of source rank 0, then 1, ...

Forward of one MoE layer (all ranks in lockstep, no host synchronisation):
  1. counts: every rank stores its per-expert copy counts into every peer's
     count table (``moe_put_counts``) -> barrier; each rank then builds, on
     the device, every destination's layout and the row of each of its copies
     (``moe_layout`` / ``moe_copy_rows``), identically on all ranks;
  2. dispatch (``rows_scatter``): each rank stores its token rows straight
     into the destination rank's ``xs`` row over NVLink -> barrier;
  3. padding rows zeroed locally; grouped tcgen05 expert GEMMs on ``xs`` (tiles
     past the used rows are skipped), writing ``y`` -> barrier;
  4. combine (``rows_gather_sum``): each token loads its k expert outputs from
     the owning ranks and forms x2 + sum_k w_k y_k in one pass.
Backward mirrors it: ``dy`` rows (dout scaled by the routing weight) are
dispatched, the expert backward runs locally, and ``dxs`` rows are gathered
back and summed per token.  Each direction costs the bytes of the NCCL path
but no staging copies, and the gather, weighting and residual add ride on
the transfers.  Buffers hold ``capacity`` rows, fixed at construction: by
default the worst case (every rank sends each of its ``max_tokens`` tokens to
min(k, experts per rank) experts of one rank), or ``capacity_factor`` x the
average copies per rank to save memory, plus a padding tile per local expert.
A layout that would not fit is detected on the device: that layer's layout
is empty and its transfers are skipped (nothing is written or read past a
buffer, nothing unwritten is read), and ``check()`` raises before the
optimizer step: raise ``fsdp.ep_capacity_factor`` or leave it unset.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops
from ..utils import nvtx
from .fabric import Fabric

PAD = 128
ERR_EP_OVERFLOW = 1 << 6  # csrc/common.cuh kErrEpOverflow


@dataclass
class FabricPlan:
    R: int  # rows of this rank's layout buffers (the capacity)
    tile_group: torch.Tensor  # int32 [R / 128]: local expert of each tile, -1 past the used rows
    k_start: torch.Tensor  # int32 [El]: segment start of each local expert
    k_len: torch.Tensor  # int32 [El]: padded segment length
    n_recv: torch.Tensor  # int32 [El]: received copies per local expert
    overflow: torch.Tensor  # int32 [1]: 1 when some rank's layout exceeded the capacity
    dst_rank: torch.Tensor  # int32 [T*k] rank owning each copy's expert ((token, slot) order)
    dst_row: torch.Tensor  # int64 [T*k] row of the copy in that rank's layout
    src_tok: torch.Tensor  # int64 [T*k] token of each copy
    counts: torch.Tensor  # int32 [E]: this rank's per-expert copy counts


class EPCapacityError(RuntimeError):
    pass


class FabricEP:
    def __init__(self, fabric: Fabric, group, E: int, H: int, capacity: int, dtype=torch.bfloat16, k: int = 8,
                 max_tokens: int = 0, capacity_factor: float | None = None):
        self.fab = fabric
        self.group = group
        self.ep = fabric.world
        self.rank = fabric.rank
        self.E = E
        self.El = E // self.ep
        self.H = H
        if max_tokens > 0:
            # worst case per destination: every token sends one copy to each of
            # up to min(k, El) of its experts, from every rank
            worst = self.ep * max_tokens * min(k, self.El)
            rows = worst if capacity_factor is None or capacity_factor <= 0 else \
                min(worst, int(capacity_factor * max_tokens * k))
            capacity = max(capacity, rows + self.El * PAD)
        self.capacity = (capacity + PAD - 1) // PAD * PAD
        self.bufs = {n: fabric.alloc(self.capacity * H, dtype) for n in ("xs", "y", "dy", "dxs")}
        self.cnt = fabric.alloc(self.ep * E, torch.int32)  # every rank's per-expert counts

    def view(self, name: str, rows: int) -> torch.Tensor:
        return self.bufs[name].tensor[: rows * self.H].view(rows, self.H)

    def ptrs(self, name: str) -> list[int]:
        return self.bufs[name].ptrs

    # ------------------------------------------------------------------ plan
    def plan(self, topi: torch.Tensor, counts: torch.Tensor | None = None) -> FabricPlan:
        T, k = topi.shape
        dev = topi.device
        m = ops.ext()
        e = topi.reshape(-1).contiguous()
        if counts is None:
            counts = torch.bincount(e, minlength=self.E).to(torch.int32)
        with nvtx.range("ep.plan"):
            m.moe_put_counts(self.cnt.ptrs, self.ep, self.rank, counts)
            self.fab.barrier()
            El = self.El
            base = torch.empty(self.E, dtype=torch.int64, device=dev)
            tile_group = torch.empty(self.capacity // PAD, dtype=torch.int32, device=dev)
            k_start = torch.empty(El, dtype=torch.int32, device=dev)
            k_len = torch.empty(El, dtype=torch.int32, device=dev)
            n_recv = torch.empty(El, dtype=torch.int32, device=dev)
            rows = torch.empty(1, dtype=torch.int32, device=dev)
            overflow = torch.empty(1, dtype=torch.int32, device=dev)
            m.moe_layout(self.cnt.tensor, self.ep, self.rank, PAD, self.capacity, base, tile_group, k_start, k_len,
                         n_recv, rows, overflow)
            dst_row = torch.empty(T * k, dtype=torch.int64, device=dev)
            dst_rank = torch.empty(T * k, dtype=torch.int32, device=dev)
            m.moe_copy_rows(e, self.E, El, base, dst_row, dst_rank)
        return FabricPlan(R=self.capacity, tile_group=tile_group, k_start=k_start, k_len=k_len, n_recv=n_recv,
                          overflow=overflow, dst_rank=dst_rank, dst_row=dst_row,
                          src_tok=torch.arange(T, device=dev).repeat_interleave(k), counts=counts)

    # --------------------------------------------------------------- transfers
    def dispatch(self, name: str, src: torch.Tensor, p: FabricPlan, scale: torch.Tensor | None = None) -> torch.Tensor:
        """Rows of ``src`` (one per copy, optionally scaled) into every owner's
        ``name`` buffer; returns this rank's received [R, H] view."""
        with nvtx.range(f"ep.dispatch.{name}"):
            ops.ext().rows_scatter(src, p.src_tok, p.dst_rank, p.dst_row, scale, self.ptrs(name), self.ep, self.H,
                                   self.capacity)
            self.fab.barrier()
        out = self.view(name, p.R)
        ops.ext().moe_zero_pad(out, p.k_start, p.k_len, p.n_recv, p.overflow)
        return out

    def combine(self, name: str, p: FabricPlan, k: int, w: torch.Tensor | None, res: torch.Tensor | None,
                out: torch.Tensor) -> torch.Tensor:
        """out[t] = res[t] + sum_j w[t, j] * owner_rows[copy (t, j)] (after a barrier
        that orders the owners' writes of ``name``)."""
        with nvtx.range(f"ep.combine.{name}"):
            self.fab.barrier()
            ops.ext().rows_gather_sum(self.ptrs(name), self.ep, self.H, p.dst_rank, p.dst_row,
                                      None if w is None else w.reshape(-1).float().contiguous(), k, res, out,
                                      self.capacity)
        return out

    def gather_copies(self, name: str, p: FabricPlan, T: int, k: int) -> torch.Tensor:
        """The [T*k, H] rows of this rank's copies (no sum)."""
        out = torch.empty(T * k, self.H, device=p.dst_row.device, dtype=torch.bfloat16)
        ops.ext().rows_gather_sum(self.ptrs(name), self.ep, self.H, p.dst_rank, p.dst_row, None, 1, None, out,
                                  self.capacity)
        return out

    def check(self) -> None:
        """Raise when a layer's layout exceeded the buffer capacity (its
        transfers were skipped, so that step's results are invalid)."""
        dev = self.fab.device.index if self.fab.device.index is not None else torch.cuda.current_device()
        m = ops.ext()
        err = m.read_error(dev)
        if err & ERR_EP_OVERFLOW:
            m.clear_error(dev)
            raise EPCapacityError(f"rank {self.rank}: an expert-parallel layout exceeded the {self.capacity}-row "
                                  "buffers; raise fsdp.ep_capacity_factor")

    def close(self) -> None:
        pass  # buffers belong to the fabric (freed by Fabric.close)
