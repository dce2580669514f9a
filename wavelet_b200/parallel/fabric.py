"""Peer-memory fabric: buffers that every rank of a node can load and store.

Each rank allocates its buffer with ``cudaMalloc`` (outside the PyTorch
caching allocator), exports a CUDA IPC handle, and opens every peer's handle,
so every rank holds one device pointer per rank for the same logical buffer.
The fused collective kernels (``csrc/comm.cu``) take those pointer lists and
move data over NVLink with plain loads and stores from inside the kernel that
also does the math: the B200-native replacement for the NCCL
reduce-scatter / all-gather pair that FSDP issues around the optimizer
(reference: trainer/model.py:1136-1195 wraps blocks with FSDP2 whose
collectives run in NCCL).

Cross-rank ordering uses signal pads (``Fabric.pads``) with monotonically
increasing epochs and bounded waits; a wait that runs out sets an error bit
that ``check()`` turns into an exception on the host.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .. import ops

PAD_WORDS = 256
SLOT_BARRIER = 0
SLOT_NORM = 8
ERR_TIMEOUT_PEER = 1 << 4


class PeerTimeoutError(RuntimeError):
    pass


@dataclass
class SharedBuffer:
    tensor: torch.Tensor  # this rank's buffer
    ptrs: list[int]  # device pointer of rank r's buffer, valid on this rank
    owned: int = 0
    imported: list[int] = field(default_factory=list)


class Fabric:
    def __init__(self, rank: int, world: int, device: torch.device, group=None, budget_s: float = 60.0):
        if world > 8:
            raise ValueError("the peer fabric spans at most 8 GPUs (one NVLink node)")
        self.rank = rank
        self.world = world
        self.device = torch.device(device)
        self.group = group
        self.budget_s = budget_s
        self.m = ops.ext()
        self._bufs: list[SharedBuffer] = []
        self._epoch = {SLOT_BARRIER: 0, SLOT_NORM: 0}
        self.pads = self.alloc(PAD_WORDS, torch.int32)

    # ---------------------------------------------------------------- memory
    def alloc(self, numel: int, dtype: torch.dtype) -> SharedBuffer:
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        p = self.m.fabric_malloc(nbytes, dev)
        torch.cuda.synchronize(self.device)
        handle = self.m.fabric_export(p)
        handles: list = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, handle, group=self.group)
        else:
            handles = [handle]
        ptrs, imported = [], []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(p)
            else:
                q = self.m.fabric_import(handles[r], dev)
                ptrs.append(q)
                imported.append(q)
        t = self.m.from_ptr(p, numel, dtype, dev)
        buf = SharedBuffer(t, ptrs, p, imported)
        self._bufs.append(buf)
        return buf

    def allocator(self):
        """``(numel, dtype) -> tensor`` for ``FlatParams``; remembers the peers."""
        def alloc(numel: int, dtype: torch.dtype) -> torch.Tensor:
            return self.alloc(numel, dtype).tensor
        return alloc

    def ptrs_of(self, t: torch.Tensor) -> list[int]:
        base = t.data_ptr()
        for b in self._bufs:
            lo = b.tensor.data_ptr()
            hi = lo + b.tensor.numel() * b.tensor.element_size()
            if lo <= base < hi:
                off = base - lo
                return [p + off for p in b.ptrs]
        raise KeyError("tensor is not in fabric memory")

    # ---------------------------------------------------------------- sync
    def next_epoch(self, slot: int) -> int:
        self._epoch[slot] += 1
        return self._epoch[slot]

    def barrier(self) -> None:
        """Device-side barrier over the node (ordered on the current stream)."""
        e = self.next_epoch(SLOT_BARRIER)
        self.m.peer_barrier(self.pads.ptrs, self.rank, self.world, e, SLOT_BARRIER, self.budget_s)

    def check(self) -> None:
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        err = self.m.read_error(dev)
        if err & ERR_TIMEOUT_PEER:
            self.m.clear_error(dev)
            raise PeerTimeoutError(f"rank {self.rank}: a peer did not reach the fabric barrier within {self.budget_s}s")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for b in self._bufs:
            for q in b.imported:
                self.m.fabric_close(q)
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)
        for b in self._bufs:
            self.m.fabric_free(b.owned)
        self._bufs.clear()


def maybe_fabric(world: int, rank: int, device, group=None) -> Fabric | None:
    """A fabric for multi-GPU runs on one node with the CUDA extension loaded."""
    dev = torch.device(device)
    if world <= 1 or dev.type != "cuda" or world > 8:
        return None
    local = torch.cuda.device_count()
    if local < world:
        return None  # ranks span nodes: NCCL only
    return Fabric(rank, world, dev, group)
