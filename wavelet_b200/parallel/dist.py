"""Process-group bootstrap and parallel-dimension bookkeeping.

One process per GPU.  ``init_distributed`` reads the torchrun environment
(RANK / LOCAL_RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT), selects NCCL for
CUDA ranks and gloo for CPU ranks, and creates the device mesh sub-groups:

    world = dp_replicate x dp_shard x cp x tp      (ep carved out of dp_shard x cp)

Parity: trainer/distributed.py:26-256 (ParallelDims and the flattened
``dp``/``dp_cp``/``ep``/``tp`` meshes) and the hybrid ``cpu:gloo,cuda:nccl``
init at trainer/trainer.py:519-589.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


@dataclass
class World:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    local_world_size: int = 1
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))

    @property
    def is_master(self) -> bool:
        return self.rank == 0

    @property
    def distributed(self) -> bool:
        return self.world_size > 1


def get_world() -> World:
    rank = int(os.environ.get("RANK", 0))
    ws = int(os.environ.get("WORLD_SIZE", 1))
    lr = int(os.environ.get("LOCAL_RANK", 0))
    lws = int(os.environ.get("LOCAL_WORLD_SIZE", ws))
    if torch.cuda.is_available() and os.environ.get("WAVELET_FORCE_CPU", "0") != "1":
        dev = torch.device("cuda", lr % max(1, torch.cuda.device_count()))
    else:
        dev = torch.device("cpu")
    return World(rank, ws, lr, lws, dev)


def init_distributed(backend: str = "auto", timeout_s: float = 600.0) -> World:
    """Initialise the default process group when WORLD_SIZE > 1."""
    w = get_world()
    if w.device.type == "cuda":
        torch.cuda.set_device(w.device)
    if w.world_size > 1 and not dist.is_initialized():
        if backend == "auto":
            backend = "nccl" if w.device.type == "cuda" else "gloo"
        elif backend == "hybrid":
            backend = "cpu:gloo,cuda:nccl"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if "nccl" in backend and w.device.type == "cuda":
            kwargs["device_id"] = w.device
        dist.init_process_group(**kwargs)
    return w


def destroy_distributed() -> None:
    if dist.is_initialized():
        try:
            dist.barrier()
        except Exception:
            pass
        dist.destroy_process_group()


@dataclass
class ParallelDims:
    dp_replicate: int = 1
    dp_shard: int = -1
    cp: int = 1
    tp: int = 1
    ep: int = 1
    pp: int = 1
    world_size: int = 1

    def __post_init__(self):
        fixed = self.dp_replicate * self.cp * self.tp * self.pp
        if self.dp_shard == -1:
            if self.world_size % fixed:
                raise ValueError(f"world size {self.world_size} not divisible by dp_replicate*cp*tp*pp={fixed}")
            self.dp_shard = self.world_size // fixed
        if self.dp_replicate * self.dp_shard * self.cp * self.tp * self.pp != self.world_size:
            raise ValueError(
                f"dp_replicate({self.dp_replicate}) * dp_shard({self.dp_shard}) * cp({self.cp}) * "
                f"tp({self.tp}) * pp({self.pp}) != world_size({self.world_size})"
            )
        if self.ep > 1:
            if (self.dp_shard * self.cp) % self.ep:
                raise ValueError("ep must divide dp_shard * cp")
            if self.tp > 1:
                raise ValueError("expert parallelism cannot be combined with tensor parallelism")
        if self.pp > 1:
            raise ValueError("pipeline parallelism is not supported (pp must be 1)")

    @property
    def dp(self) -> int:
        return self.dp_replicate * self.dp_shard

    def coords(self, rank: int) -> dict[str, int]:
        # rank layout: [dp_replicate][dp_shard][cp][tp] with tp fastest
        tp = rank % self.tp
        r = rank // self.tp
        cp = r % self.cp
        r //= self.cp
        dps = r % self.dp_shard
        dpr = r // self.dp_shard
        return {"tp": tp, "cp": cp, "dp_shard": dps, "dp_replicate": dpr}


class Groups:
    """Process sub-groups built from ParallelDims (created collectively)."""

    def __init__(self, dims: ParallelDims, rank: int):
        self.dims = dims
        self.rank = rank
        self.dp = None  # data parallel (replicate x shard), tp/cp fixed
        self.tp = None
        self.cp = None
        self.ep = None
        self.ep_dp = None  # ranks holding the same expert shard (dp_mod_ep)
        self.ep_dp_rank = 0
        self.ep_dp_size = dims.world_size // max(1, dims.ep)
        self.dp_rank = 0
        self.dp_size = dims.dp
        self.tp_rank = 0
        self.ep_rank = 0
        self.cp_rank = 0
        self.cp_size = dims.cp
        # dp x cp: the ranks that hold the same parameters (gradients and
        # optimizer shards reduce over them; the reference's dp_cp mesh)
        self.dp_cp = None
        self.dp_cp_rank = 0
        self.dp_cp_size = dims.dp * dims.cp
        # hybrid sharding (HSDP, sharded parameters with dp_replicate > 1):
        # one copy of the sharded model per replica over dp_shard x cp
        # ("shard"), gradients all-reduced across the replicas ("replicate")
        self.shard = None
        self.shard_rank = 0
        self.shard_size = dims.dp_shard * dims.cp
        self.replicate = None
        self.replicate_rank = 0
        self.replicate_size = dims.dp_replicate
        if not dist.is_initialized() or dims.world_size == 1:
            return
        W = dims.world_size
        c = dims.coords(rank)
        self.tp_rank = c["tp"]
        # data-parallel groups: same (cp, tp)
        for cp in range(dims.cp):
            for tp in range(dims.tp):
                ranks = [r for r in range(W) if dims.coords(r)["cp"] == cp and dims.coords(r)["tp"] == tp]
                g = dist.new_group(ranks)
                if rank in ranks:
                    self.dp = g
                    self.dp_rank = ranks.index(rank)
        for base in range(0, W, dims.tp):
            ranks = list(range(base, base + dims.tp))
            g = dist.new_group(ranks) if dims.tp > 1 else None
            if rank in ranks:
                self.tp = g
        self.cp_rank = c["cp"]
        if dims.cp > 1:
            # context-parallel groups: same data-parallel coordinates and tp
            seen = set()
            for r0 in range(W):
                c0 = dims.coords(r0)
                key = (c0["dp_replicate"], c0["dp_shard"], c0["tp"])
                if key in seen:
                    continue
                seen.add(key)
                ranks = [r for r in range(W) if (dims.coords(r)["dp_replicate"], dims.coords(r)["dp_shard"],
                                                 dims.coords(r)["tp"]) == key]
                g = dist.new_group(ranks)
                if rank in ranks:
                    self.cp = g
            for tp in range(dims.tp):
                ranks = [r for r in range(W) if dims.coords(r)["tp"] == tp]
                g = dist.new_group(ranks)
                if rank in ranks:
                    self.dp_cp = g
                    self.dp_cp_rank = ranks.index(rank)
        else:
            self.dp_cp, self.dp_cp_rank = self.dp, self.dp_rank
        if dims.dp_replicate > 1:
            seen_s, seen_r = set(), set()
            for r0 in range(W):
                c0 = dims.coords(r0)
                ks, kr = (c0["dp_replicate"], c0["tp"]), (c0["dp_shard"], c0["cp"], c0["tp"])
                if ks not in seen_s:
                    seen_s.add(ks)
                    ranks = [r for r in range(W) if (dims.coords(r)["dp_replicate"], dims.coords(r)["tp"]) == ks]
                    g = dist.new_group(ranks) if len(ranks) > 1 else None
                    if rank in ranks:
                        self.shard, self.shard_rank = g, ranks.index(rank)
                if kr not in seen_r:
                    seen_r.add(kr)
                    ranks = [r for r in range(W) if (dims.coords(r)["dp_shard"], dims.coords(r)["cp"],
                                                     dims.coords(r)["tp"]) == kr]
                    g = dist.new_group(ranks)
                    if rank in ranks:
                        self.replicate, self.replicate_rank = g, ranks.index(rank)
        else:
            self.shard, self.shard_rank = self.dp_cp, self.dp_cp_rank
        if dims.ep > 1:
            # contiguous blocks of ep ranks among the dp_shard x cp ranks
            for base in range(0, W, dims.ep):
                ranks = list(range(base, base + dims.ep))
                g = dist.new_group(ranks)
                if rank in ranks:
                    self.ep = g
                    self.ep_rank = ranks.index(rank)
            for j in range(dims.ep):
                ranks = list(range(j, W, dims.ep))
                g = dist.new_group(ranks) if len(ranks) > 1 else None
                if rank in ranks:
                    self.ep_dp = g
                    self.ep_dp_rank = ranks.index(rank)


def all_ranks_true(flag: bool, device: torch.device, group=None) -> bool:
    """Collective AND of a host flag (trainer/distributed.py:391-398)."""
    if not dist.is_initialized():
        return bool(flag)
    t = torch.tensor([1 if flag else 0], device=device, dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


def any_rank_true(flag: bool, device: torch.device, group=None) -> bool:
    if not dist.is_initialized():
        return bool(flag)
    t = torch.tensor([1 if flag else 0], device=device, dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return bool(t.item())
