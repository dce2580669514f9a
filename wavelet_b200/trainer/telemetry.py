"""Per-rank step telemetry aggregated per node.

Each rank contributes (tokens, seconds, allocated GiB, peak GiB) for the
optimizer step.  Node labels are exchanged once (``all_gather_object`` at
construction); afterwards every step moves one small float tensor with
``all_gather_into_tensor`` on the data-parallel backend, so the per-step cost
is one tiny collective instead of pickled objects.  Rank 0 turns the samples
into ``node/<name>/*`` metrics and a per-rank table for ``heartbeat.json``
(same metric names as the reference, trainer/telemetry.py:25-134).
"""

from __future__ import annotations

import os
import socket
from dataclasses import asdict, dataclass

import torch
import torch.distributed as dist

GIB = float(1 << 30)


def node_name() -> str:
    name = os.environ.get("WAVELET_NODE_NAME") or socket.gethostname() or "local"
    return name.strip().replace("/", "_") or "local"


@dataclass(frozen=True)
class RankSample:
    rank: int
    local_rank: int
    node: str
    device: str
    tokens: float
    seconds: float
    memory_allocated_gib: float
    peak_memory_gib: float

    @property
    def tokens_per_second(self) -> float:
        return self.tokens / max(self.seconds, 1e-9)


class Telemetry:
    def __init__(self, world=None, replication: int = 1):
        self.world = world
        self.replication = max(1, int(replication))
        self.rank = world.rank if world is not None else 0
        self.size = world.world_size if world is not None else 1
        self.device = world.device if world is not None else torch.device("cpu")
        me = (node_name(), str(self.device), world.local_rank if world is not None else 0)
        self.peers = [me]
        if self._collective():
            peers: list = [None] * self.size
            dist.all_gather_object(peers, me)
            self.peers = peers

    def _collective(self) -> bool:
        return self.size > 1 and dist.is_available() and dist.is_initialized()

    def sample(self, tokens: float, seconds: float) -> list[RankSample]:
        if self.device.type == "cuda":
            alloc = torch.cuda.memory_allocated(self.device) / GIB
            peak = torch.cuda.max_memory_reserved(self.device) / GIB
        else:
            alloc = peak = 0.0
        row = torch.tensor([tokens / self.replication, seconds, alloc, peak], dtype=torch.float64,
                           device=self.device if self.device.type == "cuda" else "cpu")
        if self._collective():
            allrows = torch.empty(self.size * 4, dtype=row.dtype, device=row.device)
            dist.all_gather_into_tensor(allrows, row)
            vals = allrows.view(self.size, 4).tolist()
        else:
            vals = [row.tolist()]
        out = []
        for r, v in enumerate(vals):
            node, dev, lr = self.peers[r]
            out.append(RankSample(r, lr, node, dev, v[0], v[1], v[2], v[3]))
        return out


def node_metrics(ranks: list[RankSample]) -> dict[str, float]:
    if not ranks:
        return {}
    by_node: dict[str, list[RankSample]] = {}
    for s in ranks:
        by_node.setdefault(s.node, []).append(s)
    m: dict[str, float] = {"perf/nodes": float(len(by_node))}
    for node, members in sorted(by_node.items()):
        sec = max(x.seconds for x in members)
        p = f"node/{node}"
        tok = sum(x.tokens for x in members)
        m[f"{p}/ranks"] = float(len(members))
        m[f"{p}/tokens"] = tok
        m[f"{p}/tokens_per_second"] = tok / max(sec, 1e-9)
        m[f"{p}/step_seconds"] = sec
        m[f"{p}/peak_memory_gib"] = max(x.peak_memory_gib for x in members)
        m[f"{p}/memory_allocated_gib"] = max(x.memory_allocated_gib for x in members)
    rates = [x.tokens_per_second for x in ranks]
    m["perf/rank_tokens_per_second_min"] = min(rates)
    m["perf/rank_tokens_per_second_max"] = max(rates)
    m["perf/rank_peak_memory_gib_max"] = max(x.peak_memory_gib for x in ranks)
    return m


def rank_rows(ranks: list[RankSample]) -> list[dict]:
    return [{**asdict(x), "tokens_per_second": x.tokens_per_second} for x in ranks]
