"""Device, port and rank placement for process-mode RL
(orchestrator/placement.py:6-194 of the reference).

Splits the node's GPUs between the trainer and the inference replicas
(explicit ``launcher.*_cuda_visible_devices`` or an even split), assigns one
HTTP port per replica, and checks for overlaps.
"""

from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass
class Placement:
    trainer_devices: list[str]
    inference_devices: list[list[str]]  # one group per replica
    ports: list[int]
    host: str


def _as_list(v) -> list[str] | None:
    if v is None:
        return None
    if isinstance(v, str):
        return [x.strip() for x in v.split(",") if x.strip()]
    return [str(x) for x in v]


def visible_devices(total: int | None = None) -> list[str]:
    env = os.environ.get("CUDA_VISIBLE_DEVICES")
    if env:
        return [x for x in env.split(",") if x]
    if total is None:
        try:
            import torch

            total = torch.cuda.device_count()
        except Exception:
            total = 0
    return [str(i) for i in range(total)]


def plan(cfg, available: list[str] | None = None) -> Placement:
    lc = cfg.launcher
    avail = available if available is not None else visible_devices()
    reps = lc.inference_num_replicas
    h = cfg.inference.http
    if not avail and lc.trainer_cuda_visible_devices is None and lc.inference_cuda_visible_devices is None:
        # CPU-only host: roles run without device pinning
        ports = list(h.ports) if h.ports else [h.port + r for r in range(reps)]
        return Placement([], [[] for _ in range(reps)], ports, h.host)
    t = _as_list(lc.trainer_cuda_visible_devices)
    i = _as_list(lc.inference_cuda_visible_devices)
    if lc.mode in ("colocate", "colocate_sleep"):
        t = t or avail[: lc.trainer_num_processes]
        i = i or list(t)
    else:
        if t is None and i is None:
            n_t = lc.trainer_num_processes
            if n_t + reps > len(avail):
                raise ValueError(f"need {n_t} trainer + {reps} inference GPUs but only {len(avail)} are visible")
            t = avail[:n_t]
            i = avail[n_t:]
        elif t is None:
            t = [d for d in avail if d not in i][: lc.trainer_num_processes]
        elif i is None:
            i = [d for d in avail if d not in t]
        overlap = set(t) & set(i)
        if overlap:
            raise ValueError(f"trainer and inference devices overlap: {sorted(overlap)}")
    if t and len(t) != lc.trainer_num_processes:
        raise ValueError(f"launcher.trainer_num_processes={lc.trainer_num_processes} but {len(t)} trainer devices")
    if reps < 1 or (i and len(i) < reps):
        raise ValueError("not enough inference devices for the requested replicas")
    per = max(1, len(i) // reps) if i else 0
    groups = [i[r * per : (r + 1) * per] for r in range(reps)] if i else [[] for _ in range(reps)]
    ports = list(h.ports) if h.ports else [h.port + r for r in range(reps)]
    if len(ports) != reps:
        raise ValueError("inference.http.ports must list one port per replica")
    return Placement(t, groups, ports, h.host)
