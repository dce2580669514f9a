"""Policy transfer from the trainer to the generator.

Filesystem transfer (``policy_transfer.type: filesystem``): rank 0 writes
``<policy_dir>/step-XXXXXX/`` with the model in Hugging Face safetensors
layout (or only the LoRA adapter when ``lightweight_lora``), ``policy.json``
and finally ``STABLE``; older snapshots beyond ``keep_last`` are pruned
(transport/policy.py:564-915 of the reference).

Device transfer (``policy_transfer.type: nccl``): the generator receives the
trainer's bf16 weights without touching the filesystem.  Both sides use the
same flat parameter layout, so a transfer is one contiguous buffer:

* same process (integrated launcher): the generator reads the trainer's
  compute buffer in place (zero copy);
* separate processes on one node: the trainer's buffer is exported through
  CUDA IPC and the generator pulls it with a copy kernel over NVLink, or a
  NCCL broadcast over a trainer-rank-0 + generator group
  (``DeviceWeightBroadcaster``).  A ``layerwise_v1``-style ``update_info.json``
  records the protocol in the policy directory.
"""

from __future__ import annotations

import json
import os
import shutil
import time
from pathlib import Path
from typing import Any

import torch

from .queue import POLICY_META, STABLE, resolve_policy_dir, stable_steps, step_dir, utc_now


class PolicyExporter:
    def __init__(self, output_dir: Path, cfg, rank: int = 0, lora=None):
        self.cfg = cfg
        self.rank = rank
        self.output_dir = Path(output_dir)
        self.policy_dir = resolve_policy_dir(output_dir, cfg)
        self.lora = lora
        self.broadcaster = None

    def export(self, model, step: int) -> Path | None:
        if self.cfg.type == "nccl":
            return self._export_device(model, step)
        if self.rank != 0:
            return None
        d = step_dir(self.policy_dir, step)
        if (d / STABLE).exists():
            return d
        tmp = d.with_name(d.name + f".tmp-{os.getpid()}")
        if tmp.exists():
            shutil.rmtree(tmp)
        tmp.mkdir(parents=True)
        t0 = time.perf_counter()
        kind = "model"
        if self.lora is not None and self.cfg.lightweight_lora:
            self.lora.save_adapter(tmp / "adapter")
            kind = "adapter"
        else:
            from ..models.hf_io import save_hf

            save_hf(model, tmp / "model")
        meta = {"step": step, "kind": kind, "created_at": utc_now(), "export_seconds": time.perf_counter() - t0,
                "adapter_name": self.cfg.adapter_name, "adapter_id": self.cfg.adapter_id,
                "arch": model.cfg.to_dict()}
        (tmp / POLICY_META).write_text(json.dumps(meta, indent=2))
        if d.exists():
            shutil.rmtree(d)
        os.replace(tmp, d)
        (d / STABLE).touch()
        self._prune()
        return d

    def _export_device(self, model, step: int) -> Path | None:
        """Announce a device-transfer policy; the bytes move through the broadcaster."""
        if self.rank == 0:
            d = step_dir(self.policy_dir, step)
            d.mkdir(parents=True, exist_ok=True)
            (d / "update_info.json").write_text(json.dumps({"protocol": "flat_v1", "numel": model.flat.numel,
                                                             "dtype": str(model.flat.compute_dtype)}))
            (d / POLICY_META).write_text(json.dumps({"step": step, "kind": "device", "created_at": utc_now()}))
            (d / STABLE).touch()
            self._prune()
        if self.broadcaster is not None:
            self.broadcaster.broadcast(model.flat.compute)
        return None

    def _prune(self) -> None:
        steps = stable_steps(self.policy_dir)
        for s in steps[: -self.cfg.keep_last] if len(steps) > self.cfg.keep_last else []:
            shutil.rmtree(step_dir(self.policy_dir, s), ignore_errors=True)


def load_policy_into(model, snapshot_dir: Path) -> dict[str, Any]:
    """Load a filesystem policy snapshot into a generator model (same arch)."""
    meta = json.loads((Path(snapshot_dir) / POLICY_META).read_text())
    if meta.get("kind") == "model":
        from ..models.hf_io import load_hf_weights

        load_hf_weights(model, Path(snapshot_dir) / "model")
    elif meta.get("kind") == "adapter":
        from ..models.lora import merge_adapter_into

        merge_adapter_into(model, Path(snapshot_dir) / "adapter")
    return meta


class DeviceWeightBroadcaster:
    """Broadcast the flat bf16 compute buffer from trainer rank 0 to generator
    ranks over a dedicated NCCL group (one collective per policy update)."""

    def __init__(self, group, src_rank: int = 0):
        self.group = group
        self.src = src_rank

    def broadcast(self, buf: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.broadcast(buf.detach(), src=self.src, group=self.group)
