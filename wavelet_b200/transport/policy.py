"""Policy transfer from the trainer to the generator.

Filesystem transfer (``policy_transfer.type: filesystem``): rank 0 writes
``<policy_dir>/step-XXXXXX/`` with the model in Hugging Face safetensors
layout (or only the LoRA adapter when ``lightweight_lora``), ``policy.json``
and finally ``STABLE``; older snapshots beyond ``keep_last`` are pruned
(transport/policy.py:564-915 of the reference).

Device transfer (``policy_transfer.type: nccl``): the generator receives the
trainer's weights without touching the filesystem:

* same process (integrated launcher): the generator reads the trainer's
  compute buffer in place (zero copy);
* separate processes on one node: every trainer rank pushes its part of the
  weights into receive slots on the generator GPUs over peer memory,
  resharding and casting on the way (``peer_policy``; protocol ``peer_v1``);
* otherwise: trainer rank 0 broadcasts the flat buffer over a trainer-rank-0 +
  generators NCCL group after the generators mark themselves ready
  (protocol ``flat_v1``).

``update_info.json`` in the policy step directory records the protocol; the
step directory becomes STABLE once the weights are in place (peer) or when
the generators may join the broadcast (NCCL).
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
    def __init__(self, output_dir: Path, cfg, rank: int = 0, lora=None, world: int = 1, barrier=None):
        self.cfg = cfg
        self.rank = rank
        self.world = world
        self.barrier = barrier or (lambda: None)
        self.output_dir = Path(output_dir)
        self.policy_dir = resolve_policy_dir(output_dir, cfg)
        self.lora = lora
        self.broadcaster = None
        self.peer = None
        self.device_mode: str | None = None  # "peer" or "nccl", fixed at the first device export
        self.last_update: dict[str, Any] = {}

    def export(self, model, step: int) -> Path | None:
        if self.cfg.type == "nccl":
            return self._export_device(model, step)
        if getattr(model.flat, "sharded_compute", False) and not (self.lora is not None and self.cfg.lightweight_lora):
            model = _gathered_view(model)  # every rank takes part in the gathers; rank 0 writes
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

    def _choose_device_mode(self, model) -> str:
        """Peer push when every trainer rank reaches the generators' memory
        (same host, receivers announced), else the NCCL broadcast; the ranks
        agree on one answer."""
        from .peer_policy import PeerPolicySender, PeerUnavailable

        ok = True
        err = ""
        if self.cfg.peer:
            try:
                self.peer = PeerPolicySender(model, self.policy_dir, rank=self.rank, world=self.world,
                                             expect=self.cfg.nccl_inference_world_size,
                                             timeout_s=self.cfg.nccl_timeout_seconds, barrier=self.barrier)
            except PeerUnavailable as e:
                ok, err = False, str(e)
        else:
            ok, err = False, "peer transfer off"
        if self.world > 1:
            import torch.distributed as dist

            votes: list = [None] * self.world
            dist.all_gather_object(votes, ok)
            ok = all(votes)
        if not ok and self.peer is not None:
            self.peer.close()
            self.peer = None
        if not ok and self.rank == 0:
            import logging

            logging.getLogger(__name__).warning("device policy transfer over NCCL (%s)", err or "a rank cannot "
                                                "reach the generators' memory")
        return "peer" if ok else "nccl"

    def _write_device_step(self, model, step: int, info: dict[str, Any]) -> Path:
        d = step_dir(self.policy_dir, step)
        tmp = d.with_name(d.name + f".tmp-{os.getpid()}")
        if tmp.exists():
            shutil.rmtree(tmp)
        tmp.mkdir(parents=True)
        (tmp / "update_info.json").write_text(json.dumps(info))
        (tmp / POLICY_META).write_text(json.dumps({"step": step, "kind": "device", "created_at": utc_now(),
                                                   "arch": model.cfg.to_dict()}))
        if d.exists():
            shutil.rmtree(d)
        os.replace(tmp, d)
        (d / STABLE).touch()
        self._prune()
        return d

    def _export_device(self, model, step: int) -> Path | None:
        """Device transfer: peer push (every rank) or NCCL broadcast (rank 0)."""
        from .peer_policy import FLAT_PROTOCOL, PolicyBroadcastGroup, used_numel, wait_ready

        if self.device_mode is None:
            self.device_mode = self._choose_device_mode(model)
        if self.device_mode == "peer":
            info = self.peer.push(step)
            self.last_update = info
            return self._write_device_step(model, step, info) if self.rank == 0 else None
        if getattr(model, "tp_size", 1) > 1 or getattr(model, "expert_flat", None) is not None:
            raise NotImplementedError("the NCCL policy broadcast sends one flat buffer; tensor- or expert-parallel "
                                      "trainers need the peer transfer (generators on the trainer's node) or the "
                                      "filesystem transfer")
        d = None
        if self.rank == 0:
            n = used_numel(model.flat)
            info = {"protocol": FLAT_PROTOCOL, "numel": n, "dtype": str(model.flat.compute.dtype).removeprefix("torch.")}
            d = self._write_device_step(model, step, info)
            if self.broadcaster is None:
                c = self.cfg
                self.broadcaster = PolicyBroadcastGroup(c.nccl_host, c.nccl_port, 0, 1 + c.nccl_inference_world_size,
                                                        model.flat.compute.device, c.nccl_timeout_seconds,
                                                        backend="nccl" if model.flat.compute.is_cuda else "gloo")
            wait_ready(d, self.cfg.nccl_inference_world_size, self.cfg.nccl_timeout_seconds)
            t0 = time.perf_counter()
            self.broadcaster.broadcast(model.flat.compute[:n])
            self.last_update = {**info, "push_seconds": time.perf_counter() - t0}
        self.barrier()
        return d

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None
        if self.broadcaster is not None and hasattr(self.broadcaster, "close"):
            self.broadcaster.close()
            self.broadcaster = None

    def _prune(self) -> None:
        steps = stable_steps(self.policy_dir)
        for s in steps[: -self.cfg.keep_last] if len(steps) > self.cfg.keep_last else []:
            shutil.rmtree(step_dir(self.policy_dir, s), ignore_errors=True)


class _FullStore:
    """Read-only flat-store stand-in over gathered full tensors."""

    def __init__(self, tensors: dict, offsets: dict):
        self._t = tensors
        self.offsets = offsets

    def view(self, name: str):
        return self._t[name]

    def names(self):
        return list(self._t)


class _GatheredModel:
    def __init__(self, model, tensors: dict):
        self.cfg = model.cfg
        self.flat = _FullStore(tensors, model.flat.offsets)
        self.quant = {}
        self.lora = None


def _gathered_view(model):
    """Collective: the full weights of a ZeRO-3 model as host tensors on
    data-parallel rank 0 (a stand-in model the exporters read), None elsewhere."""
    full = model.zero3.full_state(lambda n, t: t.detach().to("cpu", copy=True))
    return _GatheredModel(model, full) if full is not None else model


class DevicePolicyReceiver:
    """Generator side of the device transfer: the peer receive slots (created
    when the generator starts, so the trainer finds them) and, lazily, the
    NCCL broadcast group of the fallback."""

    def __init__(self, model, output_dir: Path, cfg, index: int = 0):
        from .peer_policy import PeerPolicyReceiver

        self.model = model
        self.cfg = cfg
        self.index = index
        self.peer = None
        if cfg.peer:
            self.peer = PeerPolicyReceiver(model, resolve_policy_dir(output_dir, cfg), index, cfg.peer_slots)
        self.group = None

    def load(self, snapshot_dir: Path, step: int) -> int:
        from .peer_policy import FLAT_PROTOCOL, PROTOCOL, PolicyBroadcastGroup, mark_ready, used_numel

        info = json.loads((Path(snapshot_dir) / "update_info.json").read_text())
        proto = info.get("protocol")
        if proto == PROTOCOL:
            if self.peer is None:
                raise RuntimeError("a peer policy update arrived but this generator has no receive slots")
            return self.peer.load(step, timeout_s=self.cfg.nccl_timeout_seconds)
        if proto == FLAT_PROTOCOL:
            flat = self.model.flat
            n = int(info["numel"])
            if n != used_numel(flat):
                raise ValueError(f"NCCL policy update of {n} elements for a generator layout of {used_numel(flat)}")
            if self.group is None:
                c = self.cfg
                self.group = PolicyBroadcastGroup(c.nccl_host, c.nccl_port, c.nccl_rank_offset + self.index,
                                                  1 + c.nccl_inference_world_size, flat.compute.device,
                                                  c.nccl_timeout_seconds,
                                                  backend="nccl" if flat.compute.is_cuda else "gloo")
            mark_ready(snapshot_dir, self.index)
            self.group.broadcast(flat.compute[:n])
            return step
        raise ValueError(f"unsupported device policy protocol {proto!r}")

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None
        if self.group is not None:
            self.group.close()
            self.group = None


def load_policy_into(model, snapshot_dir: Path, device_receiver: DevicePolicyReceiver | None = None,
                     step: int | None = None) -> dict[str, Any]:
    """Load a policy snapshot into a generator model (same arch): filesystem
    weights or adapter, or a device update through ``device_receiver``."""
    meta = json.loads((Path(snapshot_dir) / POLICY_META).read_text())
    if meta.get("kind") == "device":
        if device_receiver is None:
            raise RuntimeError(f"{snapshot_dir} is a device policy update; this generator has no device receiver "
                               "(policy_transfer.type: nccl needs one per generator process)")
        meta["loaded_step"] = device_receiver.load(Path(snapshot_dir), int(meta["step"] if step is None else step))
        return meta
    if meta.get("kind") == "model":
        from ..models.hf_io import load_hf_weights

        load_hf_weights(model, Path(snapshot_dir) / "model")
    elif meta.get("kind") == "adapter":
        from ..models.lora import merge_adapter_into

        merge_adapter_into(model, Path(snapshot_dir) / "adapter")
    return meta
