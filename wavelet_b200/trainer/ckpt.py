"""Checkpoints: asynchronous, sharded, resumable.

Layout of ``<output_dir>/checkpoint-<step>/`` (``STABLE`` is written last, after
every rank finished, so a crash never leaves a checkpoint that looks valid):

    meta.json                       step, world size, model arch, flat layout hash
    trainer/model.safetensors       full bf16 compute weights (rank 0)
    trainer/experts-ep<e>.safetensors  expert store of expert-parallel rank e (MoE)
    trainer/extra.safetensors       model buffers outside the flat stores (routing tables)
    trainer/optim-rank<r>.pt        fp32 master / exp_avg / exp_avg_sq shard of rank r
    trainer/scheduler.json          optimizer step counter and LR state
    dataloader/rank<r>.json         data cursor of rank r
    STABLE

Saving copies device state into (optionally pinned) host buffers on the
caller's stream, then writes files on a background thread so the next
training step overlaps the I/O (``ckpt.mode: async`` /
``async_with_pinned_mem``).  A gloo group coordinates ranks so the NCCL
stream is never blocked by file I/O.  Resuming on a different world size
re-shards the optimizer state from the saved shards (the flat layout is
identical for every world size up to padding).

Parity: trainer/ckpt.py:55-436 of the reference (DCP async_save on a gloo
group, STABLE markers, keep_last / keep_interval, skip flags).
"""

from __future__ import annotations

import json
import shutil
import threading
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from ..utils import pathing


def _save_safetensors(tensors: dict[str, torch.Tensor], path: Path) -> None:
    from safetensors.torch import save_file

    save_file({k: v.contiguous() for k, v in tensors.items()}, str(path))


class CheckpointManager:
    def __init__(self, output_dir: Path, *, mode: str = "async", keep_last: int = 2, keep_interval: int | None = None,
                 rank: int = 0, world: int = 1):
        self.output_dir = Path(output_dir)
        self.mode = mode
        self.keep_last = keep_last
        self.keep_interval = keep_interval
        self.rank = rank
        self.world = world
        self._thread: threading.Thread | None = None
        self._error: BaseException | None = None
        self._gloo = None
        if world > 1 and dist.is_initialized():
            self._gloo = dist.new_group(backend="gloo")
        self._pinned: dict[str, torch.Tensor] = {}

    # ---------------------------------------------------------------- save
    def _host(self, name: str, t: torch.Tensor) -> torch.Tensor:
        if t.device.type == "cpu":
            return t.detach().clone()
        if self.mode == "async_with_pinned_mem":
            buf = self._pinned.get(name)
            if buf is None or buf.shape != t.shape or buf.dtype != t.dtype:
                buf = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                self._pinned[name] = buf
            buf.copy_(t.detach(), non_blocking=True)
            return buf
        return t.detach().to("cpu")

    def save(self, step: int, *, model, optimizer, data_state: dict | None, meta: dict[str, Any],
             scheduler_state: dict | None = None, block: bool = False) -> Path:
        self.wait()
        d = pathing.checkpoint_dir(self.output_dir, step)
        flat = getattr(model, "trainable", model.flat)  # LoRA: only the adapters are saved
        weights = None
        tp_size = getattr(model, "tp_size", 1)
        wname = "model.safetensors" if tp_size == 1 else f"model-tp{model.tp_rank}.safetensors"
        if getattr(flat, "sharded_compute", False):  # ZeRO-3: gathered unit by unit (every rank takes part)
            weights = flat.gatherer.full_state(lambda n, t: self._host("w:" + n, t))
            if self.rank != 0:  # hybrid sharding: every replica gathers its own copy; global rank 0 writes
                weights = None
        elif (self.rank == 0) if tp_size == 1 else (flat.dp_rank == 0):  # one copy of every TP shard
            weights = {n: self._host("w:" + n, flat.view(n)) for n in flat.names()}
        experts = None
        ef = getattr(model, "expert_flat", None)
        if ef is not None and getattr(model, "ep_dp_rank", 0) == 0:  # one copy per expert shard
            experts = {n: self._host("e:" + n, ef.view(n)) for n in ef.names()}
        ep_rank = getattr(model, "ep_rank", 0)
        extra = None  # model state outside the flat stores (e.g. routing tables)
        if self.rank == 0 and hasattr(model, "extra_state"):
            extra = {n: self._host("x:" + n, t) for n, t in model.extra_state().items()}
        opt = {k: (self._host("o:" + k, v) if torch.is_tensor(v) else v) for k, v in optimizer.state_dict().items()}
        if torch.cuda.is_available():
            torch.cuda.synchronize()

        def work():
            try:
                (d / "trainer").mkdir(parents=True, exist_ok=True)
                (d / "dataloader").mkdir(parents=True, exist_ok=True)
                if weights is not None:
                    _save_safetensors(weights, d / "trainer" / wname)
                if self.rank == 0:
                    (d / "meta.json").write_text(json.dumps({"step": step, "world_size": self.world,
                                                             "tp": tp_size, **meta}, indent=2))
                    (d / "trainer" / "scheduler.json").write_text(json.dumps(scheduler_state or {}, indent=2))
                if experts is not None:
                    _save_safetensors(experts, d / "trainer" / f"experts-ep{ep_rank}.safetensors")
                if extra:
                    _save_safetensors(extra, d / "trainer" / "extra.safetensors")
                torch.save({**opt, "shard_rank": self.rank, "shard_world": self.world}, d / "trainer" / f"optim-rank{self.rank}.pt")
                if data_state is not None:
                    (d / "dataloader" / f"rank{self.rank}.json").write_text(json.dumps(data_state))
            except BaseException as e:  # surfaced by wait()
                self._error = e

        if self.mode == "disabled" or block:
            work()
            self._finalize(d, step)
        else:
            self._thread = threading.Thread(target=lambda: (work(), self._finalize(d, step)), daemon=True)
            self._thread.start()
        return d

    def _finalize(self, d: Path, step: int) -> None:
        ok = torch.tensor([0 if self._error is None else 1])
        if self._gloo is not None:
            dist.all_reduce(ok, group=self._gloo)
        if int(ok.item()) == 0 and self.rank == 0:
            (d / pathing.STABLE).write_text(str(step))
            self._cleanup()

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            e, self._error = self._error, None
            raise RuntimeError(f"checkpoint save failed: {e}") from e

    def _cleanup(self) -> None:
        steps = pathing.list_checkpoint_steps(self.output_dir)
        keep = set(steps[-self.keep_last:])
        if self.keep_interval:
            keep |= {s for s in steps if s % self.keep_interval == 0}
        for s in steps:
            if s not in keep:
                shutil.rmtree(pathing.checkpoint_dir(self.output_dir, s), ignore_errors=True)

    # ---------------------------------------------------------------- load
    def load(self, d: Path, *, model, optimizer=None, skip_optimizer=False) -> dict[str, Any]:
        from safetensors.torch import load_file

        meta = json.loads((d / "meta.json").read_text())
        tp_size = getattr(model, "tp_size", 1)
        if int(meta.get("tp", 1)) != tp_size:
            raise ValueError(f"checkpoint was written with tp={meta.get('tp', 1)}, resuming with tp={tp_size}")
        w = load_file(str(d / "trainer" / ("model.safetensors" if tp_size == 1 else
                                           f"model-tp{model.tp_rank}.safetensors")))
        flat = getattr(model, "trainable", model.flat)
        flat.load_state({k: v.to(flat.device) for k, v in w.items()})
        ef = getattr(model, "expert_flat", None)
        if ef is not None:
            we = load_file(str(d / "trainer" / f"experts-ep{model.ep_rank}.safetensors"))
            ef.load_state({k: v.to(ef.device) for k, v in we.items()})
        if hasattr(model, "load_extra_state") and (d / "trainer" / "extra.safetensors").exists():
            model.load_extra_state(load_file(str(d / "trainer" / "extra.safetensors")))
        if optimizer is not None and not skip_optimizer:
            saved_world = int(meta.get("world_size", 1))
            if saved_world == self.world:
                sd = torch.load(d / "trainer" / f"optim-rank{self.rank}.pt", map_location=flat.device, weights_only=False)
            else:
                # re-shard: concatenate every saved shard then take ours
                parts = [torch.load(d / "trainer" / f"optim-rank{r}.pt", map_location="cpu", weights_only=False) for r in range(saved_world)]
                sd = {"step": parts[0]["step"]}
                if "m8" in parts[0]:  # 8-bit moments: block scales do not survive re-sharding; go through fp32
                    from ..ops import q8_dequant_moments

                    for q in parts:
                        q["exp_avg"], q["exp_avg_sq"] = q8_dequant_moments(q["m8"], q["v8"], q["m8_scale"],
                                                                           q["v8_scale"])
                for k in ("master", "exp_avg", "exp_avg_sq"):
                    full = torch.cat([p[k] for p in parts])
                    full = torch.nn.functional.pad(full, (0, max(0, flat.numel - full.numel())))[: flat.numel]
                    sd[k] = full[flat.global_shard_slice].to(flat.device)
                if "momentum" in parts[0]:
                    full = torch.cat([p["momentum"] for p in parts])
                    full = torch.nn.functional.pad(full, (0, max(0, flat.numel - full.numel())))[: flat.numel]
                    sd["momentum"] = full[flat.global_shard_slice].to(flat.device)
            optimizer.load_state_dict(sd)
        data_state = None
        p = d / "dataloader" / f"rank{self.rank}.json"
        if p.exists():
            data_state = json.loads(p.read_text())
        sched = {}
        sp = d / "trainer" / "scheduler.json"
        if sp.exists():
            sched = json.loads(sp.read_text())
        return {"meta": meta, "data_state": data_state, "scheduler": sched}
