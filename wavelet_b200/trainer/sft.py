"""``wavelet sft``: supervised fine-tuning.

    python -m wavelet_b200 sft @ cfg.yaml [--section.key value ...]
    torchrun --nproc-per-node N -m wavelet_b200 sft @ cfg.yaml

Setup order: seed -> distributed -> model -> data -> optimizer -> run state
(monitor, checkpoints, resume).  Each optimizer step runs
``batch_size / (micro_batch_size * dp)`` micro-batches per rank, normalises
the loss by the global count of trainable tokens, clips, steps the sharded
optimizer and logs ``loss``, ``optim/grad_norm``, ``optim/lr`` and the
``perf/*`` metrics.

Parity: trainer/trainer.py:1162-1683 of the reference (SFTTrainer and main).
"""

from __future__ import annotations

import gc
import logging
import os
import sys
import time
from pathlib import Path
from typing import Any

import torch

from ..configs.config import SFTConfig
from ..models.config import resolve_arch
from ..models.qwen import build_model
from .gc_control import StepGarbageCollector
from .profiling import CudaMemoryProfiler, StepProfiler
from .telemetry import Telemetry, node_metrics, rank_rows
from ..monitor import RunMonitor, setup_logger
from ..parallel.dist import Groups, ParallelDims, destroy_distributed, init_distributed
from ..utils import pathing
from ..utils.config import config_to_plain, dump_yaml, load_config
from .ckpt import CheckpointManager
from .engine import Engine
from .optim import FlatOptimizer, lr_at
from .perf import PerfTracker

log = logging.getLogger("wavelet")


class SFTTrainer:
    def __init__(self, config: SFTConfig):
        self.config = config
        self.step = 0
        self.world = None
        self.model = None
        self.engine = None
        self.optimizer = None
        self.dataset = None
        self.monitor = None
        self.ckpt = None
        self.perf = None

    # ------------------------------------------------------------------ setup
    def setup(self) -> "SFTTrainer":
        c = self.config
        torch.manual_seed(c.seed)
        backend = c.fsdp.backend
        self.world = init_distributed(backend, timeout_s=c.dist_timeout_seconds)
        w = self.world
        dims = ParallelDims(dp_replicate=c.fsdp.dp_replicate, dp_shard=c.fsdp.dp_shard, cp=c.fsdp.cp, tp=c.fsdp.tp,
                            ep=c.fsdp.ep, world_size=w.world_size)
        self.groups = Groups(dims, w.rank)
        dp_rank, dp_world = self.groups.dp_rank, dims.dp
        # parameters are replicated over dp x cp: their shards and gradient
        # reductions use that group (data is split over dp only)
        self.cp = dims.cp
        opt_group, opt_rank, opt_world = self.groups.dp_cp, self.groups.dp_cp_rank, self.groups.dp_cp_size
        # hybrid sharding: sharded parameters and optimizer state over one
        # replica (dp_shard x cp), gradients all-reduced across dp_replicate
        hsdp = c.fsdp.shard_params and dims.dp_replicate > 1
        shard_group, shard_rank, shard_world = ((self.groups.shard, self.groups.shard_rank, self.groups.shard_size)
                                                if hsdp else (opt_group, opt_rank, opt_world))
        dev = w.device
        arch = resolve_arch(c.model.name, c.model.arch_overrides or None)
        dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        self.fabric = None
        self.norm_fabric = None
        shard = c.fsdp.shard_params
        if dev.type == "cuda" and dims.cp == 1 and dims.ep == 1 and c.fsdp.backend != "gloo" and not shard:
            from ..parallel.fabric import maybe_fabric

            # the fused optimizer step runs over the data-parallel group (inside
            # each tensor-parallel slice); under TP the gradient-norm exchange
            # spans every rank of the job
            self.fabric = maybe_fabric(dp_world, dp_rank, dev, group=self.groups.dp)
            if self.fabric is not None and dims.tp > 1:
                from ..parallel.fabric import Fabric

                self.norm_fabric = Fabric(w.rank, w.world_size, dev)
        self.ep_fabric = None
        if dev.type == "cuda" and dims.ep > 1 and c.fsdp.backend != "gloo":
            from ..parallel.fabric import Fabric

            self.ep_fabric = Fabric(self.groups.ep_rank, dims.ep, dev, group=self.groups.ep)
        self.model = build_model(arch, dev, dtype, dp_rank=shard_rank, dp_world=shard_world, seed=c.seed,
                                 fabric=self.fabric,
                                 ep_fabric=self.ep_fabric,
                                 init=c.model.random_init or not _has_weights(c.model.name), lora=c.lora,
                                 load_in_4bit=c.model.load_in_4bit, lora_seed=c.seed,
                                 ep=(dims.ep, self.groups.ep_rank, self.groups.ep_dp_rank, self.groups.ep_dp_size)
                                 if dims.ep > 1 else None,
                                 tp=(dims.tp, self.groups.tp_rank) if dims.tp > 1 else None,
                                 shard_params=shard)
        if shard:
            from ..parallel.zero3 import ParamGatherer

            ParamGatherer(self.model, group=shard_group if shard_world > 1 else None)
        self.model.tp_group = self.groups.tp
        self.tp_fabric = None
        if dims.tp > 1 and dev.type == "cuda" and c.fsdp.backend != "gloo" and c.fsdp.tp_reduce == "fabric":
            from ..parallel.fabric import Fabric

            self.tp_fabric = Fabric(self.groups.tp_rank, dims.tp, dev, group=self.groups.tp)
            self.model.attach_tp_fabric(self.tp_fabric)
        if self.groups.ep is not None:
            self.model.ep_group = self.groups.ep
            if self.ep_fabric is not None and c.fsdp.ep_dispatch == "fabric":
                self.model.attach_ep_fabric(self.ep_fabric, max_tokens=c.data.seq_len * c.data.micro_batch_size,
                                            capacity_factor=c.fsdp.ep_capacity_factor)
        from .model_options import apply_model_options

        apply_model_options(self.model, c.model, c.fsdp, c)
        ac = c.model.activation_checkpointing
        self.model.set_activation_checkpointing(ac.freq if ac is not None else None)
        if c.model.smart_gc:
            self.model.enable_activation_offload()
        if not c.model.random_init and _has_weights(c.model.name):
            from ..models.hf_io import load_hf_weights

            load_hf_weights(self.model, Path(c.model.name))
        self.optimizer = FlatOptimizer(self.model.trainable, c.optim, c.max_grad_norm, shard_group, shard_world,
                                       fabric=self.fabric, expert_flat=self.model.expert_flat,
                                       ep_dp_group=self.groups.ep_dp, ep_dp_world=self.groups.ep_dp_size,
                                       norm_fabric=self.norm_fabric,
                                       replicate_group=self.groups.replicate if hsdp else None)
        from .model_options import lm_head_chunk

        self.engine = Engine(self.model, self.optimizer.adamw.h, opt_group, opt_world, lm_head_chunk=lm_head_chunk(c.model))
        self.engine.opt = self.optimizer  # type: ignore[assignment]
        from ..data.sft import SFTDataset
        from ..data.tokenizer import tokenizer_for

        tok = None if c.data.source == "fake" else tokenizer_for(c.model)
        self.dataset = SFTDataset(c.data, tok, dp_rank, dp_world, seed=c.seed)
        self.val_dataset = SFTDataset(c.val.data, tok, dp_rank, dp_world, seed=c.seed) if c.val is not None else None
        gm = c.data.micro_batch_size * dp_world
        if c.data.batch_size % gm:
            raise ValueError(
                f"SFT data.batch_size is the global optimizer batch and must be divisible by "
                f"micro_batch_size * dp ({c.data.micro_batch_size} * {dp_world})"
            )
        self.accum = c.data.batch_size // gm
        self.total_steps = c.max_steps or max(1, c.epochs * len(self.dataset.samples()) // c.data.batch_size)
        out = Path(c.output_dir)
        resume = None
        if c.ckpt is not None:
            resume = pathing.resolve_resume_dir(c.checkpoint_output_dir, c.ckpt.resume_step, c.ckpt.resume_dir)
        # a SLURM job controller validated the output directory and created the
        # launch attempt before starting this role (WAVELET_SLURM_OUTPUT_PREPARED)
        if w.rank == 0 and os.environ.get("WAVELET_SLURM_OUTPUT_PREPARED") != "1":
            pathing.validate_output_dir(out, clean=c.clean_output_dir, resuming=resume is not None,
                                        protected_paths=(c.model.name, c.model.adapter_path))
            attempt = pathing.create_launch_attempt(out)
            dump_yaml(attempt.config_dir / "sft.yaml", config_to_plain(c))
        if w.distributed:
            torch.distributed.barrier()
        setup_logger("sft", out, c.log.level, c.log.json_console, c.log.json_file)
        from ..configs.inert import warn_inert

        warn_inert(c)  # settings of the reference's schema that do nothing here, named
        self.monitor = RunMonitor.from_config(out, c.monitor, checkpoint_dir=c.checkpoint_output_dir)
        self.ckpt = None
        if c.ckpt is not None and c.ckpt.mode != "disabled":
            self.ckpt = CheckpointManager(c.checkpoint_output_dir, mode=c.ckpt.mode, keep_last=c.ckpt.keep_last,
                                          keep_interval=c.ckpt.keep_interval, rank=w.rank, world=w.world_size)
        if resume is not None:
            mgr = self.ckpt or CheckpointManager(c.checkpoint_output_dir, mode="disabled", rank=w.rank, world=w.world_size)
            st = mgr.load(resume, model=self.model, optimizer=self.optimizer, skip_optimizer=c.ckpt.skip_optimizer)
            if not c.ckpt.skip_progress:
                self.step = int(st["meta"]["step"])
            if c.ckpt.skip_scheduler:  # the learning-rate schedule restarts at the resumed step
                self.sched_offset = self.step
            if st["data_state"] is not None and not c.ckpt.skip_dataloader:
                self.dataset.load_state_dict(st["data_state"])
        if getattr(c.data, "num_workers", 0) and c.data.num_workers > 0:  # batches built ahead on a thread
            from ..data.sft import PrefetchingDataset

            self.dataset = PrefetchingDataset(self.dataset, 2 * c.data.num_workers)
        self.monitor.start_run(run_config=config_to_plain(c), world=w, resumed_from=str(resume) if resume else None)
        lora_params = self.model.lora.num_trainable() if self.model.lora is not None else None
        self.perf = PerfTracker(arch, w.device, lora_rank=c.lora.rank if c.lora else None, lora_params=lora_params)
        self.telemetry = Telemetry(w, replication=max(1, dims.tp * dims.cp))
        self.gc = StepGarbageCollector(c.gc.interval) if c.gc is not None else None
        self.profiler = None
        if c.profiler is not None:
            path = c.profiler.trace_path or out / "traces" / f"rank{w.rank}.json"
            self.profiler = StepProfiler(path, start_step=c.profiler.start_step, end_step=c.profiler.end_step,
                                         record_shapes=c.profiler.record_shapes,
                                         profile_memory=c.profiler.profile_memory)
        self.mem_profiler = None
        if c.memory_profiler is not None and dev.type == "cuda":
            self.mem_profiler = CudaMemoryProfiler(c.memory_profiler.output_dir or out / "memory", rank=w.rank,
                                                   interval=c.memory_profiler.interval,
                                                   max_entries=c.memory_profiler.max_entries)
        return self

    # ------------------------------------------------------------ validation
    def _shard(self, b):
        """This rank's context-parallel share of a host micro-batch."""
        if self.cp == 1:
            return b
        from ..parallel.context_parallel import shard_batch

        align = 128 if self.world.device.type == "cuda" else 8
        return shard_batch(b, self.cp, self.groups.cp_rank, self.groups.cp, align=align)

    def validate(self) -> dict[str, float]:
        """Token-mean masked CE over one pass of the validation set (all ranks)."""
        dev = self.world.device
        tot = torch.zeros(2, dtype=torch.float64, device=dev)
        for b in self.val_dataset.eval_batches():
            loss, n = self.engine.sft_eval(self._shard(b).to(dev))
            tot[0] += loss.double()
            tot[1] += n
        if self.world.distributed:
            torch.distributed.all_reduce(tot, group=self.groups.dp_cp)
        loss_v, n_v = tot.tolist()
        return {"val/loss": loss_v / max(n_v, 1.0), "val/tokens": n_v}

    # ------------------------------------------------------------------ loop
    def train_step(self) -> dict[str, Any]:
        c = self.config
        t0 = time.perf_counter()
        batches = [self._shard(self.dataset.next_micro_batch()) for _ in range(self.accum)]
        local = float(sum(float(b.loss_mask.sum()) for b in batches))
        total = self.engine.global_token_count(local, self.world.device)
        scale = 1.0 / max(total, 1.0)
        dev = self.world.device
        loss = torch.zeros((), device=dev)
        tokens = 0
        for b in batches:
            if c.data.pin_memory and dev.type == "cuda":
                b = b.pin_memory()
            b = b.to(dev)
            tokens += b.num_tokens
            loss += self.engine.sft_micro_step(b, scale)
        lr = lr_at(self.step - getattr(self, "sched_offset", 0), c.optim.lr, self.total_steps, c.scheduler)
        self.model.finalize_grads()
        stats = self.optimizer.step(lr)
        if self.world.distributed:
            torch.distributed.all_reduce(loss, group=self.groups.dp_cp)
        loss_v = float(loss.item())
        if not (loss_v == loss_v) or loss_v in (float("inf"), float("-inf")):
            raise FloatingPointError(f"non-finite SFT loss at step {self.step}")
        self.step += 1
        dt = time.perf_counter() - t0
        m = {"loss": loss_v, "optim/grad_norm": stats["grad_norm"], "optim/lr": lr, "train/loss_tokens": total}
        m.update(self.perf.step_metrics(tokens * (self.world.world_size // max(1, self.config.fsdp.tp * self.cp)), dt))
        m["_tokens"], m["_seconds"] = float(tokens), dt
        return m

    def train(self) -> int:
        c = self.config
        status = "failed"
        try:
            if self.val_dataset is not None and c.val.eval_on_start:
                self.monitor.log(self.validate(), self.step)
            while self.step < self.total_steps:
                if self.profiler is not None:
                    self.profiler.before_step(self.step + 1)
                metrics = self.train_step()
                ranks = self.telemetry.sample(metrics.pop("_tokens"), metrics.pop("_seconds"))
                metrics.update(node_metrics(ranks))
                if self.profiler is not None:
                    self.profiler.after_step(self.step)
                if self.mem_profiler is not None:
                    self.mem_profiler.step(self.step)
                if self.val_dataset is not None and self.step % c.val.interval == 0:
                    metrics.update(self.validate())
                if self.step % c.log.log_every == 0:
                    self.monitor.log(metrics, self.step, ranks=rank_rows(ranks))
                    log.info("step %d loss %.4f grad_norm %.3f tok/s %.0f", self.step, metrics["loss"],
                             metrics["optim/grad_norm"], metrics.get("perf/tokens_per_second", 0))
                if self.ckpt is not None and c.ckpt.interval and self.step % c.ckpt.interval == 0:
                    self.save_checkpoint()
                if self.gc is not None:
                    self.gc.run(self.step)
            if self.ckpt is not None:
                self.save_checkpoint(block=True)
            status = "completed"
            return 0
        finally:
            if self.ckpt is not None:
                try:
                    self.ckpt.wait()
                except Exception:
                    status = "failed"
            self.monitor.finish(status=status, step=self.step)
            for closer in (self.profiler, self.mem_profiler, self.gc):
                if closer is not None:
                    closer.close()

    def save_checkpoint(self, block: bool = False) -> None:
        c = self.config
        self.ckpt.save(
            self.step, model=self.model, optimizer=self.optimizer, data_state=self.dataset.state_dict(),
            meta={"arch": self.model.cfg.to_dict(), "numel": self.model.flat.numel, **_lora_meta(self.config, self.model)},
            scheduler_state={"step": self.step}, block=block,
        )
        self.monitor.log_event("checkpoint_saved", step=self.step)


def _has_weights(name: str) -> bool:
    p = Path(name)
    return p.is_dir() and any(p.glob("*.safetensors"))


def _lora_meta(cfg, model) -> dict:
    if model.lora is None:
        return {"model_name": cfg.model.name}
    return {"model_name": cfg.model.name, "lora_rank": model.lora.rank, "lora_alpha": model.lora.alpha,
            "lora_target_modules": model.lora.target_modules}


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config(SFTConfig, argv)
    if cfg.dry_run:
        print(cfg.model_dump_json(indent=2))
        return 0
    if cfg.slurm is not None:
        from ..deployment.slurm import launch_slurm

        return launch_slurm(cfg, "sft", argv)
    trainer = SFTTrainer(cfg).setup()
    try:
        return trainer.train()
    finally:
        for fab in (trainer.fabric, trainer.norm_fabric, trainer.ep_fabric, trainer.tp_fabric):
            if fab is not None:
                fab.close()
        destroy_distributed()


if __name__ == "__main__":
    sys.exit(main())
