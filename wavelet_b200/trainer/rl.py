"""``wavelet rl-trainer``: the RL trainer role.

Per optimizer step: wait for the rollout batch of this step in the
filesystem queue, claim it, pack its records into per-rank micro-batches,
compute trainer log-probs with the chunked LM head at the sampling
temperature, evaluate the configured RL loss (+ CE / reference-KL
components) with global normalisation, step the sharded optimizer, mark the
batch consumed and export the new policy.

Parity: trainer/rl.py of the reference (RLTrainer._train_step :742,
component scales :641-740, logprob computation :1050-1125, main loop
:1398-1488).
"""

from __future__ import annotations

import logging
import sys
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from ..configs.config import RLConfig
from ..data.rl import RLExample, example_from_payload, make_rank_batches
from ..models.config import resolve_arch
from ..models.qwen import build_model
from ..monitor import RunMonitor, emit_perf, setup_logger
from ..ops import lm_head
from ..parallel.dist import Groups, ParallelDims, destroy_distributed, init_distributed
from ..transport.policy import PolicyExporter
from ..transport.queue import FileSystemRolloutReceiver, read_training_records
from ..utils import pathing
from ..utils.config import config_to_plain, dump_yaml, load_config
from .ckpt import CheckpointManager
from .losses import compute_loss, segment_ids, seg_sum, setup_rl_loss_fn
from .optim import FlatOptimizer, lr_at
from .perf import PerfTracker

log = logging.getLogger("wavelet")


class RLTrainer:
    def __init__(self, config: RLConfig):
        self.config = config
        self.step = 0

    def setup(self, world=None, model=None) -> "RLTrainer":
        c = self.config
        torch.manual_seed(c.seed)
        self.world = world or init_distributed(c.fsdp.backend, timeout_s=c.dist_timeout_seconds)
        w = self.world
        dims = ParallelDims(dp_replicate=c.fsdp.dp_replicate, dp_shard=c.fsdp.dp_shard, cp=c.fsdp.cp, tp=c.fsdp.tp,
                            ep=c.fsdp.ep, world_size=w.world_size)
        if dims.cp > 1:
            # rollout batches are packed varlen sequences with per-sequence
            # normalisations; context parallelism shards SFT micro-batches
            raise NotImplementedError("fsdp.cp > 1 is supported by the SFT trainer; RL trains with cp = 1")
        self.groups = Groups(dims, w.rank)
        self.dp_rank, self.dp_world = self.groups.dp_rank, dims.dp
        arch = resolve_arch(c.model.name, c.model.arch_overrides or None)
        dtype = torch.bfloat16 if w.device.type == "cuda" else torch.float32
        if model is None:
            self.ep_fabric = None
            if dims.ep > 1 and w.device.type == "cuda" and c.fsdp.backend != "gloo":
                from ..parallel.fabric import Fabric

                self.ep_fabric = Fabric(self.groups.ep_rank, dims.ep, w.device, group=self.groups.ep)
            model = build_model(arch, w.device, dtype, dp_rank=self.dp_rank, dp_world=self.dp_world, seed=c.seed,
                                ep_fabric=self.ep_fabric,
                                lora=c.lora, load_in_4bit=c.model.load_in_4bit, lora_seed=c.seed,
                                ep=(dims.ep, self.groups.ep_rank, self.groups.ep_dp_rank, self.groups.ep_dp_size)
                                if dims.ep > 1 else None,
                                tp=(dims.tp, self.groups.tp_rank) if dims.tp > 1 else None)
            model.tp_group = self.groups.tp
            self.tp_fabric = None
            if dims.tp > 1 and w.device.type == "cuda" and c.fsdp.backend != "gloo" and c.fsdp.tp_reduce == "fabric":
                from ..parallel.fabric import Fabric

                self.tp_fabric = Fabric(self.groups.tp_rank, dims.tp, w.device, group=self.groups.tp)
                model.attach_tp_fabric(self.tp_fabric)
            p = Path(c.model.name)
            if not c.model.random_init and p.is_dir() and any(p.glob("*.safetensors")):
                from ..models.hf_io import load_hf_weights

                load_hf_weights(model, p)
        self.model = model
        from .model_options import apply_model_options

        apply_model_options(model, c.model, c.fsdp)
        ac = c.model.activation_checkpointing
        model.set_activation_checkpointing(ac.freq if ac is not None else None)
        if c.model.smart_gc:
            model.enable_activation_offload()
        if self.groups.ep is not None:
            model.ep_group = self.groups.ep
            if getattr(self, "ep_fabric", None) is not None and c.fsdp.ep_dispatch == "fabric":
                model.attach_ep_fabric(self.ep_fabric, max_tokens=c.data.seq_len,
                                       capacity_factor=c.fsdp.ep_capacity_factor)
        self.optimizer = FlatOptimizer(model.trainable, c.optim, c.max_grad_norm, self.groups.dp, self.dp_world,
                                       expert_flat=model.expert_flat, ep_dp_group=self.groups.ep_dp,
                                       ep_dp_world=self.groups.ep_dp_size)
        self.loss_fn = setup_rl_loss_fn(c.loss)
        out = Path(c.output_dir)
        self.output_dir = out
        setup_logger("rl-trainer", out, c.log.level, c.log.json_console, c.log.json_file)
        self.monitor = RunMonitor.from_config(out, c.monitor, checkpoint_dir=c.checkpoint_output_dir)
        self.ckpt = None
        if c.ckpt is not None and c.ckpt.mode != "disabled":
            self.ckpt = CheckpointManager(c.checkpoint_output_dir, mode=c.ckpt.mode, keep_last=c.ckpt.keep_last,
                                          keep_interval=c.ckpt.keep_interval, rank=w.rank, world=w.world_size)
        resume = None
        if c.ckpt is not None:
            resume = pathing.resolve_resume_dir(c.checkpoint_output_dir, c.ckpt.resume_step, c.ckpt.resume_dir)
        if resume is not None:
            mgr = self.ckpt or CheckpointManager(c.checkpoint_output_dir, mode="disabled", rank=w.rank, world=w.world_size)
            st = mgr.load(resume, model=model, optimizer=self.optimizer, skip_optimizer=c.ckpt.skip_optimizer)
            if not c.ckpt.skip_progress:
                self.step = int(st["meta"]["step"])
        self.receiver = FileSystemRolloutReceiver(out, c.transport, start_step=self.step)
        self.exporter = PolicyExporter(out, c.policy_transfer, rank=w.rank)
        self.perf = PerfTracker(arch, w.device)
        self.monitor.start_run(run_config=config_to_plain(c), world=w, resumed_from=str(resume) if resume else None)
        return self

    # ----------------------------------------------------------------- step
    def train_on_examples(self, examples: list[RLExample]) -> dict[str, Any]:
        c = self.config
        m = self.model
        dev = self.world.device
        t0 = time.perf_counter()
        temp = c.inference.sampling.temperature or c.inference.default_temperature
        batches = make_rank_batches(examples, c.data.seq_len, self.dp_rank, self.dp_world, temp)
        # global normalisers (trainer/rl.py:641-740): RL units by loss.normalization, CE / ref-KL tokens
        local = torch.zeros(3, dtype=torch.float64)
        for b in batches:
            cu = b.base.cu_seqlens
            seg = segment_ids(cu, b.base.num_tokens)
            mask = b.loss_mask
            rlm = mask if b.advantages is None else mask
            if c.loss.normalization == "sequence":
                local[0] += float((seg_sum(rlm.float(), seg, cu.numel() - 1) > 0).sum())
            else:
                local[0] += float(rlm.sum())
            if b.ce_weights is not None:
                local[1] += float((mask & (b.ce_weights != 0)).sum())
            if b.ref_kl_weights is not None:
                local[2] += float((mask & (b.ref_kl_weights != 0)).sum())
        if self.dp_world > 1:
            t = local.to(dev)
            dist.all_reduce(t, group=self.groups.dp)
            local = t.cpu()
        scales = {"rl": float(local[0]), "ce": float(local[1]), "ref_kl": float(local[2])}
        agg: dict[str, list[float]] = {}
        tokens = 0
        loss_total = 0.0
        for b in batches:
            b = b.to(dev)
            tokens += b.base.num_tokens
            ctx = m.batch_ctx(b.base.position_ids, b.base.cu_seqlens, b.base.max_seqlen)
            h = m.hidden(b.base.input_ids, ctx)
            tgt = b.base.targets.clamp_min(0)
            lp, ent = self._logprobs(h, tgt, b)
            loss, met = compute_loss(lp, b.inference_logprobs, b.teacher_logprobs, b.advantages, b.loss_mask, c.loss,
                                     cu_seqlens=b.base.cu_seqlens, ce_weights=b.ce_weights,
                                     ref_kl_weights=b.ref_kl_weights, component_scales=scales,
                                     rl_loss_fn=self.loss_fn)
            loss.backward()
            if not h.is_cuda:
                m.collect_cpu_grads()
            loss_total += float(loss.detach())
            with torch.no_grad():
                mk = b.loss_mask
                if bool(mk.any()):
                    agg.setdefault("entropy", []).append(float(ent[mk].mean()))
                    agg.setdefault("trainer_logprob", []).append(float(lp.detach()[mk].mean()))
            for k, v in met.items():
                agg.setdefault(k, []).append(v)
        lr = lr_at(self.step, c.optim.lr, max(1, c.max_steps or 1), c.scheduler)
        m.finalize_grads()
        st = self.optimizer.step(lr)
        self.step += 1
        metrics = {k: sum(v) / len(v) for k, v in agg.items() if v}
        lt = torch.tensor([loss_total], device=dev)
        if self.dp_world > 1:
            dist.all_reduce(lt, group=self.groups.dp)
        metrics.update({"loss": float(lt), "optim/grad_norm": st["grad_norm"], "optim/lr": lr,
                        "train/rl_units": scales["rl"], "train/num_samples": float(len(examples)),
                        "train/tokens": float(tokens)})
        dt = time.perf_counter() - t0
        metrics.update(self.perf.step_metrics(tokens * self.dp_world, dt, c.data.seq_len))
        emit_perf("trainer_step", step=self.step, seconds=dt, tokens=tokens)
        return metrics

    def _logprobs(self, h, tgt, b):
        m = self.model
        if b.sampling_mask is not None and any(b.sampling_mask):
            return self._support_logprobs(h, tgt, b)
        if h.is_cuda:
            return lm_head.logprob_entropy(h, m.head_weight(), tgt, b.temperature, gW=m.head_grad(), anchor=m.anchor)
        z = m.logits(h)
        return lm_head.ref.logprob_entropy(z, tgt, b.temperature)

    def _support_logprobs(self, h, tgt, b):
        """Log-prob renormalised over each token's sampling support set
        (trainer/losses.py:30-69): lp = z_t/T - logsumexp_{j in S}(z_j/T)."""
        m = self.model
        if h.is_cuda:
            lp_full, ent = lm_head.logprob_entropy(h, m.head_weight(), tgt, b.temperature, gW=m.head_grad(), anchor=m.anchor)
        else:
            z = m.logits(h)
            lp_full, ent = lm_head.ref.logprob_entropy(z, tgt, b.temperature)
        rows = [i for i, s in enumerate(b.sampling_mask) if s]
        if not rows:
            return lp_full, ent
        K = max(len(b.sampling_mask[i]) for i in rows)
        ids = torch.full((len(rows), K), -1, dtype=torch.long)
        for r, i in enumerate(rows):
            ids[r, : len(b.sampling_mask[i])] = torch.tensor(b.sampling_mask[i])
        ids = ids.to(h.device)
        ridx = torch.tensor(rows, device=h.device)
        valid = ids >= 0
        W = m.head_weight()
        from ..ops.support_head import SupportLogZ

        logz_s = SupportLogZ.apply(h, ridx, ids.clamp_min(0), valid, W, m.head_grad(), b.temperature, m.anchor)
        zt = SupportLogZ.target_logit(h, ridx, tgt, W, m.head_grad(), b.temperature, m.anchor)
        lp = lp_full.clone()
        lp = lp.index_put((ridx,), zt - logz_s)
        return lp, ent

    # ----------------------------------------------------------------- loop
    def run(self) -> int:
        c = self.config
        total = c.max_steps
        status = "failed"
        try:
            if c.policy_transfer.export_initial and self.step == 0:
                self.exporter.export(self.model, 0)
            while total is None or self.step < total:
                batch = self.receiver.wait()
                before = self.step
                if self.world.rank == 0:
                    self.receiver.claim(batch, before)
                records = [example_from_payload(r) for r in read_training_records(batch.training_path)]
                metrics = self.train_on_examples(records)
                if self.world.rank == 0:
                    self.receiver.consumed(batch, before, self.step)
                self.monitor.log(metrics, self.step)
                log.info("rl step %d loss %.4f grad_norm %.3f", self.step, metrics["loss"], metrics["optim/grad_norm"])
                if self.step % c.policy_transfer.export_every_steps == 0:
                    self.exporter.export(self.model, self.step)
                if self.ckpt is not None and c.ckpt.interval and self.step % c.ckpt.interval == 0:
                    self.ckpt.save(self.step, model=self.model, optimizer=self.optimizer, data_state=None,
                                   meta={"arch": self.model.cfg.to_dict(), **_lora_meta(self.config, self.model)}, scheduler_state={"step": self.step})
            status = "completed"
            return 0
        finally:
            if self.ckpt is not None:
                self.ckpt.wait()
            self.monitor.finish(status=status, step=self.step)


def _lora_meta(cfg, model) -> dict:
    if model.lora is None:
        return {"model_name": cfg.model.name}
    return {"model_name": cfg.model.name, "lora_rank": model.lora.rank, "lora_alpha": model.lora.alpha,
            "lora_target_modules": model.lora.target_modules}


def _close_fabric(t) -> None:
    for name in ("ep_fabric", "tp_fabric"):
        fab = getattr(t, name, None)
        if fab is not None:
            fab.close()
            setattr(t, name, None)


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config(RLConfig, argv)
    if cfg.dry_run:
        print(cfg.model_dump_json(indent=2))
        return 0
    t = RLTrainer(cfg).setup()
    try:
        return t.run()
    finally:
        _close_fabric(t)
        destroy_distributed()


if __name__ == "__main__":
    sys.exit(main())
