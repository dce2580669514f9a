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
        self.groups = Groups(dims, w.rank)
        self.dp_rank, self.dp_world = self.groups.dp_rank, dims.dp
        # context parallelism: the micro-batches of a data-parallel rank are
        # split along the tokens over its cp ranks; parameters, gradients and
        # optimizer shards live on the dp x cp ranks (reference trainer/rl.py:682-740)
        self.cp = dims.cp
        opt_group, opt_rank, opt_world = self.groups.dp_cp, self.groups.dp_cp_rank, self.groups.dp_cp_size
        arch = resolve_arch(c.model.name, c.model.arch_overrides or None)
        dtype = torch.bfloat16 if w.device.type == "cuda" else torch.float32
        if model is None:
            self.ep_fabric = None
            if dims.ep > 1 and w.device.type == "cuda" and c.fsdp.backend != "gloo":
                from ..parallel.fabric import Fabric

                self.ep_fabric = Fabric(self.groups.ep_rank, dims.ep, w.device, group=self.groups.ep)
            model = build_model(arch, w.device, dtype, dp_rank=opt_rank, dp_world=opt_world, seed=c.seed,
                                ep_fabric=self.ep_fabric,
                                lora=c.lora, load_in_4bit=c.model.load_in_4bit, lora_seed=c.seed,
                                ep=(dims.ep, self.groups.ep_rank, self.groups.ep_dp_rank, self.groups.ep_dp_size)
                                if dims.ep > 1 else None,
                                tp=(dims.tp, self.groups.tp_rank) if dims.tp > 1 else None,
                                shard_params=c.fsdp.shard_params)
            if c.fsdp.shard_params:
                from ..parallel.zero3 import ParamGatherer

                ParamGatherer(model, group=opt_group if opt_world > 1 else None)
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
        from .model_options import apply_model_options, lm_head_chunk

        self.lm_head_chunk = lm_head_chunk(c.model)

        apply_model_options(model, c.model, c.fsdp, c)
        ac = c.model.activation_checkpointing
        model.set_activation_checkpointing(ac.freq if ac is not None else None)
        if c.model.smart_gc:
            model.enable_activation_offload()
        if self.groups.ep is not None:
            model.ep_group = self.groups.ep
            if getattr(self, "ep_fabric", None) is not None and c.fsdp.ep_dispatch == "fabric":
                model.attach_ep_fabric(self.ep_fabric, max_tokens=c.data.seq_len,
                                       capacity_factor=c.fsdp.ep_capacity_factor)
        self.optimizer = FlatOptimizer(model.trainable, c.optim, c.max_grad_norm, opt_group, opt_world,
                                       expert_flat=model.expert_flat, ep_dp_group=self.groups.ep_dp,
                                       ep_dp_world=self.groups.ep_dp_size)
        self.loss_fn = setup_rl_loss_fn(c.loss)
        out = Path(c.output_dir)
        self.output_dir = out
        setup_logger("rl-trainer", out, c.log.level, c.log.json_console, c.log.json_file)
        from ..configs.inert import warn_inert

        warn_inert(c)  # settings of the reference's schema that do nothing here, named
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
            if c.ckpt.skip_scheduler:  # the learning-rate schedule restarts at the resumed step
                self.sched_offset = self.step
        from ..orchestrator.schedule import chunks_per_step

        # with streamed chunks, queue step q holds chunk q % C of optimizer step q // C
        self.receiver = FileSystemRolloutReceiver(out, c.transport, start_step=self.step * chunks_per_step(c))
        self.exporter = PolicyExporter(out, c.policy_transfer, rank=w.rank, world=w.world_size,
                                       barrier=dist.barrier if w.world_size > 1 and dist.is_initialized() else None)
        self.perf = PerfTracker(arch, w.device)
        self.monitor.start_run(run_config=config_to_plain(c), world=w, resumed_from=str(resume) if resume else None)
        return self

    # ----------------------------------------------------------------- step
    def _local_batches(self, examples: list[RLExample]) -> list:
        c = self.config
        temp = c.inference.sampling.temperature or c.inference.default_temperature
        return make_rank_batches(examples, c.data.seq_len, self.dp_rank, self.dp_world, temp)

    def _unit_counts(self, batches) -> torch.Tensor:
        """This rank's (RL units by loss.normalization, CE tokens, ref-KL
        tokens) of its micro-batches, counted on the host (trainer/rl.py:641-740)."""
        c = self.config
        local = torch.zeros(3, dtype=torch.float64)
        for b in batches:
            cu = b.base.cu_seqlens
            mask = b.loss_mask
            if c.loss.normalization == "sequence":
                seg = segment_ids(cu, b.base.num_tokens)
                local[0] += float((seg_sum(mask.float(), seg, cu.numel() - 1) > 0).sum())
            else:
                local[0] += float(mask.sum())
            if b.ce_weights is not None:
                local[1] += float((mask & (b.ce_weights != 0)).sum())
            if b.ref_kl_weights is not None:
                local[2] += float((mask & (b.ref_kl_weights != 0)).sum())
        return local

    def _reduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sum over the ranks that hold different data (dp; dp x cp for the
        counts of a context-parallel run are taken before sharding, so dp)."""
        if self.dp_world > 1 and dist.is_initialized():
            t = t.to(self.world.device)
            dist.all_reduce(t, group=self.groups.dp)
            t = t.cpu()
        return t

    def _need_inference_recompute(self, batches) -> bool:
        """Whether any rank has RL / ref-KL tokens without inference log-probs
        (one collective: every rank must run the same extra forwards, which
        hold collectives under tensor / expert / context parallelism)."""
        local = any(bool(b.missing_inference().any()) for b in batches)
        if dist.is_initialized() and dist.get_world_size() > 1:
            t = torch.tensor([1.0 if local else 0.0], device=self.world.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return bool(t.item() > 0)
        return local

    def _shard_for_cp(self, hb):
        """(this rank's share of host micro-batch ``hb``, (sequence id per local
        token, sequences, RL tokens per sequence over all cp ranks)) under
        context parallelism; (hb, None) without it."""
        if self.cp == 1:
            return hb, None
        from dataclasses import replace

        from ..parallel.context_parallel import shard_batch, shard_index

        align = 128 if self.world.device.type == "cuda" else 8
        base = shard_batch(hb.base, self.cp, self.groups.cp_rank, self.groups.cp, align=align)
        src, real, seq = shard_index(hb.base.cu_seqlens, self.cp, self.groups.cp_rank, align)

        def take(t, fill):
            if t is None:
                return None
            return torch.where(real, t[src], torch.full_like(t[src], fill))

        sm = None
        if hb.sampling_mask is not None:
            sm = [hb.sampling_mask[int(i)] if bool(r) else [] for i, r in zip(src, real)]
        cu = hb.base.cu_seqlens
        n_seq = cu.numel() - 1
        seq_counts = seg_sum(hb.loss_mask.float(), segment_ids(cu, hb.base.num_tokens), n_seq)
        local = replace(hb, base=base, inference_logprobs=take(hb.inference_logprobs, 0.0),
                        teacher_logprobs=take(hb.teacher_logprobs, 0.0), advantages=take(hb.advantages, 0.0),
                        loss_mask=take(hb.loss_mask, False), ce_weights=take(hb.ce_weights, 0.0),
                        ref_kl_weights=take(hb.ref_kl_weights, 0.0), sampling_mask=sm,
                        has_inference=take(hb.has_inference, False) if hb.has_inference is not None else None)
        return local, (seq, n_seq, seq_counts)

    @torch.no_grad()
    def _recompute_inference_logprobs(self, b, ctx) -> None:
        """Fill the missing inference log-probs of micro-batch ``b`` (on the
        device) from the base model with the LoRA adapters disabled (the
        reference policy; reference trainer/rl.py:1004-1040)."""
        m = self.model
        if m.lora is None:
            raise RuntimeError("inference_logprobs are required: the rollouts carry none and the model has no "
                               "LoRA adapter to disable for a reference forward")
        with m.adapters_disabled():
            h = m.hidden(b.base.input_ids, ctx)
            tgt = b.base.targets.clamp_min(0)
            if h.is_cuda:
                lp, _ = lm_head.logprob_entropy(h, m.head_weight(), tgt, b.temperature, want_entropy=False,
                                                chunk=self.lm_head_chunk)
            else:
                lp, _ = lm_head.ref.logprob_entropy(m.logits(h), tgt, b.temperature)
        miss = b.missing_inference()
        b.inference_logprobs = torch.where(miss, lp.float().reshape(-1), b.inference_logprobs)

    def accumulate(self, batches, scales: dict[str, float], recompute: bool = False) -> dict[str, Any]:
        """Forward + backward of ``batches`` (this rank's micro-batches) into the
        gradient buffers with the given component normalisers.  No host
        synchronisation inside the loop: per-micro-batch metrics stay on the
        device and are returned as tensors."""
        c = self.config
        m = self.model
        dev = self.world.device
        dev_metrics: dict[str, list[torch.Tensor]] = {}
        loss_total = torch.zeros((), device=dev, dtype=torch.float32)
        tokens = 0
        for hb in batches:
            present = {"rl": bool(hb.loss_mask.any()),
                       "ce": hb.ce_weights is not None and bool((hb.loss_mask & (hb.ce_weights != 0)).any()),
                       "ref_kl": hb.ref_kl_weights is not None and bool((hb.loss_mask & (hb.ref_kl_weights != 0)).any())}
            any_tok = bool(hb.loss_mask.any())
            local_b, seq_info = self._shard_for_cp(hb)
            b = local_b.to(dev)
            tokens += hb.base.num_tokens
            ctx = m.batch_ctx(b.base.position_ids, b.base.cu_seqlens, b.base.max_seqlen, cp=b.base.cp)
            if recompute:
                self._recompute_inference_logprobs(b, ctx)
            h = m.hidden(b.base.input_ids, ctx)
            tgt = b.base.targets.clamp_min(0)
            lp, ent = self._logprobs(h, tgt, b)
            seg, n_seq, seq_counts = (None, None, None) if seq_info is None else (
                seq_info[0].to(dev), seq_info[1], seq_info[2].to(dev))
            loss, met = compute_loss(lp, b.inference_logprobs, b.teacher_logprobs, b.advantages, b.loss_mask, c.loss,
                                     cu_seqlens=b.base.cu_seqlens, ce_weights=b.ce_weights,
                                     ref_kl_weights=b.ref_kl_weights, component_scales=scales,
                                     rl_loss_fn=self.loss_fn, present=present, sync=False,
                                     seg=seg, n_seq=n_seq, seq_counts=seq_counts)
            loss.backward()
            if not h.is_cuda or getattr(m, "eager", False):
                m.collect_cpu_grads()
            loss_total += loss.detach().float()
            if any_tok:
                with torch.no_grad():
                    mk = b.loss_mask.float()
                    den = mk.sum().clamp_min(1.0)
                    dev_metrics.setdefault("entropy", []).append((ent.float() * mk).sum() / den)
                    dev_metrics.setdefault("trainer_logprob", []).append((lp.detach().float() * mk).sum() / den)
            for k, v in met.items():
                dev_metrics.setdefault(k, []).append(v)
        return {"loss_sum": loss_total, "metrics": dev_metrics, "tokens": tokens}

    def optimizer_step(self, acc: dict[str, Any], *, grad_scale: float = 1.0, extra: dict | None = None,
                       t0: float | None = None, num_samples: int = 0) -> dict[str, Any]:
        """Scale the accumulated gradients (streaming chunks), clip, step, and
        turn the step's device metrics into floats with one transfer."""
        c = self.config
        m = self.model
        if grad_scale != 1.0:
            for f in (m.trainable, m.expert_flat):
                if f is not None and f.grad is not None:
                    f.grad.mul_(grad_scale)
        lr = lr_at(self.step - getattr(self, "sched_offset", 0), c.optim.lr, max(1, c.max_steps or 1), c.scheduler)
        m.finalize_grads()
        st = self.optimizer.step(lr)
        after = getattr(m, "after_optimizer_step", None)
        if after is not None:
            after()
        self.step += 1
        lt = acc["loss_sum"].reshape(1) * grad_scale
        if dist.is_initialized() and self.dp_world * self.cp > 1:
            dist.all_reduce(lt, group=self.groups.dp_cp if self.cp > 1 else self.groups.dp)
        keys = list(acc["metrics"])
        means = [torch.stack([v.float().reshape(()) for v in acc["metrics"][k]]).mean() for k in keys]
        vals = torch.cat([lt.float().reshape(1)] + [x.reshape(1) for x in means]).cpu().tolist()
        metrics = dict(zip(keys, vals[1:]))
        metrics.update({"loss": vals[0], "optim/grad_norm": st["grad_norm"], "optim/lr": lr,
                        "train/num_samples": float(num_samples), "train/tokens": float(acc["tokens"])})
        metrics.update(extra or {})
        if t0 is not None:
            dt = time.perf_counter() - t0
            metrics.update(self.perf.step_metrics(acc["tokens"] * self.dp_world, dt, c.data.seq_len))
            emit_perf("trainer_step", step=self.step, seconds=dt, tokens=acc["tokens"])
        return metrics

    def train_on_examples(self, examples: list[RLExample]) -> dict[str, Any]:
        """One optimizer step on a whole rollout batch: global normalisers
        first (one small all-reduce), then the micro-batches, then the step."""
        t0 = time.perf_counter()
        batches = self._local_batches(examples)
        units = self._reduce(self._unit_counts(batches))
        scales = {"rl": float(units[0]), "ce": float(units[1]), "ref_kl": float(units[2])}
        acc = self.accumulate(batches, scales, recompute=self._need_inference_recompute(batches))
        return self.optimizer_step(acc, extra={"train/rl_units": scales["rl"]}, t0=t0, num_samples=len(examples))

    def train_streaming_step(self, chunk_iter) -> dict[str, Any]:
        """One optimizer step over rollout chunks that arrive one after another
        (reference trainer/rl.py:1491-1720): each chunk's micro-batches run
        forward + backward as soon as it is read, with unnormalised sums; the
        RL normaliser (units over every chunk and data-parallel rank) is known
        after the last chunk and applied as one gradient scale before the
        optimizer step.  CE / reference-KL components need their normalisers
        up front, so they are refused when a step spans several chunks, as in
        the reference."""
        t0 = time.perf_counter()
        total_units = torch.zeros(3, dtype=torch.float64)
        acc = None
        n_samples = 0
        for examples in chunk_iter:
            n_samples += len(examples)
            batches = self._local_batches(examples)
            if any(b.ce_weights is not None or b.ref_kl_weights is not None for b in batches):
                raise ValueError("CE / ref-KL loss components need non-streaming rollout publication when an "
                                 "optimizer step spans several chunks (orchestrator.rollout_chunk_examples)")
            total_units += self._unit_counts(batches)
            part = self.accumulate(batches, {"rl": 1.0, "ce": 1.0, "ref_kl": 1.0},
                                   recompute=self._need_inference_recompute(batches))
            if acc is None:
                acc = part
            else:
                acc["loss_sum"] = acc["loss_sum"] + part["loss_sum"]
                acc["tokens"] += part["tokens"]
                for k, v in part["metrics"].items():
                    acc["metrics"].setdefault(k, []).extend(v)
        units = self._reduce(total_units)
        rl = max(float(units[0]), 1.0)
        return self.optimizer_step(acc, grad_scale=1.0 / rl, extra={"train/rl_units": float(units[0])}, t0=t0,
                                   num_samples=n_samples)

    def _logprobs(self, h, tgt, b):
        m = self.model
        if b.sampling_mask is not None and any(b.sampling_mask):
            return self._support_logprobs(h, tgt, b)
        if h.is_cuda:
            return lm_head.logprob_entropy(h, m.head_weight(), tgt, b.temperature, gW=m.head_grad(), anchor=m.anchor,
                                           chunk=self.lm_head_chunk)
        z = lm_head.cpu_head_logits(h, m.head_weight(), m.head_grad())
        return lm_head.ref.logprob_entropy(z, tgt, b.temperature)

    def _support_logprobs(self, h, tgt, b):
        """Log-prob renormalised over each token's sampling support set
        (trainer/losses.py:30-69): lp = z_t/T - logsumexp_{j in S}(z_j/T)."""
        m = self.model
        if h.is_cuda:
            lp_full, ent = lm_head.logprob_entropy(h, m.head_weight(), tgt, b.temperature, gW=m.head_grad(),
                                                   anchor=m.anchor, chunk=self.lm_head_chunk)
        else:
            z = lm_head.cpu_head_logits(h, m.head_weight(), m.head_grad())
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
    def _chunks_of_step(self, step: int, C: int, claimed: list):
        """The C rollout chunks of optimizer step ``step`` (queue steps
        step*C .. step*C + C-1), read as each becomes STABLE."""
        for ci in range(C):
            batch = self.receiver.wait()
            want = step * C + ci
            if batch.step != want:
                raise ValueError(f"rollout queue step {batch.step} arrived where chunk {ci} of optimizer step "
                                 f"{step} (queue step {want}) was expected")
            man = batch.manifest
            if man is not None and man.optimizer_step is not None and man.optimizer_step != step:
                raise ValueError(f"rollout chunk {batch.step} belongs to optimizer step {man.optimizer_step}, "
                                 f"the trainer is at {step}")
            if self.world.rank == 0:
                self.receiver.claim(batch, step)
            claimed.append(batch)
            yield [example_from_payload(r, self.config.data) for r in read_training_records(batch.training_path)]

    def _log_samples(self, claimed: list) -> None:
        """``monitor.samples``: a sample of this step's rollouts into samples.jsonl."""
        sc = self.config.monitor.samples
        if not sc.enabled or self.step % sc.interval != 0:
            return
        recs = [example_from_payload(r, self.config.data) for b in claimed
                for r in read_training_records(b.training_path)]
        if getattr(self, "_sample_tok", None) is None:
            from ..data.tokenizer import tokenizer_for

            self._sample_tok = tokenizer_for(self.config.model)
        self.monitor.log_samples(sample_rows(recs, sc, self.config.seed, self.step, self._sample_tok), self.step)

    def run(self) -> int:
        from ..orchestrator.schedule import chunks_per_step

        c = self.config
        total = c.max_steps
        C = chunks_per_step(c)
        status = "failed"
        try:
            if c.policy_transfer.export_initial and self.step == 0:
                self.exporter.export(self.model, 0)
            while total is None or self.step < total:
                before = self.step
                if C > 1:
                    claimed: list = []
                    metrics = self.train_streaming_step(self._chunks_of_step(before, C, claimed))
                else:
                    batch = self.receiver.wait()
                    if self.world.rank == 0:
                        self.receiver.claim(batch, before)
                    claimed = [batch]
                    records = [example_from_payload(r, c.data) for r in read_training_records(batch.training_path)]
                    metrics = self.train_on_examples(records)
                if self.world.rank == 0:
                    for bt in claimed:
                        self.receiver.consumed(bt, before, self.step)
                self.monitor.log(metrics, self.step)
                if self.world.rank == 0:
                    self._log_samples(claimed)
                log.info("rl step %d loss %.4f grad_norm %.3f", self.step, metrics["loss"], metrics["optim/grad_norm"])
                if self.step % c.policy_transfer.export_every_steps == 0:
                    self.exporter.export(self.model, self.step)
                if self.ckpt is not None and c.ckpt.interval and self.step % c.ckpt.interval == 0:
                    self.ckpt.save(self.step, model=self.model, optimizer=self.optimizer, data_state=None,
                                   meta={"arch": self.model.cfg.to_dict(), **_lora_meta(self.config, self.model)},
                                   scheduler_state={"step": self.step})
            status = "completed"
            return 0
        finally:
            if self.ckpt is not None:
                self.ckpt.wait()
            self.exporter.close()
            self.monitor.finish(status=status, step=self.step)


def sample_rows(records: list[RLExample], sample_cfg, seed: int, step: int, tokenizer=None) -> list[dict]:
    """The rollouts of one step to keep in ``samples.jsonl``
    (``monitor.samples``): ``sample_ratio`` of them (at least one), at most
    ``max_samples``, drawn with a seed of the run and step; each row carries
    the prompt and completion (decoded when a tokenizer is given), reward,
    advantage and token counts."""
    import random

    if not records or (sample_cfg.sample_ratio is not None and sample_cfg.sample_ratio <= 0):
        return []
    n = len(records)
    if sample_cfg.sample_ratio is not None:
        n = max(1, int(len(records) * sample_cfg.sample_ratio))
    if sample_cfg.max_samples is not None:
        n = min(n, sample_cfg.max_samples)
    picked = records if n >= len(records) else random.Random(seed + step).sample(records, n)
    rows = []
    for r in picked:
        ids, mask = list(r.input_ids or []), list(r.loss_mask or [])
        first = next((i for i, m in enumerate(mask) if m), len(ids))
        prompt, completion = ids[:first], ids[first:]
        md = r.metadata or {}
        row = {"example_id": md.get("example_id", md.get("group")), "reward": r.reward,
               "advantage": r.advantage if isinstance(r.advantage, (int, float)) else None,
               "prompt_tokens": len(prompt), "completion_tokens": len(completion)}
        if tokenizer is not None:
            row["prompt"] = tokenizer.decode(prompt)
            row["completion"] = tokenizer.decode(completion)
        else:
            row["prompt_ids"], row["completion_ids"] = prompt, completion
        rows.append(row)
    return rows


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
