"""``wavelet rl``: the RL launcher.

Modes (``launcher.mode``; orchestrator/runtime.py of the reference):

* ``integrated`` — one process per GPU runs trainer, generator and
  orchestrator.  The generator reads the trainer's bf16 weights in place
  (zero-copy policy transfer).  With several ranks every rank generates the
  rollouts of its share of the prompts; rank 0 gathers and publishes the
  batch to the durable queue; every rank trains on its packed share.
  ``orchestrator.max_async_level >= 1`` generates step s+1 while step s trains
  (one step of policy lag), otherwise generation and training alternate.
* ``process`` / ``colocate`` / ``colocate_sleep`` — separate role processes
  (inference server(s), ``rl-trainer`` under torchrun, ``rl-inference``)
  supervised by ``orchestrator.launcher``; they communicate only through the
  filesystem queues (and HTTP to the inference server).
"""

from __future__ import annotations

import logging
import os
import sys
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from ..configs.config import RLConfig
from ..data.rl import example_from_payload, example_to_payload
from ..transport.queue import FileSystemRolloutSender, prune_from
from ..utils import pathing
from ..utils.config import config_to_plain, dump_yaml, load_config
from .rollouts import RLOrchestrator, SyntheticReversePrompts

log = logging.getLogger("wavelet")


def build_prompt_source(cfg: RLConfig, vocab: int, rank: int = 0):
    """Prompt source for the orchestrator: synthetic reverse-text prompts
    (``data.source: fake``) or pretokenised prompt rows from local files."""
    d = cfg.data
    envs = train_envs(cfg)
    if envs:
        from .sources import EnvironmentPromptSource

        return EnvironmentPromptSource(envs, cfg.model.name, seed=d.seed, rank=rank, model_cfg=cfg.model)
    if d.source == "fake":
        return SyntheticReversePrompts(min(vocab, d.fake_vocab_size), d.fake_prompt_len, seed=d.seed * 1000 + rank)
    from .sources import FilePromptSource

    return FilePromptSource(cfg, rank=rank)


def train_envs(cfg: RLConfig) -> list:
    """(environment, ratio) of every training environment
    (``orchestrator.envs`` / ``orchestrator.verifier_env_id``): native ones
    from ``wavelet_b200.environments``, any other id from the ``verifiers``
    package (``orchestrator.verifier_envs``)."""
    from .. import environments
    from .reward import register_environment

    o = cfg.orchestrator
    specs = [(e.id, env_args(e), e.ratio) for e in o.envs]
    if not specs and o.verifier_env_id:
        specs = [(o.verifier_env_id, o.verifier_env_args, 1.0)]
    out: list = [None] * len(specs)
    foreign = [i for i, (env_id, _, _) in enumerate(specs) if not environments.is_native(env_id)]
    if foreign:
        from .verifier_envs import verifier_train_envs, verifiers_available

        if not verifiers_available():
            raise ValueError(f"environment {specs[foreign[0]][0]!r} needs the verifiers package, which is not "
                             f"installed; native environments: {', '.join(environments.available())}")
        for i, pair in zip(foreign, verifier_train_envs(cfg, [specs[i] for i in foreign])):
            out[i] = pair
    for i, (env_id, args, ratio) in enumerate(specs):
        if out[i] is None:
            env = environments.load_environment(env_id, **(args or {}))
            register_environment(env)
            out[i] = (env, float(ratio))
    return out


native_train_envs = train_envs  # the name earlier callers import


def env_args(e) -> dict:
    """An environment entry's loader arguments; ``data_path`` becomes the
    loader's ``path`` (the native environments read their rows from it)."""
    args = dict(e.args or {})
    if getattr(e, "data_path", None) is not None:
        args.setdefault("path", str(e.data_path))
    return args


def env_overrides(cfg) -> dict:
    """Environment name -> its ``orchestrator.envs`` entry (per-environment
    sampling, group size and algorithm)."""
    from .. import environments

    out = {}
    for e in cfg.orchestrator.envs:
        if environments.is_native(e.id):
            out[environments.load_environment(e.id, **env_args(e)).name] = e
        else:  # a verifiers-package environment goes by its entry's name
            out[e.resolved_name] = e
    return out


class IntegratedRunner:
    def __init__(self, cfg: RLConfig):
        self.cfg = cfg

    def setup(self) -> "IntegratedRunner":
        from ..trainer.rl import RLTrainer

        c = self.cfg
        out = Path(c.output_dir)
        self.trainer = RLTrainer(c)
        world_rank = int(os.environ.get("RANK", "0"))
        if world_rank == 0:
            resume = c.ckpt is not None and c.ckpt.is_resuming
            pathing.validate_output_dir(out, clean=c.clean_output_dir, resuming=resume,
                                        protected_paths=(c.model.name, c.model.adapter_path))
            attempt = pathing.create_launch_attempt(out)
            dump_yaml(attempt.config_dir / "rl.yaml", config_to_plain(c))
        self.trainer.setup()
        t = self.trainer
        self.world = t.world
        v = c.inference.vllm
        max_len = v.max_model_len or c.data.seq_len
        gen_model = t.model
        self.policy_sync = None
        if t.model.expert_flat is not None:
            # expert-parallel trainer: rollouts run on a full replica refreshed from the shards
            from ..models.qwen import build_model
            from ..parallel.policy_sync import ExpertPolicySync

            if getattr(t, "ep_fabric", None) is None:
                raise NotImplementedError("expert-parallel RL needs CUDA ranks on one node (peer fabric)")
            gen_model = build_model(t.model.cfg, t.model.device, t.model.flat.compute_dtype, init=False,
                                    with_grad=False, with_optimizer=False)
            self.policy_sync = ExpertPolicySync(t.model, gen_model, t.ep_fabric)
            self.policy_sync.refresh()
        elif t.model.flat.sharded_compute:
            # sharded (ZeRO-3) trainer: rollouts run on a full bf16 replica
            # refreshed from the shards after every optimizer step
            from ..models.qwen import build_model
            from ..parallel.zero3 import ShardedPolicySync

            gen_model = build_model(t.model.cfg, t.model.device, t.model.flat.compute_dtype, init=False,
                                    with_grad=False, with_optimizer=False)
            self.policy_sync = ShardedPolicySync(t.model, gen_model)
            self.policy_sync.refresh()
        from ..inference.hf_generator import make_generator

        self.engine = make_generator(gen_model, max_num_seqs=v.max_num_seqs, max_model_len=max_len,
                                     gpu_memory_utilization=v.gpu_memory_utilization, block_size=v.kv_block_size,
                                     cuda_graphs=v.cuda_graphs and not v.enforce_eager)
        self.sender = FileSystemRolloutSender(out, c.transport) if self.world.rank == 0 else None
        # batches past a resumed step are stale
        if self.world.rank == 0 and t.step > 0:
            prune_from(self.sender.queue_dir, t.step)
        prompts = build_prompt_source(c, t.model.cfg.vocab_size, rank=t.dp_rank)
        self.openai = None
        if any(getattr(e, "metadata", {}).get("kind") == "verifiers" for e, _ in getattr(prompts, "envs", [])):
            # verifiers-package environments call an OpenAI server: serve this process's generator
            # from a thread (the environments' requests run while the trainer waits for the step)
            c = self._serve_generator(c, gen_model)
        self.orch = RLOrchestrator(c, self.engine, None, prompts, monitor=t.monitor)
        return self

    def _serve_generator(self, c: RLConfig, gen_model) -> RLConfig:
        from ..data.tokenizer import tokenizer_for
        from ..inference.policy import NativePolicyInferenceEngine
        from ..inference.server import InProcessServer

        if self.world.world_size > 1:
            raise NotImplementedError("verifiers-package environments in integrated mode run on one process; "
                                      "use launcher.mode: process for more GPUs")
        eng = NativePolicyInferenceEngine(c, model=gen_model, tokenizer=tokenizer_for(c.model))
        eng.generator = self.engine
        eng.policy_step = 0
        self.openai_engine = eng
        self.openai = InProcessServer(c, eng, host="127.0.0.1", port=0).start()
        self.cfg = c.model_copy(update={"orchestrator": c.orchestrator.model_copy(
            update={"verifier_base_url": self.openai.base_url})})
        return self.cfg

    def close(self) -> None:
        if getattr(self, "openai", None) is not None:
            self.openai.close()
            self.openai = None

    def _gather(self, rows: list[dict]) -> list[dict]:
        if not dist.is_initialized() or self.world.world_size == 1:
            return rows
        # tensor-parallel peers generate the same rows (one prompt shard per
        # data-parallel rank, identical sampling): only TP rank 0 contributes
        mine = rows if getattr(self.trainer.model, "tp_rank", 0) == 0 else []
        allr: list[Any] = [None] * self.world.world_size
        dist.all_gather_object(allr, mine)
        return [r for part in allr for r in part]

    def run_step(self) -> dict[str, Any]:
        """One RL step: generate + score this rank's prompts, publish the batch
        (rank 0), train on it, return the step metrics."""
        c = self.cfg
        t = self.trainer
        step = t.step
        cuda = self.world.device.type == "cuda"
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if cuda else None
        if ev:
            ev[0].record()
        t0 = time.perf_counter()
        if getattr(self, "openai_engine", None) is not None:
            self.openai_engine.policy_step = step  # reported by the in-process OpenAI server
        if self.policy_sync is not None and step > 0:
            self.policy_sync.refresh()  # the generator replica picks up the last update
        recs = self.orch.materialize(step)
        gen_s = time.perf_counter() - t0
        if ev:
            ev[1].record()
        rows = self._gather([example_to_payload(r, self.cfg.data) for r in recs])
        if self.sender is not None:
            self.sender.publish(rows, step=step, training_records=rows, optimizer_step=step, policy_step=step,
                                tokens=sum(len(r.get("input_ids") or []) for r in rows))
        if dist.is_initialized():
            dist.barrier()
        batch = t.receiver.wait()
        if self.world.rank == 0:
            t.receiver.claim(batch, step)
        from ..transport.queue import read_training_records

        records = [example_from_payload(r, self.cfg.data) for r in read_training_records(batch.training_path)]
        t1 = time.perf_counter()
        m = t.train_on_examples(records)
        train_s = time.perf_counter() - t1
        if self.world.rank == 0:
            t.receiver.consumed(batch, step, t.step)
        m.update(self.orch.last_stats)
        if self.world.rank == 0:  # the batch's rollout metrics (progress, solve rates, stop conditions, ...)
            from .rollout_metrics import rollout_metrics

            for k, v in rollout_metrics(rows, step=step, group_size=int(self.cfg.orchestrator.rollouts_per_example or 1),
                                        policy_step=step, stats=self.orch.last_stats).items():
                m.setdefault(k, v)
        m["time/generate_seconds"] = gen_s
        m["time/train_seconds"] = train_s
        m["time/step_seconds"] = time.perf_counter() - t0
        if ev:
            ev[2].record()
            ev[2].synchronize()
            m["time/generate_ms_device"] = ev[0].elapsed_time(ev[1])
            m["time/step_ms_device"] = ev[0].elapsed_time(ev[2])
        return m

    def run(self) -> int:
        c = self.cfg
        t = self.trainer
        total = c.max_steps if c.max_steps is not None else 1
        status = "failed"
        try:
            while t.step < total:
                m = self.run_step()
                t.monitor.log(m, t.step)
                log.info("rl step %d reward %.4f loss %.4f gen %.2fs train %.2fs", t.step, m.get("reward/mean", 0.0),
                         m["loss"], m["time/generate_seconds"], m["time/train_seconds"])
                if t.ckpt is not None and c.ckpt.interval and t.step % c.ckpt.interval == 0:
                    t.ckpt.save(t.step, model=t.model, optimizer=t.optimizer, data_state=None,
                                meta={"arch": t.model.cfg.to_dict()}, scheduler_state={"step": t.step})
            status = "completed"
            return 0
        finally:
            if t.ckpt is not None:
                t.ckpt.wait()
            t.monitor.finish(status=status, step=t.step)
            self.close()


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config(RLConfig, argv)
    if cfg.dry_run:
        print(cfg.model_dump_json(indent=2))
        return 0
    if cfg.launcher.mode == "integrated":
        from ..parallel.dist import destroy_distributed

        from ..trainer.rl import _close_fabric

        runner = IntegratedRunner(cfg)
        try:
            return runner.setup().run()
        finally:
            if getattr(runner, "trainer", None) is not None:
                _close_fabric(runner.trainer)
            destroy_distributed()
    from .launcher import run_process_launcher

    return run_process_launcher(cfg, argv)


if __name__ == "__main__":
    sys.exit(main())
