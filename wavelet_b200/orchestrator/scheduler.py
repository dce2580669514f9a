"""``wavelet rl-inference``: the rollout role in process mode.

For every optimizer step s (from the resume cursor on):

1. wait until a policy snapshot >= ``required_policy_step(s)`` is STABLE
   (``max_async_level`` lets generation run ahead of training);
2. load it into the inference engine (HTTP servers or in-process);
3. materialise the step's rollouts (generate, score, advantages, zero-
   advantage filtering) and publish them to the rollout queue.

On resume, queue batches at or beyond the resume step are discarded
(orchestrator/scheduler.py:1912-1996 of the reference).  Orchestrator
metrics are appended to ``orchestrator_metrics.jsonl``.
"""

from __future__ import annotations

import logging
import sys
import time
from pathlib import Path

from ..configs.config import RLConfig
from ..monitor import append_jsonl, setup_logger, utc_now
from ..transport.queue import FileSystemPolicyReceiver, FileSystemRolloutSender, prune_from, stable_steps
from ..utils.config import load_config
from .rollouts import RLOrchestrator
from .schedule import required_policy_step, target_steps

log = logging.getLogger("wavelet")


class RolloutScheduler:
    def __init__(self, cfg: RLConfig, engine=None, prompts=None):
        self.cfg = cfg
        out = Path(cfg.output_dir)
        self.out = out
        self.sender = FileSystemRolloutSender(out, cfg.transport)
        self.policies = FileSystemPolicyReceiver(out, cfg.policy_transfer)
        if engine is None:
            from ..inference.policy import create_policy_inference_engine

            engine = create_policy_inference_engine(cfg)
            engine.setup()
        self.engine = engine
        if prompts is None:
            from .runtime import build_prompt_source

            prompts = build_prompt_source(cfg, 1 << 30)
        self.orch = RLOrchestrator(cfg, _GeneratorAdapter(engine), self.sender, prompts)

    def resume_step(self) -> int:
        """First step to produce: one past the trainer's last consumed batch."""
        done = [s for s in stable_steps(self.sender.queue_dir)]
        consumed = [s for s in done if (self.sender.queue_dir / f"step-{s:06d}" / "consumed.json").exists()]
        start = (max(consumed) + 1) if consumed else 0
        prune_from(self.sender.queue_dir, start)
        return start

    def run(self) -> int:
        total = target_steps(self.cfg)
        step = self.resume_step()
        loaded = None
        while step < total:
            need = required_policy_step(step, self.cfg)
            snap = self.policies.wait_for_step(need)
            if loaded != snap.step:
                self.engine.load_policy(snap.step_dir, step=snap.step)
                loaded = snap.step
            t0 = time.perf_counter()
            self.orch.publish(step, policy_step=loaded)
            m = dict(self.orch.last_stats)
            m.update({"step": step, "policy_step": loaded, "policy_lag": step - loaded,
                      "time/publish_seconds": time.perf_counter() - t0, "timestamp": utc_now()})
            append_jsonl(self.out / "orchestrator_metrics.jsonl", m)
            log.info("published rollouts for step %d (policy %d, reward %.4f)", step, loaded, m.get("reward/mean", 0.0))
            step += 1
        return 0


class _GeneratorAdapter:
    """Give ``RLOrchestrator`` a ``generate(prompts, params)`` over any engine."""

    def __init__(self, engine):
        self.engine = engine
        self.stats: dict[str, float] = {}

    def generate(self, prompts, params):
        from ..inference.engine import Completion
        from ..data.rl import RLExample

        if hasattr(self.engine, "generator") and getattr(self.engine, "generator", None) is not None:
            out = self.engine.generator.generate(prompts, params)
            self.stats = dict(self.engine.generator.stats)
            return out
        recs = []
        for pi, p in enumerate(prompts):
            for j in range(params.n):
                recs.append(RLExample(prompt=[], completion=[], advantage=None, reward=None,
                                      metadata={"prompt_ids": p, "prompt_index": pi, "sample_index": j}))
        ann = self.engine.annotate(recs)
        res = []
        for r in ann:
            md = r.metadata or {}
            res.append(Completion(md.get("prompt_index", 0), md.get("sample_index", 0), list(md.get("prompt_ids", [])),
                                  list(md.get("completion_ids", [])), list(r.inference_logprobs or []),
                                  md.get("finish_reason", "length"), r.sampling_mask))
        return res


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config(RLConfig, argv)
    setup_logger("rl-inference", cfg.output_dir, cfg.log.level, cfg.log.json_console, cfg.log.json_file)
    return RolloutScheduler(cfg).run()


if __name__ == "__main__":
    sys.exit(main())
