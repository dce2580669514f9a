"""``wavelet rl-inference``: the rollout role in process mode.

Steps are generated ahead of the trainer with bounded prefetch and published
in order by ``orchestrator.async_scheduler.AsyncRolloutScheduler`` (policy
loads as snapshots appear, retries, evals, colocate_sleep, resume of the
prompt and curriculum state).  On resume, queue batches at or beyond the
resume step are discarded (orchestrator/scheduler.py:1912-1996 of the
reference).  Orchestrator metrics are appended to ``orchestrator_metrics.jsonl``.
"""

from __future__ import annotations

import logging
import sys
from pathlib import Path

from ..configs.config import RLConfig
from ..monitor import setup_logger
from ..transport.queue import FileSystemPolicyReceiver, FileSystemRolloutSender
from ..utils.config import load_config
from .rollouts import RLOrchestrator

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
        return self.pipeline().resume_step()

    def pipeline(self):
        from .async_scheduler import AsyncRolloutScheduler

        if getattr(self, "_pipeline", None) is None:
            self._pipeline = AsyncRolloutScheduler(self.cfg, self.orch, self.engine, self.sender, self.policies)
        return self._pipeline

    def run(self) -> int:
        """Bounded-prefetch, in-order rollout publishing (``AsyncRolloutScheduler``),
        with the live state (``orchestrator.state_server``: HTTP) and the
        periodic pipeline status line."""
        from .state_server import OrchestratorRunState, maybe_state_server

        pipe = self.pipeline()
        state = OrchestratorRunState(self.out, max_events=self.cfg.orchestrator.state_server.max_events)
        pipe.run_state = state
        pipe.status_sink = lambda snap: state.update(pipeline=snap, queue_depth=snap["ready"] + snap["inflight"])
        handle = maybe_state_server(self.cfg, state)
        wb = self._wandb_monitor()
        if wb is not None:  # orchestrator metrics also go to W&B (the shared run of the roles when launched together)
            pipe.metrics_sink = lambda m: wb.log({k: v for k, v in m.items() if k not in ("step", "timestamp")},
                                                 m.get("optimizer_step", m.get("step")))
        status = "failed"
        try:
            rc = pipe.run()
            state.update(status="completed")
            status = "completed"
            return rc
        except BaseException:
            state.update(status="failed")
            raise
        finally:
            if handle is not None:
                handle.close()
            if wb is not None:
                wb.finish(status=status, step=None)

    def _wandb_monitor(self):
        """A W&B-only monitor of the rollout role (``monitor.wandb``); the
        local metric files stay the trainer's and ``orchestrator_metrics.jsonl``."""
        w = self.cfg.monitor.wandb
        if not self.cfg.monitor.enabled or not w.enabled or w.mode == "disabled":
            return None
        from ..monitor import RunMonitor
        from ..utils.config import config_to_plain

        mon = RunMonitor(self.out, write_events=False, write_metrics_jsonl=False, write_metrics_csv=False,
                         write_run_metadata=False, write_heartbeat=False, log_cuda_memory=False,
                         log_disk_usage=False, wandb=w)
        mon.start_run(run_config=config_to_plain(self.cfg))
        return mon if mon._wandb is not None else None


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
    from ..configs.inert import warn_inert

    warn_inert(cfg)  # settings of the reference's schema that do nothing here, named
    return RolloutScheduler(cfg).run()


if __name__ == "__main__":
    sys.exit(main())
