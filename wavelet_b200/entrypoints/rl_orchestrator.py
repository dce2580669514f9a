"""``wavelet rl-orchestrator``: publish rollout batches for ``max_steps`` steps
with the configured inference engine and print each published batch path
(reference entrypoints/rl_orchestrator.py:11).  Unlike ``rl-inference`` it
does not wait for policy snapshots: it drives the engine's current policy."""

from __future__ import annotations

import sys
from pathlib import Path

from ..configs.config import RLConfig
from ..monitor import setup_logger
from ..transport.queue import FileSystemRolloutSender
from ..utils.config import load_config


def main(argv: list[str] | None = None) -> int:
    cfg = load_config(RLConfig, list(sys.argv[1:] if argv is None else argv))
    setup_logger("rl-orchestrator", cfg.output_dir, cfg.log.level, cfg.log.json_console, cfg.log.json_file)
    from ..inference.policy import create_policy_inference_engine
    from ..orchestrator.rollouts import RLOrchestrator
    from ..orchestrator.runtime import build_prompt_source
    from ..orchestrator.scheduler import _GeneratorAdapter
    from ..orchestrator.trace import TraceWriter

    engine = create_policy_inference_engine(cfg)
    engine.setup()
    sender = FileSystemRolloutSender(Path(cfg.output_dir), cfg.transport)
    orch = RLOrchestrator(cfg, _GeneratorAdapter(engine), sender, build_prompt_source(cfg, 1 << 30))
    trace = TraceWriter(cfg.output_dir, "orchestrator")
    try:
        for step in range(cfg.max_steps or 1):
            batch = orch.publish(step)
            trace.event("batch_published", step=step, path=str(getattr(batch, "path", batch)))
            print(getattr(batch, "path", batch), flush=True)
    finally:
        close = getattr(engine, "close", None)
        if close:
            close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
