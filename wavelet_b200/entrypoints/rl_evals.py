"""``wavelet evals``: evaluate the served (or in-process) policy on every
``eval.env`` once, without training (reference entrypoints/rl_evals.py).
The config is validated as eval-only (``max_steps`` forced to 0)."""

from __future__ import annotations

import json
import sys

from ..configs.config import RLConfig
from ..monitor import setup_logger
from ..utils.config import load_config


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config(RLConfig, [*argv, "--max-steps", "0"])
    if cfg.eval is None or not cfg.eval.env:
        raise SystemExit("standalone evals need at least one eval.env entry")
    setup_logger("evals", cfg.output_dir, cfg.log.level, cfg.log.json_console, cfg.log.json_file)
    from ..inference.policy import create_policy_inference_engine
    from ..orchestrator.evals import run_evals
    from ..orchestrator.scheduler import _GeneratorAdapter

    engine = create_policy_inference_engine(cfg)
    engine.setup()
    try:
        m = run_evals(cfg, _GeneratorAdapter(engine), step=0)
    finally:
        close = getattr(engine, "close", None)
        if close:
            close()
    print(json.dumps(m, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
