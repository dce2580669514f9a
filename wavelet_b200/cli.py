"""``wavelet`` command-line dispatcher (same command names as the reference's
cli.py:6-75).  Each command's module exposes ``main(argv) -> int`` and is
imported lazily so ``wavelet --help`` stays fast."""

from __future__ import annotations

import importlib
import sys

PUBLIC_COMMANDS = {
    "rl": ("wavelet_b200.orchestrator.runtime", "Run reinforcement learning launcher"),
    "sft": ("wavelet_b200.trainer.sft", "Run supervised fine-tuning"),
    "debug": ("wavelet_b200.debug", "Inspect and probe RL subsystems"),
    "evals": ("wavelet_b200.entrypoints.rl_evals", "Evaluate a served policy without starting training"),
    "convert-checkpoint": ("wavelet_b200.tools.convert_checkpoint", "Convert a checkpoint to Hugging Face safetensors"),
    "convert-traces": ("wavelet_b200.tools.convert_traces", "Convert trace JSONL files to a dataset"),
    "benchmark": ("wavelet_b200.tools.benchmark", "Run and compare training performance benchmarks"),
    "dashboard": ("wavelet_b200.entrypoints.dashboard", "Serve the read-only run dashboard over run directories"),
    "rl-trainer": ("wavelet_b200.trainer.rl", "Run RL trainer"),
    "rl-orchestrator": ("wavelet_b200.entrypoints.rl_orchestrator", "Run RL orchestrator"),
    "rl-inference": ("wavelet_b200.orchestrator.scheduler", "Run RL inference annotation stage"),
    "inference-server": ("wavelet_b200.inference.server", "Run OpenAI-compatible inference server"),
}

INTERNAL_COMMANDS = {
    "slurm-worker": ("wavelet_b200.deployment.slurm", "Run roles inside a SLURM allocation"),
    "synth-run": ("wavelet_b200.dashboard.synth", "Write a synthetic run directory for dashboard development"),
    "native-inference-server": ("wavelet_b200.inference.server", "Run the native inference server"),
}

COMMANDS = {**PUBLIC_COMMANDS, **INTERNAL_COMMANDS}


def usage() -> str:
    lines = ["Usage: wavelet <command> [args]", "Commands:"]
    lines += [f"  {c:<22} {d}" for c, (_, d) in PUBLIC_COMMANDS.items()]
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(usage())
        return 1 if not argv else 0
    cmd = argv[0]
    if cmd not in COMMANDS:
        print(f"Unknown command: {cmd}")
        return 1
    module = importlib.import_module(COMMANDS[cmd][0])
    return int(module.main(argv[1:]) or 0)


if __name__ == "__main__":
    sys.exit(main())
