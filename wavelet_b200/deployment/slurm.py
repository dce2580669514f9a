"""SLURM deployment: render an sbatch script for ``wavelet sft`` / ``wavelet rl``
and submit it; ``wavelet slurm-worker`` runs a role inside the allocation
(reference deployment/slurm.py:26-744).

Layout of an allocation (``deployment``): the first ``num_train_nodes`` nodes
run the trainer (``torchrun`` with one rank per GPU, rendezvous on the first
train node's ``trainer_master_port``), the remaining ``num_inference_nodes``
run ``inference_replicas_per_node`` inference servers each.  The orchestrator
role (``rl-inference``) runs on the first train node.  Roles find each other
through the node list SLURM provides (``SLURM_JOB_NODELIST``) and the shared
filesystem under ``output_dir``.

``submit`` writes ``<output_dir>/slurm/<job>.sbatch`` and calls ``sbatch``;
with ``WAVELET_SLURM_DRY_RUN=1`` (or when ``sbatch`` is not installed) it only
writes the script and prints its path.
"""

from __future__ import annotations

import os
import shlex
import shutil
import subprocess
import sys
from pathlib import Path

from ..utils import pathing


def directives(cfg, nodes: int) -> list[str]:
    s = cfg.slurm
    d = cfg.deployment
    out = [f"--job-name={s.job_name}", f"--nodes={nodes}", "--ntasks-per-node=1", f"--gpus-per-node={d.gpus_per_node}"]
    for flag, v in (("--partition", s.partition), ("--account", s.account), ("--qos", s.qos),
                    ("--time", s.time_limit), ("--constraint", s.constraint), ("--reservation", s.reservation),
                    ("--nodelist", s.nodelist), ("--exclude", s.exclude), ("--cpus-per-task", s.cpus_per_task),
                    ("--mem", s.memory)):
        if v is not None:
            out.append(f"{flag}={v}")
    if s.exclusive:
        out.append("--exclusive")
    out += list(s.extra_directives)
    return out


def render_sbatch(cfg, command: str, argv: list[str]) -> str:
    s, d = cfg.slurm, cfg.deployment
    nodes = d.num_train_nodes + d.num_inference_nodes
    out_dir = Path(cfg.output_dir)
    lines = ["#!/bin/bash"]
    lines += [f"#SBATCH {x}" for x in directives(cfg, nodes)]
    lines += [f"#SBATCH --output={out_dir / 'slurm' / '%x-%j.out'}", f"#SBATCH --error={out_dir / 'slurm' / '%x-%j.err'}"]
    lines += ["set -euo pipefail", f"cd {shlex.quote(str(s.project_dir))}"]
    lines += list(s.setup_commands)
    worker = shlex.join([s.python_command, "-m", "wavelet_b200", "slurm-worker", command, *argv])
    lines.append(f"srun --nodes={nodes} --ntasks={nodes} --ntasks-per-node=1 --kill-on-bad-exit=1 {worker}")
    return "\n".join(lines) + "\n"


def launch_slurm(cfg, command: str, argv: list[str]) -> int:
    out = Path(cfg.output_dir) / "slurm"
    out.mkdir(parents=True, exist_ok=True)
    script = out / f"{cfg.slurm.job_name}.sbatch"
    script.write_text(render_sbatch(cfg, command, [a for a in argv]))
    script.chmod(0o755)
    if os.environ.get("WAVELET_SLURM_DRY_RUN") or shutil.which("sbatch") is None:
        print(f"wrote {script} (not submitted)")
        return 0
    r = subprocess.run(["sbatch", "--parsable", str(script)], capture_output=True, text=True)
    if r.returncode != 0:
        print(r.stderr, file=sys.stderr)
        return r.returncode
    print(f"submitted job {r.stdout.strip()} ({script})")
    return 0


def expand_nodelist(nodelist: str) -> list[str]:
    """Expand a SLURM node list such as ``gpu[01-03,07],login1``."""
    nodes, i, cur, depth = [], 0, "", 0
    parts = []
    for ch in nodelist:
        if ch == "[":
            depth += 1
        elif ch == "]":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append(cur)
            cur = ""
        else:
            cur += ch
    if cur:
        parts.append(cur)
    for p in parts:
        if "[" not in p:
            nodes.append(p)
            continue
        prefix, rng = p.split("[", 1)
        rng = rng.rstrip("]")
        for piece in rng.split(","):
            if "-" in piece:
                a, b = piece.split("-")
                w = len(a)
                nodes += [f"{prefix}{i:0{w}d}" for i in range(int(a), int(b) + 1)]
            else:
                nodes.append(prefix + piece)
    return nodes


def role_for_node(cfg, node_index: int) -> tuple[str, int]:
    d = cfg.deployment
    if node_index < d.num_train_nodes:
        return "train", node_index
    return "inference", node_index - d.num_train_nodes


def worker_commands(cfg, command: str, argv: list[str], node_index: int, nodes: list[str]) -> list[list[str]]:
    """Commands this node runs (the trainer node 0 also runs the orchestrator)."""
    d, s = cfg.deployment, cfg.slurm
    py = shlex.split(s.python_command)
    role, idx = role_for_node(cfg, node_index)
    master = nodes[0] if nodes else "127.0.0.1"
    if role == "train":
        train_cmd = "sft" if command == "sft" else "rl-trainer"
        cmds = [[*py, "-m", "torch.distributed.run", f"--nnodes={d.num_train_nodes}",
                 f"--nproc-per-node={d.gpus_per_node}", f"--node-rank={idx}", f"--master-addr={master}",
                 f"--master-port={d.trainer_master_port}", "-m", "wavelet_b200", train_cmd, *argv]]
        if command == "rl" and idx == 0:
            cmds.append([*py, "-m", "wavelet_b200", "rl-inference", *argv])
        return cmds
    base_port = 8000
    return [[*py, "-m", "wavelet_b200", "inference-server", *argv, "--inference.http.port", str(base_port + r)]
            for r in range(d.inference_replicas_per_node)]


def main(argv: list[str] | None = None) -> int:
    """``wavelet slurm-worker <command> <config args>``: run this node's roles."""
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        raise SystemExit("usage: wavelet slurm-worker {sft,rl} [config args]")
    command, rest = argv[0], argv[1:]
    from ..configs.config import RLConfig, SFTConfig
    from ..utils.config import load_config

    cfg = load_config(SFTConfig if command == "sft" else RLConfig, rest)
    nodes = expand_nodelist(os.environ.get("SLURM_JOB_NODELIST", "127.0.0.1"))
    node_index = int(os.environ.get("SLURM_NODEID", "0"))
    procs = [subprocess.Popen(c) for c in worker_commands(cfg, command, rest, node_index, nodes)]
    codes = [p.wait() for p in procs]
    return next((c for c in codes if c), 0)


__all__ = ["render_sbatch", "launch_slurm", "expand_nodelist", "worker_commands", "pathing"]
