"""SLURM deployment of ``wavelet sft`` / ``wavelet rl`` (reference
deployment/slurm.py:26-744).

``launch_slurm`` writes ``<output_dir>/slurm/<job>.sbatch`` and submits it with
``sbatch`` (with ``WAVELET_SLURM_DRY_RUN=1``, or without ``sbatch``, it only
writes the script).  The batch script runs ONE controller,
``wavelet slurm-worker <command> <config args>``, on the allocation's first
node; the controller places every role on the allocation with ``srun`` and
supervises it:

* hosts: ``SLURM_JOB_NODELIST`` expanded; the first
  ``deployment.num_train_nodes`` hosts train, the next
  ``deployment.num_inference_nodes`` serve inference
  (``deployment.inference_replicas_per_node`` servers each, ports
  ``inference.http.port + i`` over the replicas);
* role configs go to the launch attempt's ``configs/attempt_<n>/resolved``
  (the ``slurm`` / ``deployment`` sections stripped, each server bound to
  0.0.0.0 on its port, the rollout role pointed at every replica, an NCCL
  policy transfer pointed at the first train host) and every role logs to
  ``logs/attempt_<n>/<role>.log``;
* RL order: the inference servers first (one ``srun`` step each, pinned to its
  host with ``slurm.inference_cpus_per_replica`` / ``..._memory_per_replica``),
  then a wait until every replica answers ``/health`` (failing fast when a
  server exits), then the trainer (one ``srun`` step over the train hosts
  running ``torch.distributed.run`` with a c10d rendezvous on the first train
  host's ``trainer_master_port``) and the rollout role (``rl-inference``, on the
  controller's node, no GPUs);
* lifecycle: when any role exits non-zero every other role is terminated and
  the controller exits 1; when the trainer and the rollout role finish the
  servers are terminated and it exits 0; SIGTERM / SIGINT (job cancel,
  preemption) terminate every role first.  SFT runs the trainer step only.
"""

from __future__ import annotations

import os
import shlex
import shutil
import signal
import subprocess
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable

from ..utils import pathing
from ..utils.config import config_to_plain, dump_yaml


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
    # the controller runs on the batch host (the first node) and places the roles with srun
    lines.append("exec " + shlex.join([*shlex.split(s.python_command), "-m", "wavelet_b200", "slurm-worker",
                                        command, *argv]))
    return "\n".join(lines) + "\n"


def launch_slurm(cfg, command: str, argv: list[str]) -> int:
    out = Path(cfg.output_dir) / "slurm"
    out.mkdir(parents=True, exist_ok=True)
    script = out / f"{cfg.slurm.job_name}.sbatch"
    script.write_text(render_sbatch(cfg, command, list(argv)))
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
    nodes, cur, depth = [], "", 0
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


@dataclass
class RoleLaunch:
    name: str
    argv: list[str]
    env: dict[str, str] = field(default_factory=dict)
    service: bool = False  # a server: terminated once the jobs finish
    endpoint: str | None = None  # health URL base of a server


def _srun(hosts: list[str], *, gpus_per_task: int | None = None, cpus: int | None = None,
          mem: str | None = None) -> list[str]:
    cmd = ["srun", "--exact", "--kill-on-bad-exit=1", f"--nodes={len(hosts)}", f"--ntasks={len(hosts)}",
           "--ntasks-per-node=1", f"--nodelist={','.join(hosts)}"]
    if gpus_per_task:
        cmd.append(f"--gpus-per-task={gpus_per_task}")
    if cpus:
        cmd.append(f"--cpus-per-task={cpus}")
    if mem:
        cmd.append(f"--mem={mem}")
    return cmd


def _worker_config(cfg):
    """The role view of a config: no SLURM / multi-node sections (the roles run
    inside the allocation), output directory already prepared."""
    d = config_to_plain(cfg)
    d.pop("slurm", None)
    d["deployment"] = {"type": "single_node"}
    d["clean_output_dir"] = False
    return d


def plan_roles(cfg, command: str, hosts: list[str], config_dir: Path) -> list[RoleLaunch]:
    """Every role of the job with its command line (``srun`` placement) and
    environment; writes the role configs into ``config_dir``."""
    d, s = cfg.deployment, cfg.slurm
    py = shlex.split(s.python_command)
    need = d.num_train_nodes + d.num_inference_nodes
    if len(hosts) < need:
        raise RuntimeError(f"the allocation has {len(hosts)} node(s), the deployment needs {need}")
    train = hosts[:d.num_train_nodes]
    infer = hosts[d.num_train_nodes:need]
    base = _worker_config(cfg)
    env_base = {"WAVELET_SLURM_OUTPUT_PREPARED": "1"}
    torchrun = [*py, "-m", "torch.distributed.run", f"--nnodes={len(train)}", f"--nproc-per-node={d.gpus_per_node}",
                "--rdzv-backend=c10d", f"--rdzv-endpoint={train[0]}:{d.trainer_master_port}",
                f"--rdzv-id={s.job_name}"]
    if command == "sft":
        path = config_dir / "sft_worker.yaml"
        dump_yaml(path, base)
        return [RoleLaunch("sft_trainer", [*_srun(train, gpus_per_task=d.gpus_per_node), *torchrun, "-m",
                                           "wavelet_b200", "sft", "@", str(path)], dict(env_base))]
    roles: list[RoleLaunch] = []
    replica_hosts = [h for h in infer for _ in range(d.inference_replicas_per_node)]
    ports = [cfg.inference.http.port + i for i in range(len(replica_hosts))]
    per_replica = max(1, d.gpus_per_node // d.inference_replicas_per_node) if infer else 0
    for i, (h, port) in enumerate(zip(replica_hosts, ports)):
        rc = dict(base)
        rc["inference"] = {**base["inference"], "http": {**base["inference"]["http"], "host": "0.0.0.0",
                                                         "port": port, "hosts": None, "ports": None}}
        path = config_dir / f"inference_server_{i}.yaml"
        dump_yaml(path, rc)
        roles.append(RoleLaunch(f"inference_server_{i}",
                                [*_srun([h], gpus_per_task=per_replica, cpus=s.inference_cpus_per_replica,
                                        mem=s.inference_memory_per_replica),
                                 *py, "-m", "wavelet_b200", "inference-server", "@", str(path)],
                                {**env_base, **cfg.launcher.env_vars.for_role("inference")}, service=True,
                                endpoint=f"http://{h}:{port}"))
    wc = dict(base)
    pt = dict(base.get("policy_transfer") or {})
    if pt.get("type") == "nccl" and pt.get("nccl_host") in (None, "127.0.0.1", "localhost", "::1", "0.0.0.0"):
        pt["nccl_host"] = train[0]  # the trainer's rank 0 broadcasts
        wc["policy_transfer"] = pt
    tpath = config_dir / "rl_trainer.yaml"
    dump_yaml(tpath, wc)
    if cfg.max_steps != 0:
        roles.append(RoleLaunch("trainer", [*_srun(train, gpus_per_task=d.gpus_per_node), *torchrun, "-m",
                                            "wavelet_b200", "rl-trainer", "@", str(tpath)],
                                {**env_base, **cfg.launcher.env_vars.for_role("trainer")}))
    ic = dict(wc)
    if replica_hosts:
        ic["inference"] = {**base["inference"], "http": {**base["inference"]["http"], "hosts": replica_hosts,
                                                         "ports": ports, "port": ports[0]}}
    ipath = config_dir / "rl_inference.yaml"
    dump_yaml(ipath, ic)
    roles.append(RoleLaunch("rl_inference", [*py, "-m", "wavelet_b200", "rl-inference", "@", str(ipath)],
                            {**env_base, **cfg.launcher.env_vars.for_role("orchestrator"),
                             "CUDA_VISIBLE_DEVICES": ""}))
    return roles


def run_roles(roles: list[RoleLaunch], log_dir: Path, *, health: Callable[[list[str], float], None] | None = None,
              startup_timeout: float = 600.0, poll: float = 1.0) -> int:
    """Start the servers, wait for their health, start the jobs, supervise
    everything (see the module docstring); returns the exit code."""
    from ..orchestrator.launcher import RoleProcess, RoleSpec, wait_for_roles

    def start(r: RoleLaunch) -> RoleProcess:
        return RoleProcess(RoleSpec(r.name, r.argv, r.env, r.service), log_dir)

    services = [start(r) for r in roles if r.service]
    running: list = list(services)
    old = {}

    def _stop(signum, _frame):
        for p in running:
            p.terminate()
        raise SystemExit(128 + signum)

    for sig in (signal.SIGTERM, signal.SIGINT):
        try:
            old[sig] = signal.signal(sig, _stop)
        except ValueError:  # not the main thread
            pass
    try:
        urls = [r.endpoint for r in roles if r.service and r.endpoint]
        if urls:
            import time

            from ..inference.client import wait_healthy

            check = health or (lambda u, t: wait_healthy(u, t, poll=poll))
            deadline = time.monotonic() + startup_timeout
            while True:
                dead = [(p.spec.name, p.poll()) for p in services if p.poll() is not None]
                if dead:
                    for p in running:
                        p.terminate()
                    print(f"inference server exited before becoming healthy: {dead}", file=sys.stderr)
                    return 1
                try:
                    check(urls, min(poll * 5, max(0.0, deadline - time.monotonic())))
                    break
                except TimeoutError:
                    if time.monotonic() >= deadline:
                        for p in running:
                            p.terminate()
                        print(f"inference servers not healthy after {startup_timeout}s: {urls}", file=sys.stderr)
                        return 1
        jobs = [start(r) for r in roles if not r.service]
        running += jobs
        return wait_for_roles(jobs, services, poll)
    finally:
        for sig, h in old.items():
            signal.signal(sig, h)


def main(argv: list[str] | None = None) -> int:
    """``wavelet slurm-worker <command> <config args>``: the job controller."""
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in ("sft", "rl"):
        raise SystemExit("usage: wavelet slurm-worker {sft,rl} [config args]")
    command, rest = argv[0], argv[1:]
    from ..configs.config import RLConfig, SFTConfig
    from ..utils.config import load_config

    cfg = load_config(SFTConfig if command == "sft" else RLConfig, rest)
    hosts = expand_nodelist(os.environ.get("SLURM_JOB_NODELIST", "127.0.0.1"))
    out = Path(cfg.output_dir)
    pathing.validate_output_dir(out, clean=cfg.clean_output_dir,
                                resuming=cfg.ckpt is not None and cfg.ckpt.is_resuming,
                                protected_paths=(cfg.model.name, cfg.model.adapter_path))
    attempt = pathing.create_launch_attempt(out)
    roles = plan_roles(cfg, command, hosts, attempt.config_dir)
    print(f"SLURM placement: {', '.join(f'{r.name}' for r in roles)} on {hosts}; logs in {attempt.log_dir}",
          flush=True)
    timeout = cfg.inference.http.startup_timeout_seconds if command == "rl" else 0.0
    poll = cfg.launcher.poll_interval_seconds if command == "rl" else 1.0
    return run_roles(roles, attempt.log_dir, startup_timeout=timeout, poll=poll)


__all__ = ["render_sbatch", "launch_slurm", "expand_nodelist", "plan_roles", "run_roles", "RoleLaunch"]
