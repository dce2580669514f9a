"""Process-mode RL launcher: role processes under one supervisor.

Order (orchestrator/runtime.py:465-657 and launcher.py:18-348 of the
reference): write role configs into ``configs/attempt_<n>/resolved/``, start
the inference server(s) (one per replica, pinned with CUDA_VISIBLE_DEVICES),
wait for ``/health``, optionally put them to sleep (colocate_sleep), then
start the trainer (``torchrun ... -m wavelet_b200 rl-trainer``) and the
rollout role (``rl-inference``).  ``wait_for_roles`` polls every role; when
any exits non-zero all others are terminated and the run fails; SIGTERM is
forwarded to the children.
"""

from __future__ import annotations

import os
import signal
import subprocess
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

from ..utils import pathing
from ..utils.config import config_to_plain, dump_yaml
from .placement import plan


@dataclass
class RoleSpec:
    name: str
    argv: list[str]
    env: dict[str, str] = field(default_factory=dict)
    service: bool = False  # long-running server (terminated when jobs finish)


class RoleProcess:
    def __init__(self, spec: RoleSpec, log_dir: Path):
        self.spec = spec
        log_dir.mkdir(parents=True, exist_ok=True)
        self.log = open(log_dir / f"{spec.name}.log", "ab")
        env = {**os.environ, **spec.env}
        self.p = subprocess.Popen(spec.argv, env=env, stdout=self.log, stderr=subprocess.STDOUT,
                                  start_new_session=True)

    def poll(self):
        return self.p.poll()

    def terminate(self, grace: float = 10.0):
        if self.p.poll() is not None:
            return
        try:
            os.killpg(self.p.pid, signal.SIGTERM)
        except ProcessLookupError:
            return
        t0 = time.monotonic()
        while self.p.poll() is None and time.monotonic() - t0 < grace:
            time.sleep(0.1)
        if self.p.poll() is None:
            try:
                os.killpg(self.p.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass


def _run_role_subprocess(argv: list[str], env: dict[str, str], log_path: str, cwd: str) -> int:
    """Body of a Ray task: run one role as a child process group with its log
    file; a cancelled task (KeyboardInterrupt inside the worker) stops the
    whole group before returning."""
    Path(log_path).parent.mkdir(parents=True, exist_ok=True)
    with open(log_path, "ab") as log:
        p = subprocess.Popen(argv, env={**os.environ, **env}, stdout=log, stderr=subprocess.STDOUT, cwd=cwd,
                             start_new_session=True)
        try:
            return p.wait()
        except KeyboardInterrupt:
            try:
                os.killpg(p.pid, signal.SIGTERM)
                p.wait(timeout=10)
            except Exception:
                try:
                    os.killpg(p.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
            return 130


class RayRoleProcess:
    """A role running as a Ray task (``launcher.backend: ray``): the same
    ``poll`` / ``terminate`` surface as ``RoleProcess``, so the supervisor and
    its failure handling are shared (reference orchestrator/launcher.py:200-262)."""

    def __init__(self, spec: RoleSpec, log_dir: Path, ray_module, remote_fn):
        self.spec = spec
        self.ray = ray_module
        self.log_path = log_dir / f"{spec.name}.log"
        self.ref = remote_fn.remote(spec.argv, dict(spec.env), str(self.log_path), str(Path.cwd()))
        self._code = None

    def poll(self):
        if self._code is not None:
            return self._code
        ready, _ = self.ray.wait([self.ref], timeout=0)
        if not ready:
            return None
        self._code = int(self.ray.get(self.ref))
        return self._code

    def terminate(self, grace: float = 10.0):
        if self.poll() is not None:
            return
        self.ray.cancel(self.ref, force=False)  # interrupts the task, which stops its process group
        ready, _ = self.ray.wait([self.ref], timeout=grace)
        if not ready:
            self.ray.cancel(self.ref, force=True)


class RoleRunner:
    """Starts roles locally (``launcher.backend: local``) or as Ray tasks."""

    def __init__(self, cfg, log_dir: Path):
        self.log_dir = log_dir
        self.backend = getattr(cfg.launcher, "backend", "local")
        self.ray = None
        if self.backend == "ray":
            try:
                import ray
            except ImportError as exc:
                raise ImportError("launcher.backend='ray' requires the ray package; install it or use "
                                  "launcher.backend='local'") from exc
            self.ray = ray
            self.remote = ray.remote(_run_role_subprocess)
            ray.init(address=cfg.launcher.ray_address, runtime_env=cfg.launcher.ray_runtime_env,
                     ignore_reinit_error=True)

    def start(self, spec: RoleSpec):
        if self.ray is not None:
            return RayRoleProcess(spec, self.log_dir, self.ray, self.remote)
        return RoleProcess(spec, self.log_dir)

    def close(self) -> None:
        if self.ray is not None:
            self.ray.shutdown()


def wait_for_roles(jobs: list[RoleProcess], services: list[RoleProcess], poll: float = 1.0) -> int:
    """Return 0 when every job exits 0; tear everything down on the first failure."""
    try:
        while True:
            codes = [j.poll() for j in jobs]
            failed = [(j.spec.name, c) for j, c in zip(jobs, codes) if c not in (None, 0)]
            dead_services = [(s.spec.name, s.poll()) for s in services if s.poll() is not None]
            if failed or dead_services:
                for r in jobs + services:
                    r.terminate()
                print(f"role failure: {failed or dead_services}", file=sys.stderr)
                return 1
            if all(c == 0 for c in codes):
                return 0
            time.sleep(poll)
    finally:
        for s in services:
            s.terminate()


def build_roles(cfg, attempt: pathing.LaunchAttempt, python: str = sys.executable,
                shared_wandb: dict[str, str] | None = None) -> tuple[list[RoleSpec], list[RoleSpec]]:
    pl = plan(cfg)
    base = config_to_plain(cfg)
    device_transfer = cfg.policy_transfer.type == "nccl" and cfg.inference.mode == "vllm_http"
    if device_transfer:
        # one generator process per replica receives the device policy updates
        base["policy_transfer"] = {**base["policy_transfer"], "nccl_inference_world_size": len(pl.ports)}
    every = list(dict.fromkeys(pl.trainer_devices + [d for g in pl.inference_devices for d in g]))

    def visible(own: list[str]) -> dict[str, str]:
        """The role's own GPUs first (its cuda:0..); with device policy
        transfer every other GPU of the placement stays visible too, because
        a CUDA IPC handle only opens in a process that sees the GPU holding
        the memory."""
        if not own:
            return {}
        devs = own + [d for d in every if d not in own] if device_transfer and cfg.policy_transfer.peer else own
        return {"CUDA_VISIBLE_DEVICES": ",".join(devs)}

    services: list[RoleSpec] = []
    tp = cfg.inference.vllm.tensor_parallel_size
    if cfg.inference.mode == "vllm_http":
        for r, (devs, port) in enumerate(zip(pl.inference_devices, pl.ports)):
            c = dict(base)
            c["inference"] = {**base["inference"], "http": {**base["inference"]["http"], "port": port, "ports": None}}
            path = attempt.config_dir / f"inference_server_{r}.yaml"
            dump_yaml(path, c)
            argv = [python, "-m", "wavelet_b200", "inference-server", "@", str(path)]
            if tp > 1:  # one replica = a torchrun group of tp processes (inference.tp_server)
                if devs and len(devs) != tp:
                    raise ValueError(f"inference replica {r} has {len(devs)} GPUs for tensor_parallel_size {tp}")
                argv = [python, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
                        "--master-addr=127.0.0.1", f"--master-port={cfg.deployment.trainer_master_port + 101 + r}",
                        "-m", "wavelet_b200", "inference-server", "@", str(path)]
            services.append(RoleSpec(f"inference-server-{r}", argv,
                                     {**visible(devs), "WAVELET_INFERENCE_REPLICA": str(r)}, service=True))
    trainer_cfg = attempt.config_dir / "rl_trainer.yaml"
    dump_yaml(trainer_cfg, base)
    n = len(pl.trainer_devices) or cfg.launcher.trainer_num_processes
    port = cfg.deployment.trainer_master_port
    trainer_argv = ([python, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                     "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "wavelet_b200", "rl-trainer", "@", str(trainer_cfg)]
                    if n > 1 else [python, "-m", "wavelet_b200", "rl-trainer", "@", str(trainer_cfg)])
    env_t = visible(pl.trainer_devices)
    env_t.update(cfg.launcher.env_vars.for_role("trainer"))
    inf_cfg = dict(base)
    inf_cfg["inference"] = {**base["inference"], "http": {**base["inference"]["http"], "ports": pl.ports,
                                                          "port": pl.ports[0]}}
    inf_path = attempt.config_dir / "rl_inference.yaml"
    dump_yaml(inf_path, inf_cfg)
    env_i = cfg.launcher.env_vars.for_role("orchestrator")
    jobs = [RoleSpec("rl-trainer", trainer_argv, env_t),
            RoleSpec("rl-inference", [python, "-m", "wavelet_b200", "rl-inference", "@", str(inf_path)], env_i)]
    for s in services:
        s.env.update(cfg.launcher.env_vars.for_role("inference"))
    if shared_wandb:  # every role logs into one W&B run, labelled by its role
        env_t.update(shared_wandb, WANDB_SHARED_LABEL="trainer")
        env_i.update(shared_wandb, WANDB_SHARED_LABEL="orchestrator")
    return services, jobs


def run_process_launcher(cfg, argv: list[str]) -> int:
    out = Path(cfg.output_dir)
    pathing.validate_output_dir(out, clean=cfg.clean_output_dir, resuming=cfg.ckpt is not None and cfg.ckpt.is_resuming,
                                protected_paths=(cfg.model.name, cfg.model.adapter_path))
    attempt = pathing.create_launch_attempt(out)
    pathing.write_launch_artifacts(attempt, command="rl", argv=argv)
    dump_yaml(attempt.config_dir / "rl.yaml", config_to_plain(cfg))
    from ..monitor import finish_shared_wandb_run, shared_wandb_environment

    shared = shared_wandb_environment(cfg)
    services, jobs = build_roles(cfg, attempt, shared_wandb=shared)
    runner = RoleRunner(cfg, attempt.log_dir)
    running_services = [runner.start(s) for s in services]
    if running_services:
        from ..inference.client import endpoints, wait_healthy

        try:
            wait_healthy(endpoints(cfg), cfg.inference.http.startup_timeout_seconds,
                         probe_timeout=cfg.inference.http.liveness_timeout_seconds)
        except TimeoutError:
            for s in running_services:
                s.terminate()
            raise
    running_jobs = [runner.start(j) for j in jobs]

    def _sigterm(*_):
        raise KeyboardInterrupt

    signal.signal(signal.SIGTERM, _sigterm)
    rc = 1
    try:
        rc = wait_for_roles(running_jobs, running_services, cfg.launcher.poll_interval_seconds)
        return rc
    except KeyboardInterrupt:
        for r in running_jobs + running_services:
            r.terminate()
        rc = 130
        return rc
    finally:
        runner.close()
        finish_shared_wandb_run(cfg, shared, exit_code=rc)
