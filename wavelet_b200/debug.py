"""``wavelet debug``: cheap diagnostics that start no training.

Subcommands (reference debug.py:50-1800):

* ``preflight`` — validates an RL config without starting workers: output /
  data / adapter paths, device placement of the launcher mode, free ports,
  schedule math (target steps, policy lag, retained snapshots), algorithm
  and reward settings, and the B200 kernel constraints of the model
  (head_dim 128, NF4 column multiples, extension present).  Exit 1 on any
  error-level check.
* ``inference {inspect,health,smoke,benchmark,continuous-batch|batch}`` —
  engine/server configuration, HTTP health of every replica, a few probe
  generations, timed generation rounds, or many concurrent completion
  requests against the servers (latency percentiles, throughput, errors).
* ``orchestrator {inspect,sample,benchmark,materialize}`` — queue and policy
  state, the prompts a step would draw, one step's rollouts with per-phase
  timings, or the same published as a queue step.
* ``trainer {inspect,tokens,parity}`` — validate a rollout batch (row schema,
  token/mask/logprob alignment, advantages), dump per-token rows, or compare
  inference and trainer log-probs of its trainable tokens (a stored column,
  or ``--compute`` with the configured model).

All reports print as text, or as JSON with ``--json``.
"""

from __future__ import annotations

import argparse
import json
import socket
import sys
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Literal

from .configs.config import RLConfig

Status = Literal["ok", "warning", "error"]


@dataclass
class Check:
    name: str
    status: Status
    message: str


def _print(report: dict[str, Any], as_json: bool) -> None:
    if as_json:
        print(json.dumps(report, indent=2, default=str))
        return
    for k, v in report.items():
        if k == "checks":
            print("checks:")
            for c in v:
                print(f"  [{c['status']:7s}] {c['name']}: {c['message']}")
        else:
            print(f"{k}: {json.dumps(v, default=str) if isinstance(v, (dict, list)) else v}")


# ------------------------------------------------------------------ preflight
def _path_checks(cfg: RLConfig) -> list[Check]:
    from .utils import pathing

    out: list[Check] = []
    od = Path(cfg.output_dir)
    if pathing.has_run_state(od) and not cfg.clean_output_dir and (cfg.ckpt is None or cfg.ckpt.resume_step is None):
        out.append(Check("output_dir", "error", f"{od} holds run state; pass --clean-output-dir or resume"))
    else:
        out.append(Check("output_dir", "ok", str(od)))
    if cfg.data.source != "fake":
        paths = cfg.data.path if isinstance(cfg.data.path, list) else [cfg.data.path]
        missing = [str(p) for p in paths if not Path(p).exists()]
        out.append(Check("data_paths", "error" if missing else "ok", f"missing {missing}" if missing else "present"))
    if cfg.model.adapter_path is not None and not Path(cfg.model.adapter_path).exists():
        out.append(Check("adapter_path", "error", f"{cfg.model.adapter_path} does not exist"))
    return out


def _placement_checks(cfg: RLConfig) -> list[Check]:
    from .orchestrator.placement import plan, visible_devices

    if cfg.launcher.mode == "integrated":
        return [Check("placement", "ok", "integrated: one process per visible GPU")]
    try:
        p = plan(cfg, visible_devices())
        return [Check("placement", "ok", f"trainer {p.trainer_devices} inference {p.inference_devices}")]
    except ValueError as e:
        return [Check("placement", "error", str(e))]


def _port_checks(cfg: RLConfig) -> list[Check]:
    if cfg.launcher.mode == "integrated":
        return []
    h = cfg.inference.http
    ports = list(h.ports) if h.ports else [h.port + r for r in range(cfg.launcher.inference_num_replicas)]
    out = []
    for port in ports:
        s = socket.socket()
        try:
            s.bind((h.host if h.host not in ("0.0.0.0", "localhost") else "127.0.0.1", port))
            out.append(Check(f"port_{port}", "ok", "free"))
        except OSError:
            out.append(Check(f"port_{port}", "warning", "in use (fine if the server is already running)"))
        finally:
            s.close()
    return out


def _schedule_checks(cfg: RLConfig) -> list[Check]:
    from .orchestrator.schedule import max_policy_lag, retained_policy_snapshots, target_steps

    out = [Check("target_steps", "ok" if target_steps(cfg) > 0 else "error", str(target_steps(cfg)))]
    lag = max_policy_lag(cfg)
    keep = retained_policy_snapshots(cfg)
    if cfg.policy_transfer.keep_last < keep:
        out.append(Check("policy_retention", "warning",
                         f"policy_transfer.keep_last={cfg.policy_transfer.keep_last} < {keep} snapshots the lag can need"))
    out.append(Check("policy_lag", "ok", f"max lag {lag}, retain {keep} snapshots"))
    return out


def _algorithm_checks(cfg: RLConfig) -> list[Check]:
    o = cfg.orchestrator
    out = [Check("algorithm", "ok", cfg.algo.type if hasattr(cfg.algo, "type") else str(cfg.algo))]
    if getattr(cfg.algo, "type", None) == "grpo" and (o.rollouts_per_example or 1) < 2:
        out.append(Check("grpo_group", "error", "GRPO needs orchestrator.rollouts_per_example >= 2"))
    return out


def _model_checks(cfg: RLConfig) -> list[Check]:
    from .models.config import resolve_arch

    out = []
    try:
        arch = resolve_arch(cfg.model.name, cfg.model.arch_overrides or None)
    except Exception as e:  # unresolvable model name
        return [Check("model", "error", f"cannot resolve {cfg.model.name}: {e}")]
    out.append(Check("model", "ok", f"{arch.arch} L={arch.num_layers} H={arch.hidden_size} heads={arch.num_heads}/{arch.num_kv_heads}"))
    if arch.head_dim != 128:
        out.append(Check("attention_kernel", "warning", f"head_dim {arch.head_dim}: the tcgen05 attention kernels need 128 (CPU path only)"))
    if cfg.model.load_in_4bit:
        dims = {"hidden": arch.hidden_size, "q_dim": arch.q_dim, "intermediate": arch.intermediate_size}
        bad = {k: v for k, v in dims.items() if v % 64}
        out.append(Check("nf4_shapes", "error" if bad else "ok", f"NF4 needs multiples of 64: {bad or dims}"))
    try:
        from .ops import _ext

        out.append(Check("extension", "ok" if _ext.is_built() else "warning",
                         "built" if _ext.is_built() else "not built (first use compiles it)"))
    except Exception as e:
        out.append(Check("extension", "warning", str(e)))
    return out


def _environment_checks(cfg: RLConfig) -> list[Check]:
    """Every training / eval environment id resolves: a native one, or one
    the installed ``verifiers`` package would load."""
    from . import environments
    from .orchestrator.verifier_envs import verifiers_available

    o = cfg.orchestrator
    ids = [e.id for e in o.envs] or ([o.verifier_env_id] if o.verifier_env_id else [])
    ids += [e.id for e in (cfg.eval.env if cfg.eval is not None else [])
            if not e.id.startswith("file:") and e.resolved_name not in ("reverse", "reverse_match", "synthetic-reverse")]
    out = []
    have_vf = None
    for env_id in ids:
        if environments.is_native(env_id):
            out.append(Check(f"env:{env_id}", "ok", "native environment"))
            continue
        have_vf = verifiers_available() if have_vf is None else have_vf
        out.append(Check(f"env:{env_id}", "ok" if have_vf else "error",
                         "verifiers-package environment" if have_vf else "needs the verifiers package (not installed)"))
    return out


def _resolved_commands(cfg: RLConfig) -> list[dict[str, Any]]:
    """The processes a launch would start, with their GPUs and extra environment
    (role configs are rendered into a scratch directory, nothing is started)."""
    import tempfile

    if cfg.launcher.mode == "integrated":
        return [{"role": "rl", "argv": ["wavelet", "rl", "(integrated)"], "env": {}, "service": False}]
    from .orchestrator.launcher import build_roles
    from .utils import pathing

    with tempfile.TemporaryDirectory() as tmp:
        services, jobs = build_roles(cfg, pathing.create_launch_attempt(Path(tmp)))
    out = []
    for r in [*services, *jobs]:
        env = {k: ("<redacted>" if k in cfg.launcher.env_vars.for_role("common") or "KEY" in k or "TOKEN" in k else v)
               for k, v in r.env.items()}
        out.append({"role": r.name, "argv": [a if not a.startswith(tmp) else "<config>" for a in r.argv],
                    "env": env, "service": r.service})
    return out


def _paths(cfg: RLConfig) -> dict[str, str]:
    from .transport.queue import resolve_policy_dir, resolve_queue_dir

    od = Path(cfg.output_dir)
    return {"output_dir": str(od), "rollouts": str(resolve_queue_dir(od, cfg.transport)),
            "policies": str(resolve_policy_dir(od, cfg.policy_transfer)),
            "checkpoints": str(cfg.checkpoint_output_dir or od), "logs": str(od / "logs"),
            "evals": str(od / "evals")}


def build_preflight_report(cfg: RLConfig) -> dict[str, Any]:
    from .orchestrator.schedule import max_policy_lag, retained_policy_snapshots, target_steps

    checks = [*_path_checks(cfg), *_placement_checks(cfg), *_port_checks(cfg), *_schedule_checks(cfg),
              *_algorithm_checks(cfg), *_model_checks(cfg), *_environment_checks(cfg)]
    commands: list[dict[str, Any]] = []
    try:
        commands = _resolved_commands(cfg)
    except (ValueError, OSError) as e:
        checks.append(Check("resolved_commands", "error", str(e)))
    o = cfg.orchestrator
    return {
        "ok": not any(c.status == "error" for c in checks),
        "summary": {"model": cfg.model.name, "output_dir": str(cfg.output_dir), "launcher_mode": cfg.launcher.mode,
                    "inference_mode": cfg.inference.mode, "inference_backend": cfg.inference.vllm.server_backend,
                    "policy_transfer": cfg.policy_transfer.type, "target_steps": target_steps(cfg),
                    "max_policy_lag": max_policy_lag(cfg), "lora": cfg.lora is not None,
                    "policy_freshness": {"max_async_level": o.max_async_level,
                                         "max_off_policy_steps": o.max_off_policy_steps,
                                         "effective_max_policy_lag": max_policy_lag(cfg),
                                         "retained_policy_snapshots": retained_policy_snapshots(cfg)},
                    "algo": cfg.algo.model_dump(mode="json", exclude_none=True),
                    "training_envs": [e.model_dump(mode="json", exclude_none=True) for e in o.envs],
                    "curriculum": None if o.curriculum is None else o.curriculum.model_dump(mode="json",
                                                                                           exclude_none=True),
                    "low_precision": {"load_in_4bit": bool(cfg.model.load_in_4bit),
                                      "optimizer": cfg.optim.type if hasattr(cfg, "optim") else None}},
        "paths": _paths(cfg),
        "commands": commands,
        "checks": [asdict(c) for c in checks],
    }


def _preflight_main(argv: list[str]) -> int:
    from .utils.config import load_config

    p = argparse.ArgumentParser(prog="wavelet debug preflight")
    p.add_argument("--json", action="store_true")
    a, rest = p.parse_known_args(argv)
    report = build_preflight_report(load_config(RLConfig, rest))
    _print(report, a.json)
    return 0 if report["ok"] else 1


# ------------------------------------------------------------------ inference
def http_health(cfg: RLConfig) -> list[dict[str, Any]]:
    from .inference.client import endpoints, http_json

    out = []
    for u in endpoints(cfg):
        try:
            out.append({"url": u, "ok": True, "health": http_json(u + "/health", timeout=5.0)})
        except Exception as e:  # unreachable replica
            out.append({"url": u, "ok": False, "error": str(e)})
    return out


def _engine_and_orchestrator(cfg: RLConfig, engine=None):
    from .inference.policy import create_policy_inference_engine
    from .orchestrator.rollouts import RLOrchestrator
    from .orchestrator.runtime import build_prompt_source
    from .orchestrator.scheduler import _GeneratorAdapter

    if engine is None:
        engine = create_policy_inference_engine(cfg)
        engine.setup()
    return engine, RLOrchestrator(cfg, _GeneratorAdapter(engine), None, build_prompt_source(cfg, 1 << 30))


def _percentile(xs: list[float], q: float) -> float | None:
    if not xs:
        return None
    ys = sorted(xs)
    return ys[min(len(ys) - 1, max(0, int(round(q * (len(ys) - 1)))))]


def inference_benchmark(cfg: RLConfig, *, count: int, warmup: int, repeats: int, engine=None) -> dict[str, Any]:
    """Timed generations of ``count`` prompts (``repeats`` timed rounds after
    ``warmup`` untimed ones) through the configured engine."""
    import time

    engine, orch = _engine_and_orchestrator(cfg, engine)
    prompts = orch.prompts.take(count)
    for _ in range(warmup):
        orch.generate_records(prompts, 0)
    rounds = []
    for i in range(repeats):
        t0 = time.perf_counter()
        recs = orch.generate_records(prompts, i)
        dt = time.perf_counter() - t0
        ntok = sum(len((r.metadata or {}).get("completion_ids") or []) for r in recs)
        rounds.append({"seconds": dt, "completions": len(recs), "completion_tokens": ntok,
                       "tokens_per_second": ntok / max(dt, 1e-9)})
    tps = [r["tokens_per_second"] for r in rounds]
    return {"prompts": count, "warmup": warmup, "repeats": repeats, "rounds": rounds,
            "tokens_per_second": {"mean": sum(tps) / len(tps), "min": min(tps), "max": max(tps)}}


def continuous_batch_probe(cfg: RLConfig, *, count: int, concurrency: int, max_completion_tokens: int,
                           stagger_ms: float = 0.0, post=None) -> dict[str, Any]:
    """``count`` completion requests kept ``concurrency`` in flight against the
    HTTP inference replicas (round robin, optionally staggered): latency
    percentiles, throughput and errors of the servers' continuous batching."""
    import time
    from concurrent.futures import ThreadPoolExecutor

    from .inference.client import endpoints, http_json

    urls = endpoints(cfg)
    post = post or (lambda url, payload: http_json(url + "/v1/completions", payload,
                                                    timeout=cfg.inference.http.request_timeout_seconds))
    prompt_len = max(1, cfg.data.fake_prompt_len or 8)
    t_start = time.perf_counter()

    def one(i: int) -> dict[str, Any]:
        delay = t_start + i * stagger_ms / 1000.0 - time.perf_counter()
        if delay > 0:
            time.sleep(delay)
        url = urls[i % len(urls)]
        t0 = time.perf_counter()
        try:
            r = post(url, {"prompt_token_ids": [[3 + (i + j) % 50 for j in range(prompt_len)]],
                           "max_tokens": max_completion_tokens, "n": 1,
                           "temperature": cfg.inference.sampling.temperature})
            toks = sum(len(c.get("token_ids") or []) for c in r.get("choices", []))
            return {"index": i, "url": url, "seconds": time.perf_counter() - t0, "tokens": toks, "error": None}
        except Exception as e:  # reported per request
            return {"index": i, "url": url, "seconds": time.perf_counter() - t0, "tokens": 0, "error": str(e)}

    with ThreadPoolExecutor(max_workers=concurrency) as pool:
        reqs = list(pool.map(one, range(count)))
    wall = time.perf_counter() - t_start
    lat = [r["seconds"] for r in reqs if r["error"] is None]
    toks = sum(r["tokens"] for r in reqs)
    return {"metrics": {"requests": count, "concurrency": concurrency, "errors": sum(r["error"] is not None for r in reqs),
                        "wall_seconds": wall, "tokens": toks, "tokens_per_second": toks / max(wall, 1e-9),
                        "latency_p50": _percentile(lat, 0.5), "latency_p95": _percentile(lat, 0.95),
                        "latency_max": max(lat) if lat else None},
            "sample": reqs[:5], "errors": [r for r in reqs if r["error"] is not None][:5]}


def _inference_main(argv: list[str]) -> int:
    from .utils.config import load_config

    p = argparse.ArgumentParser(prog="wavelet debug inference",
                                description="Inspect and probe RL inference without trainer / orchestrator.")
    p.add_argument("action", choices=("inspect", "health", "smoke", "benchmark", "continuous-batch", "batch"))
    p.add_argument("--json", action="store_true")
    p.add_argument("--prompts", "--count", dest="count", type=int, default=4)
    p.add_argument("--warmup", type=int, default=0)
    p.add_argument("--repeats", type=int, default=1)
    p.add_argument("--concurrency", type=int, default=8)
    p.add_argument("--stagger-ms", type=float, default=0.0)
    p.add_argument("--max-completion-tokens", type=int, default=128)
    a, rest = p.parse_known_args(argv)
    for name, lo in (("count", 1), ("warmup", 0), ("repeats", 1), ("concurrency", 1), ("stagger_ms", 0),
                     ("max_completion_tokens", 1)):
        if getattr(a, name) < lo:
            raise SystemExit(f"--{name.replace('_', '-')} must be >= {lo}")
    cfg = load_config(RLConfig, rest)
    if a.action == "inspect":
        _print({"mode": cfg.inference.mode, "sampling": cfg.inference.sampling.model_dump(),
                "http": cfg.inference.http.model_dump(mode="json")}, a.json)
        return 0
    if a.action == "health":
        rows = http_health(cfg)
        _print({"health": rows}, a.json)
        return 0 if all(r["ok"] for r in rows) else 1
    if a.action in ("continuous-batch", "batch"):
        rep = continuous_batch_probe(cfg, count=a.count, concurrency=a.concurrency,
                                     max_completion_tokens=a.max_completion_tokens, stagger_ms=a.stagger_ms)
        _print(rep, a.json)
        return 0 if rep["metrics"]["errors"] == 0 else 1
    if a.action == "benchmark":
        _print(inference_benchmark(cfg, count=a.count, warmup=a.warmup, repeats=a.repeats), a.json)
        return 0
    eng, orch = _engine_and_orchestrator(cfg)
    recs = orch.generate_records(orch.prompts.take(a.count), 0)
    _print({"records": len(recs), "stats": orch.last_stats,
            "completion_tokens": [len((r.metadata or {}).get("completion_ids") or []) for r in recs]}, a.json)
    return 0


# -------------------------------------------------------------- orchestrator
def probe_orchestrator(cfg: RLConfig, *, step: int = 0, engine=None, write: bool = False) -> dict[str, Any]:
    """One step's rollouts end to end (prompt draw, generation, rewards,
    advantages, zero-advantage filter) with per-phase timings; ``write``
    publishes them as queue step ``step`` (the ``materialize`` action)."""
    import time

    from .data.rl import example_to_payload
    from .transport.queue import FileSystemRolloutSender

    timings: dict[str, float] = {}
    t0 = time.perf_counter()
    engine, orch = _engine_and_orchestrator(cfg, engine)
    timings["setup"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    recs = orch.materialize(step)
    timings["materialize"] = time.perf_counter() - t0
    out = None
    if write:
        t0 = time.perf_counter()
        rows = [example_to_payload(r) for r in recs]
        orch.write_materialized(rows, step)  # orchestrator.materialize_path, when set
        batch = FileSystemRolloutSender(Path(cfg.output_dir), cfg.transport).publish(
            rows, step=step, training_records=rows, optimizer_step=step,
            tokens=sum(len(r.input_ids or []) for r in recs), reward_mean=orch.last_stats.get("reward/mean"))
        out = str(batch.path)
        timings["write"] = time.perf_counter() - t0
    timings["total"] = sum(timings.values())
    return {"step": step, "records_trainable": len(recs), "examples_per_step": cfg.orchestrator.examples_per_step,
            "rollouts_per_example": cfg.orchestrator.rollouts_per_example, "timings": timings,
            "metrics": orch.last_stats, "output_path": out,
            "sample": [{"reward": r.reward, "advantage": r.advantage, "tokens": len(r.input_ids or [])}
                       for r in recs[:8]]}


def _orchestrator_main(argv: list[str]) -> int:
    from .transport.queue import resolve_policy_dir, resolve_queue_dir, scan_queue, stable_steps
    from .utils.config import load_config

    p = argparse.ArgumentParser(prog="wavelet debug orchestrator",
                                description="Inspect and benchmark RL orchestration without trainer.")
    p.add_argument("action", choices=("inspect", "sample", "benchmark", "materialize"))
    p.add_argument("--step", type=int, default=0)
    p.add_argument("--examples", type=int, default=None)
    p.add_argument("--rollouts", type=int, default=None)
    p.add_argument("--json", action="store_true")
    a, rest = p.parse_known_args(argv)
    if a.examples is not None and a.examples < 1:
        raise SystemExit("--examples must be >= 1")
    if a.rollouts is not None and a.rollouts < 1:
        raise SystemExit("--rollouts must be >= 1")
    cfg = load_config(RLConfig, rest)
    upd = {k: v for k, v in (("examples_per_step", a.examples), ("rollouts_per_example", a.rollouts)) if v}
    if upd:
        cfg = cfg.model_copy(update={"orchestrator": cfg.orchestrator.model_copy(update=upd)})
    out = Path(cfg.output_dir)
    if a.action == "inspect":
        _print({"queue": scan_queue(resolve_queue_dir(out, cfg.transport)),
                "policies": stable_steps(resolve_policy_dir(out, cfg.policy_transfer))}, a.json)
        return 0
    if a.action == "sample":
        from .orchestrator.runtime import build_prompt_source

        src = build_prompt_source(cfg, 1 << 30)
        prompts = src.take(cfg.orchestrator.examples_per_step or 1)
        _print({"step": a.step, "prompts": [{"example_id": p_.example_id, "tokens": len(p_.prompt_ids),
                                             "metadata": p_.metadata} for p_ in prompts]}, a.json)
        return 0
    _print(probe_orchestrator(cfg, step=a.step, write=a.action == "materialize"), a.json)
    return 0


# ------------------------------------------------------------------- trainer
def _records_file(path: Path) -> Path:
    from .transport.queue import TRAIN_SUFFIX

    path = Path(path)
    if path.is_file():
        return path
    side = sorted(path.glob(f"*{TRAIN_SUFFIX}"))
    return side[0] if side else path / "rollouts.jsonl"


def _resolve_batch(cfg: RLConfig | None, batch: Path | None, queue_step: int | None) -> Path:
    if batch is not None:
        return _records_file(batch)
    if cfg is None or queue_step is None:
        raise SystemExit("give a rollout batch path, or --queue-step with a config")
    from .transport.queue import resolve_queue_dir, step_dir

    return _records_file(step_dir(resolve_queue_dir(Path(cfg.output_dir), cfg.transport), queue_step))


def inspect_rollout_batch(path: Path) -> dict[str, Any]:
    """Schema and alignment checks of a rollout batch's training rows."""
    from .data.rl import example_from_payload
    from .transport.queue import read_training_records

    rows = read_training_records(_records_file(path))
    issues = []
    tokens = 0
    for i, row in enumerate(rows):
        try:
            r = example_from_payload(row)
        except Exception as e:  # malformed row
            issues.append({"row": i, "issue": f"unparseable: {e}"})
            continue
        ids, mask = r.input_ids or [], r.loss_mask or []
        tokens += len(ids)
        if len(ids) != len(mask):
            issues.append({"row": i, "issue": f"input_ids {len(ids)} vs loss_mask {len(mask)}"})
        lp = r.inference_logprobs
        if lp is not None and len(lp) not in (len(ids), sum(bool(m) for m in mask)):
            issues.append({"row": i, "issue": f"inference_logprobs length {len(lp)} matches neither tokens nor trainable tokens"})
        if r.advantage is None:
            issues.append({"row": i, "issue": "missing advantage"})
    return {"rows": len(rows), "tokens": tokens, "issues": issues, "ok": not issues}


def trainer_logprobs_of_rows(cfg: RLConfig, rows: list[dict[str, Any]], model=None) -> list[list[float]]:
    """Trainer log-probs (one per trainable token) of rollout rows under the
    configured model at the sampling temperature: the trainer's own LM-head
    path, no gradient."""
    import torch

    from .data.rl import example_from_payload, make_rank_batches
    from .models.config import resolve_arch
    from .models.qwen import build_model
    from .ops import lm_head

    if model is None:
        model = build_model(resolve_arch(cfg.model.name, cfg.model.arch_overrides or None),
                            "cuda" if torch.cuda.is_available() else "cpu", None, seed=cfg.seed, with_grad=False,
                            with_optimizer=False)
        p = Path(cfg.model.name)
        if not cfg.model.random_init and p.is_dir() and any(p.glob("*.safetensors")):
            from .models.hf_io import load_hf_weights

            load_hf_weights(model, p)
    temp = cfg.inference.sampling.temperature or cfg.inference.default_temperature
    out = []
    with torch.no_grad():
        for row in rows:
            ex = example_from_payload(row)
            (b,) = make_rank_batches([ex], max(cfg.data.seq_len, len(ex.input_ids or [])), 0, 1, temp)
            b = b.to(model.device)
            ctx = model.batch_ctx(b.base.position_ids, b.base.cu_seqlens, b.base.max_seqlen)
            h = model.hidden(b.base.input_ids, ctx)
            tgt = b.base.targets.clamp_min(0)
            if h.is_cuda:
                lp, _ = lm_head.logprob_entropy(h, model.head_weight(), tgt, b.temperature, want_entropy=False)
            else:
                lp, _ = lm_head.ref.logprob_entropy(model.logits(h), tgt, b.temperature)
            out.append(lp[b.loss_mask].float().cpu().tolist())
    return out


def runtime_parity_report(path: Path, *, trainer_column: str = "trainer_logprobs", threshold: float = 1e-3,
                          max_rows: int | None = None, computed: list[list[float]] | None = None) -> dict[str, Any]:
    """Inference vs trainer log-probs of the trainable tokens of a rollout
    batch: max / mean absolute difference, rows without either side, and
    alignment errors; passed when every compared token is within
    ``threshold``.  The trainer side is the ``trainer_column`` of the rows or,
    with ``computed``, log-probs the trainer computed for them."""
    from .transport.queue import read_training_records

    rows = read_training_records(path)
    if max_rows is not None:
        rows = rows[:max_rows]
    errors, miss_inf, miss_tr = [], 0, 0
    n_tok, max_d, sum_d = 0, 0.0, 0.0
    for i, row in enumerate(rows):
        k = sum(bool(m) for m in row.get("loss_mask") or [])
        inf = row.get("inference_logprobs")
        tr = computed[i] if computed is not None else row.get(trainer_column)
        if inf is None:
            miss_inf += 1
            continue
        if tr is None:
            miss_tr += 1
            continue
        if len(inf) != k:
            errors.append({"row": i, "field": "inference_logprobs", "message": "logprob count must match trainable token count"})
            continue
        if len(tr) != k:
            errors.append({"row": i, "field": trainer_column, "message": "trainer logprob count must match trainable token count"})
            continue
        for x, y in zip(inf, tr):
            d = abs(float(x) - float(y))
            max_d = max(max_d, d)
            sum_d += d
            n_tok += 1
    skip = None
    if n_tok == 0 and not errors:
        skip = ("no rows" if not rows else "no inference log-probs" if miss_inf == len(rows)
                else "no trainer log-probs" if miss_tr else "no trainable tokens")
    return {"path": str(path), "threshold": threshold, "rows_checked": len(rows), "token_count": n_tok,
            "max_abs_diff": max_d if n_tok else None, "mean_abs_diff": sum_d / n_tok if n_tok else None,
            "passed": bool(n_tok and max_d <= threshold and not errors), "skipped": n_tok == 0 and not errors,
            "skip_reason": skip, "coverage": {"rows_missing_inference_logprobs": miss_inf,
                                              "rows_missing_trainer_logprobs": miss_tr},
            "errors": errors}


def _trainer_main(argv: list[str]) -> int:
    from .utils.config import load_config

    p = argparse.ArgumentParser(prog="wavelet debug trainer",
                                description="Inspect trainer inputs and replay artifacts without training.")
    p.add_argument("action", choices=("inspect", "tokens", "parity"))
    p.add_argument("batch", type=Path, nargs="?", default=None,
                   help="rollout step directory (or its training-records file)")
    p.add_argument("--queue-step", type=int, default=None)
    p.add_argument("--json", action="store_true")
    p.add_argument("--limit", "--max-rows", dest="limit", type=int, default=None)
    p.add_argument("--trainer-logprobs-column", default="trainer_logprobs")
    p.add_argument("--threshold", type=float, default=1e-3)
    p.add_argument("--compute", action="store_true",
                   help="parity: compute the trainer log-probs with the configured model instead of reading a column")
    p.add_argument("--write-report", type=Path, default=None)
    p.add_argument("--write-tokens", type=Path, default=None)
    a, rest = p.parse_known_args(argv)
    if a.limit is not None and a.limit < 1:
        raise SystemExit("--max-rows must be >= 1")
    if a.threshold < 0:
        raise SystemExit("--threshold must be >= 0")
    cfg = load_config(RLConfig, rest) if (rest or a.compute or a.queue_step is not None) else None
    path = _resolve_batch(cfg, a.batch, a.queue_step)
    if a.action == "inspect":
        rep = inspect_rollout_batch(path)
        code = 0 if rep["ok"] else 1
    elif a.action == "parity":
        computed = None
        if a.compute:
            from .transport.queue import read_training_records

            rows = read_training_records(path)[: a.limit] if a.limit else read_training_records(path)
            computed = trainer_logprobs_of_rows(cfg, rows)
        rep = runtime_parity_report(path, trainer_column=a.trainer_logprobs_column, threshold=a.threshold,
                                    max_rows=a.limit, computed=computed)
        code = 0 if (rep["passed"] or rep["skipped"]) else 1
    else:
        from .data.rl import example_from_payload
        from .transport.queue import read_training_records

        rows = [example_from_payload(r) for r in read_training_records(path)][: a.limit or 2]
        rep = {"rows": []}
        for r in rows:
            lp = r.inference_logprobs or []
            k = 0
            toks = []
            for i, (t, m) in enumerate(zip(r.input_ids or [], r.loss_mask or [])):
                toks.append({"pos": i, "token": t, "trainable": bool(m),
                             "logprob": (lp[k] if m and k < len(lp) else None)})
                k += bool(m)
            rep["rows"].append(toks)
        if a.write_tokens is not None:
            a.write_tokens.parent.mkdir(parents=True, exist_ok=True)
            a.write_tokens.write_text("\n".join(json.dumps(x) for x in rep["rows"]) + "\n")
            rep = {"rows": len(rep["rows"]), "written": str(a.write_tokens)}
        code = 0
    if a.write_report is not None:
        a.write_report.parent.mkdir(parents=True, exist_ok=True)
        a.write_report.write_text(json.dumps(rep, indent=2, sort_keys=True, default=str))
    _print(rep, a.json or a.action == "tokens")
    return code


COMMANDS = {"preflight": (_preflight_main, "Validate cheap RL launch prerequisites"),
            "inference": (_inference_main, "Inspect and probe RL inference"),
            "orchestrator": (_orchestrator_main, "Inspect queue state or sample a rollout batch"),
            "trainer": (_trainer_main, "Inspect trainer inputs")}


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in COMMANDS:
        print("Usage: wavelet debug <subcommand> [args]\nSubcommands:")
        for k, (_, d) in COMMANDS.items():
            print(f"  {k:<14} {d}")
        return 1
    return COMMANDS[argv[0]][0](argv[1:])


if __name__ == "__main__":
    sys.exit(main())
