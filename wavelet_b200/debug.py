"""``wavelet debug``: cheap diagnostics that start no training.

Subcommands (reference debug.py:50-1800):

* ``preflight`` — validates an RL config without starting workers: output /
  data / adapter paths, device placement of the launcher mode, free ports,
  schedule math (target steps, policy lag, retained snapshots), algorithm
  and reward settings, and the B200 kernel constraints of the model
  (head_dim 128, NF4 column multiples, extension present).  Exit 1 on any
  error-level check.
* ``inference {inspect,health,smoke}`` — engine/server configuration, HTTP
  health of every replica, or a few probe generations with a summary.
* ``orchestrator {inspect,sample}`` — queue and policy-directory state, or
  one materialised (not published) rollout batch.
* ``trainer {inspect,tokens}`` — validate a published rollout batch (row
  schema, token/mask/logprob alignment, advantages) or dump per-token rows.

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


def build_preflight_report(cfg: RLConfig) -> dict[str, Any]:
    from .orchestrator.schedule import max_policy_lag, target_steps

    checks = [*_path_checks(cfg), *_placement_checks(cfg), *_port_checks(cfg), *_schedule_checks(cfg),
              *_algorithm_checks(cfg), *_model_checks(cfg)]
    return {
        "ok": not any(c.status == "error" for c in checks),
        "summary": {"model": cfg.model.name, "output_dir": str(cfg.output_dir), "launcher_mode": cfg.launcher.mode,
                    "policy_transfer": cfg.policy_transfer.type, "target_steps": target_steps(cfg),
                    "max_policy_lag": max_policy_lag(cfg), "lora": cfg.lora is not None},
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


def _inference_main(argv: list[str]) -> int:
    from .utils.config import load_config

    p = argparse.ArgumentParser(prog="wavelet debug inference")
    p.add_argument("action", choices=("inspect", "health", "smoke"))
    p.add_argument("--json", action="store_true")
    p.add_argument("--prompts", type=int, default=2)
    a, rest = p.parse_known_args(argv)
    cfg = load_config(RLConfig, rest)
    if a.action == "inspect":
        _print({"mode": cfg.inference.mode, "sampling": cfg.inference.sampling.model_dump(),
                "http": cfg.inference.http.model_dump(mode="json")}, a.json)
        return 0
    if a.action == "health":
        rows = http_health(cfg)
        _print({"health": rows}, a.json)
        return 0 if all(r["ok"] for r in rows) else 1
    from .inference.policy import create_policy_inference_engine
    from .orchestrator.rollouts import RLOrchestrator
    from .orchestrator.runtime import build_prompt_source
    from .orchestrator.scheduler import _GeneratorAdapter

    eng = create_policy_inference_engine(cfg)
    eng.setup()
    orch = RLOrchestrator(cfg, _GeneratorAdapter(eng), None, build_prompt_source(cfg, 1 << 30))
    recs = orch.generate_records(orch.prompts.take(a.prompts), 0)
    _print({"records": len(recs), "stats": orch.last_stats,
            "completion_tokens": [len((r.metadata or {}).get("completion_ids") or []) for r in recs]}, a.json)
    return 0


# -------------------------------------------------------------- orchestrator
def _orchestrator_main(argv: list[str]) -> int:
    from .transport.queue import resolve_policy_dir, resolve_queue_dir, scan_queue, stable_steps
    from .utils.config import load_config

    p = argparse.ArgumentParser(prog="wavelet debug orchestrator")
    p.add_argument("action", choices=("inspect", "sample"))
    p.add_argument("--json", action="store_true")
    a, rest = p.parse_known_args(argv)
    cfg = load_config(RLConfig, rest)
    out = Path(cfg.output_dir)
    if a.action == "inspect":
        _print({"queue": scan_queue(resolve_queue_dir(out, cfg.transport)),
                "policies": stable_steps(resolve_policy_dir(out, cfg.policy_transfer))}, a.json)
        return 0
    from .inference.policy import create_policy_inference_engine
    from .orchestrator.rollouts import RLOrchestrator
    from .orchestrator.runtime import build_prompt_source
    from .orchestrator.scheduler import _GeneratorAdapter

    eng = create_policy_inference_engine(cfg)
    eng.setup()
    orch = RLOrchestrator(cfg, _GeneratorAdapter(eng), None, build_prompt_source(cfg, 1 << 30))
    recs = orch.materialize(0)
    _print({"records": len(recs), "stats": orch.last_stats,
            "sample": [{"reward": r.reward, "advantage": r.advantage, "tokens": len(r.input_ids or [])}
                       for r in recs[:8]]}, a.json)
    return 0


# ------------------------------------------------------------------- trainer
def _records_file(path: Path) -> Path:
    from .transport.queue import TRAIN_SUFFIX

    path = Path(path)
    if path.is_file():
        return path
    side = sorted(path.glob(f"*{TRAIN_SUFFIX}"))
    return side[0] if side else path / "rollouts.jsonl"


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


def _trainer_main(argv: list[str]) -> int:
    p = argparse.ArgumentParser(prog="wavelet debug trainer")
    p.add_argument("action", choices=("inspect", "tokens"))
    p.add_argument("batch", type=Path, help="rollout step directory (or its training-records file)")
    p.add_argument("--json", action="store_true")
    p.add_argument("--limit", type=int, default=2)
    a = p.parse_args(argv)
    if a.action == "inspect":
        rep = inspect_rollout_batch(a.batch)
        _print(rep, a.json)
        return 0 if rep["ok"] else 1
    from .data.rl import example_from_payload
    from .transport.queue import read_training_records

    rows = [example_from_payload(r) for r in read_training_records(_records_file(a.batch))][: a.limit]
    out = []
    for r in rows:
        lp = r.inference_logprobs or []
        out.append([{"pos": i, "token": t, "trainable": bool(m), "logprob": lp[i] if i < len(lp) else None}
                    for i, (t, m) in enumerate(zip(r.input_ids or [], r.loss_mask or []))])
    _print({"rows": out}, True)
    return 0


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
