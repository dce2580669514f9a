"""Evaluation runs over configured environments (``eval.env``).

Built-in environments (no network, no external verifier package):

* ``reverse`` — synthetic reverse-the-prompt task (``args``: ``prompt_len``,
  ``vocab``, ``seed``), reward = fraction of generated tokens matching the
  reversed prompt;
* ``file:<path>`` — prompt rows from a local JSONL/Parquet file scored by the
  configured reward (``reference_match`` / ``math_format`` against ``answer``);
* the native environments of ``wavelet_b200.environments``
  (``equation_builder``, ``polaris_math_tagged``; ``args`` are their
  ``load_environment`` arguments), scored by their own reward on the
  evaluation split.

For every example ``rollouts_per_example`` samples are drawn; the metrics are
the mean reward, pass@1 and pass@k (unbiased estimator of Chen et al. 2021,
"Evaluating Large Language Models Trained on Code") with success = reward >=
``args.success_threshold`` (default 1.0).  Results go to
``eval_metrics.jsonl`` and ``evals/<env>/step-<n>.jsonl`` (reference
orchestrator/eval_utils.py and entrypoints/rl_evals.py).
"""

from __future__ import annotations

import json
import math
import shutil
from dataclasses import replace
from pathlib import Path
from types import SimpleNamespace
from typing import Any

from ..monitor import append_jsonl, utc_now
from .reward import RLRewardScorer
from .rollouts import RLOrchestrator, SyntheticReversePrompts


def pass_at_k(n: int, c: int, k: int) -> float:
    if n - c < k:
        return 1.0
    return 1.0 - math.prod(1.0 - k / i for i in range(n - c + 1, n + 1))


def pass_hat_k(n: int, c: int, k: int) -> float:
    """pass^k: probability that k draws without replacement all succeed."""
    return math.comb(c, k) / math.comb(n, k) if k <= n else 0.0


def group_metrics(prefix: str, by_example: dict[str, list[float | None]], threshold: float = 1.0) -> dict[str, float]:
    """avg@n, pass@k and pass^k for k = 1, 2, 4, ... <= n (averaged over
    examples), reward mean and failed (reward-less) rollouts, as the
    reference reports them (orchestrator/eval_utils.py)."""
    groups = list(by_example.values())
    n = min((len(v) for v in groups), default=0)
    rewards = [float(x) for v in groups for x in v if x is not None]
    m = {f"{prefix}/num_examples": float(len(groups)),
         f"{prefix}/failed_rollouts": float(sum(x is None for v in groups for x in v)),
         f"{prefix}/reward_mean": sum(rewards) / max(1, len(rewards))}
    if n == 0:
        return m
    m[f"{prefix}/avg@{n}"] = sum(float(x or 0.0) for v in groups for x in v[:n]) / (n * len(groups))
    k = 1
    while k <= n:
        succ = [sum(x is not None and float(x) >= threshold for x in v[:n]) for v in groups]
        m[f"{prefix}/pass@{k}"] = sum(pass_at_k(n, c, k) for c in succ) / len(groups)
        m[f"{prefix}/pass^{k}"] = sum(pass_hat_k(n, c, k) for c in succ) / len(groups)
        k *= 2
    return m


def prune_eval_sets(env_dir: Path, keep: int | None) -> list[Path]:
    """Keep the newest ``keep`` rollout files (``step-<n>.jsonl``) of one
    environment's eval directory (``eval.keep_last_rollout_sets``)."""
    if keep is None or not env_dir.is_dir():
        return []
    sets = []
    for f in env_dir.glob("step-*.jsonl"):
        try:
            sets.append((int(f.stem.split("-", 1)[1]), f))
        except ValueError:
            continue
    removed = [f for _, f in sorted(sets)[:-keep]] if keep > 0 else [f for _, f in sets]
    for f in removed:
        f.unlink()
        j = env_dir / f"journal-{f.stem}"  # the evaluation journal of that step
        if j.is_dir():
            shutil.rmtree(j)
    return removed


def _native(env_id: str) -> bool:
    from .. import environments

    return environments.is_native(env_id)


def _env_prompts(cfg, env):
    a = env.args or {}
    if env.id.startswith("file:"):
        from .sources import FilePromptSource

        data = cfg.data.model_copy(update={"path": Path(env.id[5:]), "shuffle": False})
        return FilePromptSource(SimpleNamespace(data=data, model=cfg.model))
    if env.resolved_name in ("reverse", "reverse_match", "synthetic-reverse"):
        vocab = int(a.get("vocab", cfg.data.fake_vocab_size))
        return SyntheticReversePrompts(vocab, int(a.get("prompt_len", cfg.data.fake_prompt_len)), seed=int(a.get("seed", 12345)))
    from .. import environments

    if environments.is_native(env.id):
        from .reward import register_environment
        from .sources import EnvironmentPromptSource

        e = environments.load_environment(env.id, **{k: v for k, v in a.items() if k not in ("success_threshold",)})
        register_environment(e)
        return EnvironmentPromptSource([(e, 1.0)], cfg.model.name, seed=int(a.get("seed", 0)),
                                       split="eval" if e.eval_examples else "train", model_cfg=cfg.model)
    raise ValueError(f"unknown eval environment {env.id!r} (built-ins: reverse, file:<path>, "
                     f"{', '.join(environments.available())}; other ids need the verifiers package, "
                     f"which is not installed)")


def _builtin(env) -> bool:
    return env.id.startswith("file:") or env.resolved_name in ("reverse", "reverse_match", "synthetic-reverse") \
        or _native(env.id)


def run_eval_env(cfg, engine, env, step: int, out_dir: Path, cancel=None) -> dict[str, float] | None:
    """Metrics of one eval environment at ``step``; None when ``cancel`` (a
    ``threading.Event``) was set before the evaluation finished."""
    if cancel is not None and cancel.is_set():
        return None
    if not _builtin(env):
        from .verifier_envs import evaluate, verifiers_available

        if verifiers_available():  # a verifiers-package environment rolls out against the inference servers
            return evaluate(cfg, env, step=step, out_dir=out_dir, engine=engine, cancel=cancel)
    if cfg.eval is None or not cfg.eval.resume:
        return _run_native_eval(cfg, engine, env, step, out_dir)
    # eval.resume: a finished evaluation of this step with the same settings is not run again
    from .eval_journal import EvalJournal, signature

    sig = signature(env_id=env.id, env_args=env.args, samples=env.rollouts_per_example, num_examples=env.num_examples,
                    sampling=env.sampling.model_dump(mode="json"), reward=cfg.reward.model_dump(mode="json"),
                    model_config=cfg.model.model_dump(mode="json"), policy_step=step)
    with EvalJournal(Path(out_dir) / "evals" / env.resolved_name / f"journal-step-{step}", sig=sig,
                     resume=True) as journal:
        done = journal.completed("metrics")
        if done is not None:
            return {k: float(v) for k, v in done.items() if k != "reward"}
        m = _run_native_eval(cfg, engine, env, step, out_dir)
        journal.record("metrics", {**m, "reward": m.get(f"eval/{env.resolved_name}/reward_mean", 0.0)})
    return m


def _run_native_eval(cfg, engine, env, step: int, out_dir: Path) -> dict[str, float]:
    n_ex = env.num_examples if env.num_examples > 0 else 32
    k = env.rollouts_per_example
    reward_cfg = cfg.reward
    if env.resolved_name in ("reverse", "reverse_match", "synthetic-reverse"):
        reward_cfg = cfg.reward.model_copy(update={"mode": "reverse_match"})
    elif _native(env.id):
        reward_cfg = cfg.reward.model_copy(update={"mode": "environment"})
    ecfg = cfg.model_copy(update={"reward": reward_cfg,
                                  "orchestrator": cfg.orchestrator.model_copy(update={
                                      "rollouts_per_example": k,
                                      "live_traces": bool(cfg.eval.live_traces if cfg.eval is not None else True)})})
    s = env.sampling
    if s.max_completion_tokens or s.temperature is not None:
        samp = cfg.inference.sampling.model_copy(update={
            kk: v for kk, v in (("max_completion_tokens", s.max_completion_tokens), ("temperature", s.temperature),
                                ("top_p", s.top_p), ("top_k", s.top_k)) if v is not None})
        ecfg = ecfg.model_copy(update={"inference": cfg.inference.model_copy(update={"sampling": samp})})
    orch = RLOrchestrator(ecfg, engine, None, _env_prompts(cfg, env))
    prompts = orch.prompts.take(n_ex)
    recs = orch.generate_records(prompts, step)
    scorer = RLRewardScorer(reward_cfg)
    recs = [replace(r, reward=scorer.score(r)) for r in recs]
    thr = float((env.args or {}).get("success_threshold", 1.0))
    by_ex: dict[str, list[float | None]] = {}
    for r in recs:
        by_ex.setdefault(str((r.metadata or {}).get("example_id")), []).append(r.reward)
    m = group_metrics(f"eval/{env.resolved_name}", by_ex, thr)
    if k > 1 and f"eval/{env.resolved_name}/pass@{k}" not in m:  # a k that is not a power of two
        n = min(len(v) for v in by_ex.values())
        m[f"eval/{env.resolved_name}/pass@{k}"] = sum(
            pass_at_k(n, sum(x is not None and float(x) >= thr for x in v[:n]), min(k, n)) for v in by_ex.values()
        ) / max(1, len(by_ex))
    d = out_dir / "evals" / env.resolved_name
    d.mkdir(parents=True, exist_ok=True)
    with (d / f"step-{step}.jsonl").open("w") as f:
        for r in recs:
            md = r.metadata or {}
            f.write(json.dumps({"example_id": md.get("example_id"), "reward": r.reward,
                                "completion_ids": md.get("completion_ids")}) + "\n")
    prune_eval_sets(d, cfg.eval.keep_last_rollout_sets if cfg.eval is not None else None)
    return m


def run_evals(cfg, engine, step: int = 0, envs=None) -> dict[str, Any]:
    out = Path(cfg.output_dir)
    metrics: dict[str, Any] = {}
    for env in envs if envs is not None else cfg.eval.env:
        metrics.update(run_eval_env(cfg, engine, env, step, out))
    append_jsonl(out / "eval_metrics.jsonl", {"step": step, "timestamp": utc_now(), **metrics})
    return metrics
