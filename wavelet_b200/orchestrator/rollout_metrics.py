"""Per-step rollout metrics of a published batch (ref monitor.py:849-1280).

Computed from the batch's records (``RLExample`` payloads) with the metric
names the reference publishes, so dashboards and W&B panels built for one
framework read the other's runs:

* ``progress/{tokens,prefill_tokens,decode_tokens,samples,problems}`` and the
  step counters ``progress/{ckpt_step,queue_step,optimizer_step}``,
  ``policy/step`` and ``policy/lag``;
* ``off_policy/{mean,max}``: optimizer steps between each rollout's policy and
  the step that trains on it;
* per-example series (one value per prompt group, the mean over its
  rollouts) summarised as ``<name>/<cohort>/{mean,max,std,min}``:
  ``seq_len``, ``decode_len``, ``prefill_len``, ``reward``, ``num_turns``,
  ``is_truncated`` and ``advantage`` (per rollout);
* ``solve_none`` / ``solve_all`` / ``effective_batch_size`` per cohort: the
  share of groups whose rollouts all scored 0, all scored full marks (reward
  sum reaching the group size), and the rest;
* ``stop_condition/<cohort>/<condition>`` rates and
  ``stop_condition/<cohort>/generation_truncated``;
* per environment ``batch/<env>`` and ``train/<env>/{batch_fraction,
  group_fraction, reward/*, advantage/*, solve_none, solve_all,
  effective_batch_size}``;
* ``fate/all/{trainable,filtered,errored}`` counts from the orchestrator's
  step statistics.

The cohort of the whole batch is ``all``.  A record that continues a
multi-row rollout (``metadata.rollout_count`` 0) adds tokens but not another
sample.
"""

from __future__ import annotations

from collections import defaultdict
from statistics import mean, pstdev
from typing import Any, Callable, Iterable


def series_stats(prefix: str, values: Iterable[float], include_min: bool = True) -> dict[str, float]:
    v = [float(x) for x in values]
    if not v:
        return {}
    out = {f"{prefix}/mean": mean(v), f"{prefix}/max": max(v), f"{prefix}/std": pstdev(v) if len(v) > 1 else 0.0}
    if include_min:
        out[f"{prefix}/min"] = min(v)
    return out


def _md(r: dict[str, Any]) -> dict[str, Any]:
    m = r.get("metadata")
    return m if isinstance(m, dict) else {}


def _num(v: Any) -> float | None:
    return float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else None


def _samples(r: dict[str, Any]) -> int:
    c = _md(r).get("rollout_count", 1)
    return int(c) if isinstance(c, (int, float)) else 1


def _seq_len(r: dict[str, Any]) -> int:
    ids = r.get("input_ids")
    return len(ids) if isinstance(ids, list) else _decode_len(r)


def _decode_len(r: dict[str, Any]) -> int:
    mask = r.get("loss_mask")
    if isinstance(mask, list):
        return sum(bool(x) for x in mask)
    lps = r.get("inference_logprobs")
    if isinstance(lps, list):
        return len(lps)
    n = _md(r).get("completion_token_count")
    return int(n) if isinstance(n, (int, float)) else 0


def _turns(r: dict[str, Any]) -> int:
    n = _md(r).get("turn_count")
    if isinstance(n, (int, float)):
        return int(n)
    return len(r.get("completion") or []) or 1


def _env(r: dict[str, Any]) -> str:
    return str(_md(r).get("env") or r.get("source") or "all")


def _groups(rows: list[dict[str, Any]]) -> dict[tuple[str, str], list[dict[str, Any]]]:
    g: dict[tuple[str, str], list[dict[str, Any]]] = defaultdict(list)
    for i, r in enumerate(rows):
        md = _md(r)
        key = md.get("group")
        key = str(key) if key is not None else str(md.get("example_id", f"row{i}"))
        g[(_env(r), key)].append(r)
    return dict(g)


def _group_means(groups, fn: Callable[[dict[str, Any]], float | None], weighted: bool = False) -> list[float]:
    out = []
    for rows in groups.values():
        vals = [(v, _samples(r) if weighted else 1) for r in rows if (v := fn(r)) is not None]
        w = sum(x for _, x in vals)
        if w > 0:
            out.append(sum(v * x for v, x in vals) / w)
    return out


def _solve_rates(groups, group_size: int) -> tuple[float, float, float]:
    if not groups:
        return 0.0, 0.0, 0.0
    none = full = 0
    for rows in groups.values():
        total = sum((_num(r.get("reward")) or 0.0) * _samples(r) for r in rows)
        size = _md(rows[0]).get("group_size") or group_size
        none += total == 0.0
        full += total >= size
    n = len(groups)
    return none / n, full / n, 1.0 - none / n - full / n


def _cohort(out: dict[str, float], rows: list[dict[str, Any]], groups, suffix: str, group_size: int) -> None:
    for name, fn in (("seq_len", _seq_len), ("decode_len", _decode_len)):
        out.update(series_stats(f"{name}/{suffix}", _group_means(groups, fn)))
    out.update(series_stats(f"reward/{suffix}", _group_means(groups, lambda r: _num(r.get("reward")), True)))
    sn, sa, eff = _solve_rates(groups, group_size)
    out.update({f"solve_none/{suffix}": sn, f"solve_all/{suffix}": sa, f"effective_batch_size/{suffix}": eff})
    conds = [_md(r).get("stop_condition") or _md(r).get("finish_reason") for r in rows]
    trunc = [bool(_md(r).get("is_truncated")) and c != "prompt_too_long" for r, c in zip(rows, conds)]
    out[f"stop_condition/{suffix}/generation_truncated"] = sum(trunc) / len(trunc) if trunc else 0.0
    seen = [str(c) for c in conds if c is not None]
    for c in sorted(set(seen)):
        out[f"stop_condition/{suffix}/{c}"] = seen.count(c) / len(seen)


def rollout_metrics(rows: list[dict[str, Any]], *, step: int, group_size: int, policy_step: int | None = None,
                    queue_step: int | None = None, optimizer_step: int | None = None,
                    stats: dict[str, float] | None = None) -> dict[str, float]:
    """Metrics of one published batch (``rows``: the records as published)."""
    groups = _groups(rows)
    seq = [_seq_len(r) for r in rows]
    dec = [_decode_len(r) for r in rows]
    opt = optimizer_step if optimizer_step is not None else step
    out: dict[str, float] = {
        "progress/tokens": float(sum(seq)), "progress/decode_tokens": float(sum(dec)),
        "progress/prefill_tokens": float(sum(max(s - d, 0) for s, d in zip(seq, dec))),
        "progress/samples": float(sum(_samples(r) for r in rows)), "progress/problems": float(len(groups)),
        "progress/ckpt_step": float(policy_step if policy_step is not None else step),
        "progress/queue_step": float(queue_step if queue_step is not None else step),
        "progress/optimizer_step": float(opt),
    }
    if policy_step is not None:
        out["policy/step"] = float(policy_step)
        out["policy/lag"] = float(opt - policy_step)
    lags = [max(0, opt - int(p)) for r in rows if _samples(r) > 0
            and isinstance(p := _md(r).get("policy_step"), int) and not isinstance(p, bool)]
    if lags:
        out["off_policy/mean"] = float(mean(lags))
        out["off_policy/max"] = float(max(lags))
    for name, fn, with_min in (("prefill_len", lambda r: max(_seq_len(r) - _decode_len(r), 0), True),
                               ("is_truncated", lambda r: float(bool(_md(r).get("is_truncated"))), False),
                               ("num_turns", _turns, True)):
        out.update(series_stats(f"{name}/all", _group_means(groups, fn), include_min=with_min))
    out.update(series_stats("advantage/all", [a for r in rows if (a := _num(r.get("advantage"))) is not None]))
    _cohort(out, rows, groups, "all", group_size)
    by_env: dict[str, list[dict[str, Any]]] = defaultdict(list)
    for r in rows:
        by_env[_env(r)].append(r)
    if len(by_env) > 1 or "all" not in by_env:
        for env, env_rows in sorted(by_env.items()):
            eg = _groups(env_rows)
            frac = len(env_rows) / max(len(rows), 1)
            out[f"batch/{env}"] = frac
            _cohort(out, env_rows, eg, env, group_size)
            p = f"train/{env}"
            out[f"{p}/batch_fraction"] = frac
            out[f"{p}/group_fraction"] = len(eg) / max(len(groups), 1)
            out.update(series_stats(f"{p}/reward", _group_means(eg, lambda r: _num(r.get("reward")), True)))
            out.update(series_stats(f"{p}/advantage",
                                    [a for r in env_rows if (a := _num(r.get("advantage"))) is not None]))
            sn, sa, eff = _solve_rates(eg, group_size)
            out.update({f"{p}/solve_none": sn, f"{p}/solve_all": sa, f"{p}/effective_batch_size": eff})
    st = stats or {}
    out["fate/all/trainable"] = float(sum(_samples(r) for r in rows))
    out["fate/all/filtered"] = float(st.get("rollout/zero_advantage_dropped", 0.0))
    out["fate/all/errored"] = float(st.get("verifier/failures/total", 0.0))
    return out
