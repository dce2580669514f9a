"""Rollout materialisation: prompts -> generations -> rewards -> advantages -> queue.

``RLOrchestrator.publish(step)`` (orchestrator/rollouts.py:43-525 of the
reference) selects the step's prompts, asks the inference engine for
``rollouts_per_example`` completions each (exact token ids + processed
log-probs + optional sampling masks), scores rewards, assigns advantages with
the configured algorithm, drops zero-advantage groups (optionally refilling
them up to ``zero_advantage_max_retries``), and publishes the batch to the
filesystem queue as ``RLExample`` training records.  A step holds
``examples_per_step`` prompt groups, or groups drawn until their rows hold
``token_batch_size`` tokens; with ``batch_selection: rollouts`` rollouts
count one by one instead of whole groups.
"""

from __future__ import annotations

import math
import random
import time
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from ..data.rl import RLExample, example_to_payload
from ..monitor import emit_perf
from ..transport.queue import FileSystemRolloutSender
from .algorithms import algorithm_epsilon, algorithm_scope, build_algorithm, score_records
from .reward import RLRewardScorer


@dataclass
class PromptRecord:
    prompt_ids: list[int]
    prompt: list[dict[str, str]] = field(default_factory=list)
    target_completion: list[dict[str, str]] | None = None
    metadata: dict[str, Any] = field(default_factory=dict)
    example_id: str = ""


class SyntheticReversePrompts:
    """The GRPO benchmark's data: uniform random prompts of ``prompt_len``
    tokens; the verifiable target is the reversed prompt."""

    def __init__(self, vocab: int, prompt_len: int, seed: int = 0, low: int = 3):
        self.vocab = vocab
        self.prompt_len = prompt_len
        self.rng = torch.Generator().manual_seed(seed)
        self.low = low
        self.cursor = 0

    def take(self, n: int) -> list[PromptRecord]:
        out = []
        for _ in range(n):
            ids = torch.randint(self.low, self.vocab, (self.prompt_len,), generator=self.rng).tolist()
            out.append(PromptRecord(ids, metadata={"task": "reverse"}, example_id=f"synthetic-{self.cursor}"))
            self.cursor += 1
        return out

    def state_dict(self) -> dict:
        return {"cursor": self.cursor, "rng": self.rng.get_state().tolist()}


class RLOrchestrator:
    def __init__(self, cfg, engine, sender: FileSystemRolloutSender | None, prompts, monitor=None,
                 custom_rollout: Callable | None = None):
        self.cfg = cfg
        self.engine = engine
        self.sender = sender
        self.prompts = prompts
        self.monitor = monitor
        self.algo = build_algorithm(cfg.algo)
        self.scope = algorithm_scope(cfg.algo)
        self.eps = algorithm_epsilon(cfg.algo)
        self.scorer = RLRewardScorer(cfg.reward)
        self.custom_rollout = custom_rollout
        self.last_stats: dict[str, float] = {}
        # orchestrator.envs[] entries with their own sampling / group size / algorithm
        self.env_cfg: dict[str, Any] = {}
        if getattr(getattr(cfg, "orchestrator", None), "envs", None):
            from .runtime import env_overrides

            self.env_cfg = env_overrides(cfg)
        self.env_algo = {n: (build_algorithm(e.algo), algorithm_scope(e.algo), algorithm_epsilon(e.algo))
                         for n, e in self.env_cfg.items() if e.algo is not None}
        # tokens per prompt group seen so far (token-sized steps); views of this
        # orchestrator share the one dict
        self._token_estimate = {"tokens": 0, "groups": 0}
        # prompts of verifiers-package environments are rolled out by the environments themselves
        vf_envs = {e.name: e for e, _ in getattr(prompts, "envs", [])
                   if getattr(e, "metadata", {}).get("kind") == "verifiers"}
        if vf_envs and self.custom_rollout is None:
            from .verifier_envs import VerifierRollouts

            self.custom_rollout = VerifierRollouts(cfg, vf_envs, engine, fallback=self.generate_records)
        # a user rollout function ("module.path:function") replaces generation and scoring
        fn_path = getattr(getattr(cfg, "orchestrator", None), "custom_rollout_function", None)
        if fn_path and self.custom_rollout is None and not cfg.orchestrator.uses_verifiers:
            from .custom_rollout import CustomRollout

            self.custom_rollout = CustomRollout(self, fn_path, engine)

    def _sampling(self):
        from ..inference.engine import SamplingParams

        s = self.cfg.inference.sampling
        return SamplingParams(
            temperature=s.temperature if s.do_sample else 0.0, top_p=s.top_p, top_k=s.top_k, min_p=s.min_p,
            max_tokens=s.max_completion_tokens or 256, min_tokens=s.min_tokens,
            n=self.cfg.orchestrator.rollouts_per_example or 1, seed=s.seed,
            return_sampling_mask=self.cfg.sampling_mask_required(),
        )

    def _live_episodes(self, prompts: list[PromptRecord], step: int) -> list:
        """One live trace document per prompt group while it is generated
        (orchestrator.live_traces; read by the dashboard's live view)."""
        o = getattr(self.cfg, "orchestrator", None)
        out_dir = getattr(self.cfg, "output_dir", None)
        if o is None or not getattr(o, "live_traces", False) or out_dir is None:
            return []
        from .live import LiveEpisode

        eps = []
        for p in prompts:
            ep = LiveEpisode(out_dir, str(p.metadata.get("task") or p.metadata.get("env") or "prompts"), "train",
                             step=step, example_id=p.example_id)
            ep.event("episode_started", prompt_tokens=len(p.prompt_ids))
            eps.append(ep)
        return eps

    def _env_params(self, env: str | None, base):
        """Sampling of one environment's prompts: the global settings with the
        entry's own ``sampling`` fields and ``group_size`` on top."""
        e = self.env_cfg.get(env) if env is not None else None
        if e is None:
            return base
        from dataclasses import replace as _replace

        p = _replace(base)
        if e.sampling is not None:
            s = e.sampling
            for k in s.model_fields_set:
                if k == "max_completion_tokens":
                    p.max_tokens = s.max_completion_tokens or p.max_tokens
                elif k == "do_sample":
                    continue
                elif hasattr(p, k):
                    setattr(p, k, getattr(s, k))
            if not s.do_sample:
                p.temperature = 0.0
        if e.group_size is not None:
            p.n = e.group_size
        return p

    def generate_records(self, prompts: list[PromptRecord], step: int) -> list[RLExample]:
        base = self._sampling()
        if base.seed is not None:
            base.seed = base.seed + step
        eps = self._live_episodes(prompts, step)
        t0 = time.perf_counter()
        keep = self.cfg.inference.sampling.max_prompt_tokens
        # prompts of environments with their own sampling run as their own batch
        batches: dict[Any, tuple[Any, list[int]]] = {}
        for i, p in enumerate(prompts):
            env = p.metadata.get("env")
            key = env if env in self.env_cfg else None
            if key not in batches:
                batches[key] = (self._env_params(key, base), [])
            batches[key][1].append(i)
        comps, temps = [], {}
        try:  # over-long prompts keep their last max_prompt_tokens tokens (as the reference fits them)
            for params, idx in batches.values():
                got = self.engine.generate([prompts[i].prompt_ids[-keep:] if keep else prompts[i].prompt_ids
                                            for i in idx], params)
                for c in got:
                    c.prompt_index = idx[c.prompt_index]
                    temps[c.prompt_index] = params.temperature
                comps += got
        except BaseException as e:
            for ep in eps:
                ep.finish("error", error=e)
            raise
        gen_s = time.perf_counter() - t0
        for i, ep in enumerate(eps):
            mine = [c for c in comps if c.prompt_index == i]
            ep.event("generation_finished", samples=len(mine), completion_tokens=[len(c.token_ids) for c in mine],
                     finish_reasons=[c.finish_reason for c in mine], seconds=gen_s)
            ep.finish("completed")
        recs = []
        for c in comps:
            p = prompts[c.prompt_index]
            ids = p.prompt_ids + c.token_ids
            mask = [False] * len(p.prompt_ids) + [True] * len(c.token_ids)
            md = dict(p.metadata)
            md.update(prompt_ids=p.prompt_ids, completion_ids=c.token_ids, finish_reason=c.finish_reason,
                      is_truncated=c.finish_reason == "length", completion_token_count=len(c.token_ids),
                      prompt_token_count=len(p.prompt_ids), input_token_count=len(p.prompt_ids), group=f"{step}:{c.prompt_index}",
                      sample_index=c.sample_index, example_id=p.example_id)
            recs.append(RLExample(prompt=p.prompt, completion=[], advantage=None, reward=None, input_ids=ids,
                                  loss_mask=mask, target_completion=p.target_completion,
                                  inference_logprobs=c.logprobs, temperatures=temps[c.prompt_index],
                                  sampling_mask=c.sampling_mask, metadata=md, source="orchestrator"))
        st = getattr(self.engine, "stats", {}) or {}
        ntok = sum(len(c.token_ids) for c in comps)
        self.last_stats = {"rollout/generate_seconds": gen_s, "rollout/generated_tokens": float(ntok),
                           "rollout/tokens_per_second": ntok / max(gen_s, 1e-9),
                           "rollout/samples": float(len(comps))}
        self.last_stats.update({f"inference/{k}": float(v) for k, v in st.items()})
        return recs

    def score(self, recs: list[RLExample]) -> list[RLExample]:
        from dataclasses import replace

        recs = [replace(r, reward=self.scorer.score(r)) for r in recs]
        group = lambda r: (r.metadata or {}).get("group")  # noqa: E731
        if not self.env_algo:
            return score_records(self.algo, recs, self.scope, group_key=group)
        # environments with their own algorithm score their records with it
        by_env: dict[Any, list[int]] = {}
        for i, r in enumerate(recs):
            env = (r.metadata or {}).get("env")
            by_env.setdefault(env if env in self.env_algo else None, []).append(i)
        out: list[RLExample | None] = [None] * len(recs)
        for env, idx in by_env.items():
            algo, scope, _ = self.env_algo[env] if env is not None else (self.algo, self.scope, self.eps)
            for i, r in zip(idx, score_records(algo, [recs[i] for i in idx], scope, group_key=group)):
                out[i] = r
        return out

    def _filter_zero(self, recs: list[RLExample]) -> tuple[list[RLExample], int]:
        if not self.cfg.orchestrator.filter_zero_advantage or self.scope == "rollout":
            return recs, 0
        if self.cfg.orchestrator.batch_selection == "rollouts":
            # rollouts count one by one: a zero-advantage rollout is left out on its own (its reward is
            # still in the step's metrics) unless a CE / ref-KL weight still trains it
            keep = [r for r in recs if abs(float(r.advantage or 0.0)) > 0.0 or _aux_weighted(r)]
            return keep, len(recs) - len(keep)
        groups: dict[Any, list[RLExample]] = {}
        for r in recs:
            groups.setdefault((r.metadata or {}).get("group"), []).append(r)
        keep, dropped = [], 0
        for g in groups.values():
            if all(abs(float(r.advantage or 0.0)) <= self.eps for r in g):
                dropped += len(g)
            else:
                keep += g
        return keep, dropped

    def _curriculum_gate(self, recs: list[RLExample]) -> tuple[list[RLExample], int]:
        """Report each scored group to the prompt source's curriculum (sampler
        EMA + gates) and keep the admitted groups."""
        cur = getattr(self.prompts, "curriculum", None)
        if cur is None:
            return recs, 0
        groups: dict[Any, list[RLExample]] = {}
        for r in recs:
            groups.setdefault((r.metadata or {}).get("group"), []).append(r)
        keep, rejected = [], 0
        for g in groups.values():
            key = (g[0].metadata or {}).get("task_key")
            if key is None:
                keep += g
                continue
            if cur.on_result(key, [{"reward": r.reward, "advantage": r.advantage} for r in g]):
                keep += g
            else:
                rejected += len(g)
        self.last_stats.update({f"curriculum/{k}": v for k, v in cur.metrics().items()})
        return keep, rejected

    def for_step(self, prompts) -> "RLOrchestrator":
        """A view of this orchestrator with its own prompt source and stats,
        for one step generated concurrently with others (the algorithm,
        scorer and engine are shared)."""
        view = type(self).__new__(type(self))
        view.__dict__.update(self.__dict__)
        view.prompts = prompts
        view.last_stats = {}
        return view

    def _rollout(self, prompts: list[PromptRecord], step: int) -> list[RLExample]:
        """Records of ``prompts``: the native generator, or the rollout function
        (verifiers-package environments, a user function); a function may
        return ``(records, statistics)``."""
        if self.custom_rollout is None:
            return self.generate_records(prompts, step)
        kw = {"fallback": self.generate_records} if getattr(self.custom_rollout, "takes_fallback", False) else {}
        out = self.custom_rollout(prompts, step, **kw)
        if isinstance(out, tuple):
            recs, stats = out
            self.last_stats.update(stats or {})
            return recs
        return out

    def _materialize_tokens(self, step: int) -> list[RLExample]:
        """A step sized by tokens (``orchestrator.token_batch_size``): prompt
        groups are drawn in rounds, each sized from the running tokens-per-group
        estimate (shared across steps), until the kept rows hold at least the
        target; the last round may overshoot by less than its groups' tokens
        (ref orchestrator/scheduler.py:553-560, 700-760)."""
        o = self.cfg.orchestrator
        target = int(o.token_batch_size)
        est = self._token_estimate
        kept: list[RLExample] = []
        scored: list[RLExample] = []
        tokens = dropped = gated = rounds = 0
        while tokens < target and rounds < 64:
            per_group = est["tokens"] / est["groups"] if est["groups"] else 0.0
            need = max(1, math.ceil((target - tokens) / per_group)) if per_group > 0 else 1
            recs = self.score(self._rollout(self.prompts.take(need), step))
            recs, g = self._curriculum_gate(recs)
            k, d = self._filter_zero(recs)
            scored += recs
            kept += k
            gated += g
            dropped += d
            n_tok = sum(len(r.input_ids or []) for r in recs)
            n_groups = len({(r.metadata or {}).get("group") for r in recs})
            est["tokens"] += n_tok
            est["groups"] += n_groups
            tokens += sum(len(r.input_ids or []) for r in k)
            rounds += 1
        if not kept:
            kept = scored
        from .teacher import attach_teacher_logprobs, scorer_for

        kept = attach_teacher_logprobs(kept, self.cfg, scorer_for(self.cfg, self.engine))
        rewards = [float(r.reward or 0.0) for r in scored]
        self.last_stats.update({"reward/mean": sum(rewards) / max(1, len(rewards)),
                                "rollout/curriculum_rejected": float(gated),
                                "rollout/zero_advantage_dropped": float(dropped),
                                "rollout/token_batch_tokens": float(tokens),
                                "rollout/token_batch_rounds": float(rounds)})
        return kept

    def materialize(self, step: int) -> list[RLExample]:
        o = self.cfg.orchestrator
        if getattr(o, "token_batch_size", None):
            return self._materialize_tokens(step)
        n_prompts = o.examples_per_step or 1
        # oversampling_factor: draw more groups than the step needs, keep the first usable ones
        prompts = self.prompts.take(max(n_prompts, math.ceil(n_prompts * float(getattr(o, "oversampling_factor", 1.0)))))
        recs = self.score(self._rollout(prompts, step))
        recs, gated = self._curriculum_gate(recs)
        kept, dropped = self._filter_zero(recs)
        retries = 0
        while (o.refill_zero_advantage and dropped and retries < o.zero_advantage_max_retries
               and len(kept) < len(recs)):
            need = max(1, dropped // max(1, o.rollouts_per_example or 1))
            more, _ = self._curriculum_gate(self.score(self._rollout(self.prompts.take(need), step)))
            more_kept, dropped = self._filter_zero(more)
            kept += more_kept
            retries += 1
        if not kept:
            kept = recs  # never publish an empty batch; zero-advantage rows contribute no gradient
        if o.batch_selection == "rollouts":
            kept = _trim_rollouts(kept, n_prompts * (o.rollouts_per_example or 1))
        elif len(prompts) > n_prompts:
            kept = _trim_groups(kept, n_prompts)
        from .teacher import attach_teacher_logprobs, scorer_for

        kept = attach_teacher_logprobs(kept, self.cfg, scorer_for(self.cfg, self.engine))  # OPD / OPSD
        rewards = [float(r.reward or 0.0) for r in recs]
        self.last_stats["rollout/curriculum_rejected"] = float(gated)
        self.last_stats.update({"reward/mean": sum(rewards) / max(1, len(rewards)),
                                "rollout/zero_advantage_dropped": float(dropped),
                                "rollout/zero_advantage_retries": float(retries)})
        return kept

    def reusable_batch(self, step: int) -> Any:
        """The stable queue batch of ``step`` when the trainer would still
        accept it (its policy is within the allowed lag), so a restarted
        producer does not generate it again (ref orchestrator/rollouts.py:306-334)."""
        if self.sender is None:
            return None
        batch = self.sender.stable_batch(step)
        if batch is None:
            return None
        from .schedule import required_policy_step

        man = batch.manifest
        ps = man.policy_step if man is not None else None
        if ps is not None and not required_policy_step(step, self.cfg) <= ps <= step:
            raise ValueError(f"rollout queue step {step} is stable but was generated with policy {ps}, outside the "
                             f"allowed range [{required_policy_step(step, self.cfg)}, {step}]; remove it or "
                             f"start from a fresh output directory")
        from ..transport.queue import append_event

        append_event(self.sender.output_dir / "events", "rollout_reused", queue_step=step, optimizer_step=step,
                     details={"path": str(batch.path)})
        return batch

    def write_materialized(self, rows: list[dict], step: int) -> Any:
        """``orchestrator.materialize_path``: the step's rows also as one JSONL
        file (an existing file is an error when ``orchestrator.overwrite`` is off)."""
        from pathlib import Path

        path = getattr(self.cfg.orchestrator, "materialize_path", None)
        if path is None:
            return None
        path = Path(path)
        if path.exists() and not self.cfg.orchestrator.overwrite:
            raise FileExistsError(f"Rollout file '{path}' already exists and overwrite is disabled.")
        path.parent.mkdir(parents=True, exist_ok=True)
        import json

        with path.open("w", encoding="utf-8") as f:
            for r in rows:
                f.write(json.dumps(r, separators=(",", ":"), default=str) + "\n")
        return path

    def publish(self, step: int, policy_step: int | None = None) -> Any:
        existing = self.reusable_batch(step)
        if existing is not None:
            return existing
        t0 = time.perf_counter()
        recs = self.materialize(step)
        emit_perf("rollout_materialized", step=step, seconds=time.perf_counter() - t0, rows=len(recs))
        rows = [example_to_payload(r, self.cfg.data) for r in recs]
        tokens = sum(len(r.input_ids or []) for r in recs)
        self.write_materialized(rows, step)
        if self.sender is None:
            return recs
        return self.sender.publish(rows, step=step, training_records=rows, optimizer_step=step, policy_step=policy_step,
                                   tokens=tokens, reward_mean=self.last_stats.get("reward/mean"))


def _aux_weighted(r: RLExample) -> bool:
    """True when a CE or reference-KL weight still trains the record."""
    for w in (r.ce_weight, r.ref_kl_weight):
        if isinstance(w, list) and any(x != 0.0 for x in w):
            return True
        if w is not None and not isinstance(w, list) and w != 0.0:
            return True
    return False


def _trim_rollouts(recs: list[RLExample], target: int) -> list[RLExample]:
    """The first ``target`` rollouts (every row of a multi-row rollout stays
    with it; ``metadata.rollout_count`` is 0 on a rollout's later rows)."""
    out, n = [], 0
    for r in recs:
        c = int((r.metadata or {}).get("rollout_count", 1))
        if c and n >= target:
            break
        out.append(r)
        n += c
    return out


def _trim_groups(recs: list[RLExample], n_groups: int) -> list[RLExample]:
    """The records of the first ``n_groups`` prompt groups, in order."""
    seen: set = set()
    out = []
    for r in recs:
        g = (r.metadata or {}).get("group")
        if g not in seen:
            if len(seen) >= n_groups:
                continue
            seen.add(g)
        out.append(r)
    return out
