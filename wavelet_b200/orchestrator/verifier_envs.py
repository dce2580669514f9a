"""Environments of the ``verifiers`` package (reference orchestrator/envs.py:69-1842).

A ``verifiers`` environment drives its own rollouts: it renders the prompt,
calls an OpenAI-compatible server (here the native inference server's chat
routes, which return the prompt and completion token ids with their
log-probs), runs its tools or user turns, and scores the result.  This module
is the bridge between those environments and the orchestrator:

* ``load_env``: ``verifiers.load_environment(id, **args)`` once per id,
  arguments and run settings (``max_seq_len``, ``max_total_completion_tokens``
  and ``timeout_seconds`` are handed to the environment with ``set_kwargs``).
* ``client_configs``: one ``verifiers.ClientConfig`` per server URL
  (``orchestrator.verifier_base_url``, else the configured inference servers).
* ``VerifierEnvironment``: an environment as a prompt source sees it (name,
  training and evaluation rows, chat prompt), so ``EnvironmentPromptSource``
  mixes verifier and native environments by ratio with resumable cursors.
* ``VerifierRollouts``: the orchestrator's rollout function for verifier
  prompts, with admission control (in-flight cap ``max_inflight_rollouts``,
  start rate ``tasks_per_minute``, and the adaptive cap of
  ``orchestrator.concurrency`` fed by the servers' load metrics).  Each prompt's group runs as ``rollouts_per_example`` (or the
  entry's ``group_size``) concurrent ``env.run_rollout`` calls, or one
  ``env.run_group`` for environments that score groups jointly; failed
  rollouts are dropped and counted by kind, a provider's rate-limit error
  stops the run.  Advantages are assigned per rollout within its group with
  the environment's algorithm, then every model call of a rollout becomes a
  token segment and ``agent_trajectory.merge_token_segments`` stitches them
  into training rows that share the rollout's reward and advantage.
* ``evaluate``: ``eval.env`` entries whose id is a verifier environment,
  over its evaluation rows, ``rollouts_per_example`` samples each (the seed
  offset per sample), with avg@n / pass@k metrics, the rollouts written to
  ``evals/<env>/step-<n>.jsonl`` and the metrics appended to
  ``eval_metrics.jsonl``.

In process mode the environments call the inference servers; in integrated
mode the runner serves its own generator on an in-process OpenAI server
(``inference.server.InProcessServer``) and points the clients at it.

The package is optional: nothing here imports it until an environment that
is not a native one is requested, and then a missing package is an error
that names it.
"""

from __future__ import annotations

import asyncio
import json
import logging
import math
import os
from collections import Counter
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from ..data.rl import RLExample
from .agent_trajectory import TokenSegment, merge_token_segments, to_rl_example

log = logging.getLogger("wavelet")

# markers of a reward provider's (judge model's) rate limit in an error text
_RATE_LIMIT_MARKERS = ("rate limit", "rate_limit", "ratelimit", "too many requests", "quota")
STATE_COLUMNS = ["trajectory", "sampling_args"]


def load_verifiers(feature: str = "environments"):
    """The ``verifiers`` module, or an ImportError that says what needs it."""
    try:
        import verifiers as vf
    except ImportError as exc:
        raise ImportError(f"verifier {feature} need the 'verifiers' package, which is not installed "
                          "(native environments need nothing)") from exc
    return vf


def verifiers_available() -> bool:
    try:
        load_verifiers()
    except ImportError:
        return False
    return True


# ----------------------------------------------------------------------------------------------------------------
# run settings -> environment and client settings
# ----------------------------------------------------------------------------------------------------------------


def base_urls(cfg) -> list[str]:
    """OpenAI base URLs the environments call: ``orchestrator.verifier_base_url``
    or every configured inference server."""
    urls = cfg.orchestrator.verifier_base_url
    if urls is None:
        http = cfg.inference.http
        return [f"http://{http.host}:{p}/v1" for p in (http.ports or [http.port])]
    return [urls] if isinstance(urls, str) else list(urls)


def model_name(cfg, engine: Any | None = None) -> str:
    """The model name sent with each request (the served policy's name when
    the engine reports one)."""
    name = getattr(engine, "policy_model_name", None)
    if isinstance(name, str) and name:
        return name
    return cfg.orchestrator.verifier_model or cfg.model.name


def env_kwargs(cfg) -> dict[str, Any]:
    """Run settings handed to every environment."""
    out: dict[str, Any] = {"max_seq_len": cfg.inference.vllm.max_model_len or cfg.data.seq_len,
                           "max_total_completion_tokens": cfg.orchestrator.verifier_max_total_completion_tokens}
    if cfg.orchestrator.verifier_timeout_seconds is not None:
        out["timeout_seconds"] = cfg.orchestrator.verifier_timeout_seconds
    return out


def client_configs(vf, cfg, *, urls: list[str] | None = None, client_type: str | None = None) -> list[Any]:
    """One client per server URL (a native inference server runs one engine;
    replicas are separate servers, so no data-parallel routing header is
    needed); groups are spread over them round robin."""
    key_var = cfg.orchestrator.verifier_api_key_var
    os.environ.setdefault(key_var, "EMPTY")  # local servers take any key
    routes = list(urls or base_urls(cfg))
    if not routes:
        raise ValueError("verifier environments need at least one server URL")
    return [vf.ClientConfig(client_idx=i, client_type=client_type or cfg.orchestrator.verifier_client_type,
                            api_base_url=u, api_key_var=key_var, extra_headers={})
            for i, u in enumerate(routes)]


_ENV_CACHE: dict[tuple, Any] = {}


def load_env(vf, env_id: str, args: dict[str, Any] | None, extra: dict[str, Any] | None = None) -> tuple[Any, bool]:
    """(environment, cache hit) for an id and its arguments."""
    args, extra = dict(args or {}), dict(extra or {})
    key = (env_id, json.dumps(args, sort_keys=True, default=str), json.dumps(extra, sort_keys=True, default=str))
    if key in _ENV_CACHE:
        return _ENV_CACHE[key], True
    env = vf.load_environment(env_id, **args)
    if extra:
        setter = getattr(env, "set_kwargs", None)
        if callable(setter):
            setter(**extra)
        else:
            for k, v in extra.items():
                setattr(env, k, v)
    _ENV_CACHE[key] = env
    return env, False


async def teardown_envs() -> None:
    """Close every cached environment once (``teardown`` may be async)."""
    envs = list({id(e): e for e in _ENV_CACHE.values()}.values())
    _ENV_CACHE.clear()
    errors = []
    for env in envs:
        fn = getattr(env, "teardown", None)
        if not callable(fn):
            continue
        try:
            res = fn()
            if asyncio.iscoroutine(res) or isinstance(res, asyncio.Future):
                await res
        except Exception as exc:  # noqa: BLE001 - every environment gets its teardown
            errors.append(exc)
    if errors:
        raise RuntimeError(f"{len(errors)} verifier environment teardown(s) failed") from errors[0]


def sampling_args(sampling, *, cache_salt: str | None = None) -> dict[str, Any]:
    """OpenAI request arguments of a sampling section; the server returns
    token ids and log-probs (``logprobs`` + ``extra_body.return_token_ids``)."""
    args: dict[str, Any] = {"temperature": sampling.temperature if sampling.do_sample else 0.0,
                            "top_p": sampling.top_p, "logprobs": True}
    if sampling.max_completion_tokens is not None:
        args["max_completion_tokens"] = sampling.max_completion_tokens
    extra: dict[str, Any] = dict(getattr(sampling, "extra_body", None) or {})
    extra["return_token_ids"] = True
    if cache_salt is not None:
        extra["cache_salt"] = cache_salt
    if sampling.top_k:
        extra["top_k"] = sampling.top_k
    extra["min_p"] = sampling.min_p
    if sampling.min_tokens > 0:
        extra["min_tokens"] = sampling.min_tokens
    if sampling.seed is not None:
        args["seed"] = sampling.seed
    args["extra_body"] = extra
    return args


def normalize_example(example: dict[str, Any]) -> dict[str, Any]:
    """A dataset row as a rollout input: a string ``task`` route moves into
    ``info.env_id``, as current ``verifiers`` expects."""
    out = dict(example)
    task = out.get("task")
    if isinstance(task, str):
        info = dict(out.get("info") or {}) if isinstance(out.get("info"), dict) else {}
        info.setdefault("env_id", task)
        out["info"] = info
        out.pop("task")
    return out


# ----------------------------------------------------------------------------------------------------------------
# results
# ----------------------------------------------------------------------------------------------------------------


@dataclass
class FailureStats:
    """Dropped rollouts by kind, reported (and reset) with each step's metrics."""
    counts: Counter = field(default_factory=Counter)

    def record(self, error: object) -> None:
        kind = type(error).__name__ if isinstance(error, BaseException) else str(error).split(":", 1)[0][:60]
        self.counts[kind or "Error"] += 1

    def consume(self) -> dict[str, float]:
        m = {f"verifier/failures/{k}": float(v) for k, v in self.counts.items()}
        m["verifier/failures/total"] = float(sum(self.counts.values()))
        self.counts.clear()
        return m


def _truncate(text: str, limit: int = 500) -> str:
    text = " ".join(str(text).split())
    return text if len(text) <= limit else text[: limit - 3] + "..."


def raise_if_rate_limited(error: Any) -> None:
    """A reward provider's rate limit is not a failed sample: it would fail
    every later rollout too, so it stops the run with a message."""
    low = str(error).lower()
    if any(m in low for m in _RATE_LIMIT_MARKERS) and ("429" in low or "limit" in low):
        raise RuntimeError("the verifier's reward provider is rate limited; retry after its limit resets or "
                           f"lower the judge concurrency. Original error: {_truncate(str(error))}")


def has_trainable_trajectory(output: dict[str, Any]) -> bool:
    for st in output.get("trajectory") or []:
        toks = st.get("tokens") if isinstance(st, dict) else None
        if isinstance(toks, dict) and any(bool(x) for x in (toks.get("completion_mask") or [])):
            return True
    return False


def successful_outputs(results: list[Any], failures: FailureStats | None = None,
                       require_trainable: bool = True) -> list[dict[str, Any]]:
    """The results that can be trained on: no exception, no ``error``, a
    reward, and (for training) at least one trained completion token."""
    out = []
    for res in results:
        why: object | None = None
        if isinstance(res, BaseException):
            raise_if_rate_limited(res)
            why = res
        else:
            try:
                o = dict(res)
            except (TypeError, ValueError):
                why = "InvalidResult"
            else:
                if o.get("error") is not None:
                    raise_if_rate_limited(o["error"])
                    why = o["error"] if isinstance(o["error"], BaseException) else f"{o['error']}"
                elif "reward" not in o or o["reward"] is None:
                    why = "MissingReward"
                elif require_trainable and not has_trainable_trajectory(o):
                    why = "UntrainableTrajectory"
        if why is not None:
            if failures is not None:
                failures.record(why)
            log.warning("verifier rollout dropped: %s", _truncate(str(why), 200))
            continue
        out.append(o)
    return out


def output_segments(output: dict[str, Any]) -> list[TokenSegment]:
    """One token segment per model call of a rollout."""
    segs = []
    for i, st in enumerate(output.get("trajectory") or []):
        toks = (st or {}).get("tokens") or {}
        comp = list(toks.get("completion_ids") or [])
        if not comp and not toks.get("prompt_ids"):
            continue
        lps = list(toks.get("completion_logprobs") or [0.0] * len(comp))
        mask = toks.get("completion_mask")
        segs.append(TokenSegment(list(toks.get("prompt_ids") or []), comp, lps,
                                 output_loss_mask=[bool(m) for m in mask] if mask is not None else None,
                                 turn_id=str(i)))
    return segs


def output_records(output: dict[str, Any], *, group: str, env_name: str, step: int,
                   advantage: float | None) -> list[RLExample]:
    """Training rows of one rollout: its model calls merged into rows, each
    with the rollout's reward and advantage."""
    temp = float((output.get("sampling_args") or {}).get("temperature", 1.0) or 1.0)
    rows = merge_token_segments(output_segments(output), temperature=temp)
    traj = output.get("trajectory") or []
    last = traj[-1] if traj else {}
    completion_tokens = sum(len(((s or {}).get("tokens") or {}).get("completion_ids") or []) for s in traj)
    recs = []
    for k, row in enumerate(rows):
        if not any(row.loss_mask[1:]):
            continue
        md = {"group": group, "env": env_name, "reward_source": "verifier", "step": step,
              "example_id": str(output.get("example_id", "")), "sample_index": k,
              "stop_condition": output.get("stop_condition"), "is_truncated": bool(output.get("is_truncated")),
              "turn_count": len(traj), "completion_token_count": completion_tokens,
              "rollout_count": 1 if k == 0 else 0}
        r = to_rl_example(row, reward=float(output["reward"]), advantage=advantage, temperature=temp, metadata=md)
        r.prompt = [dict(m) for m in (last.get("prompt") or []) if isinstance(m, dict)]
        r.completion = [dict(m) for m in (last.get("completion") or []) if isinstance(m, dict)]
        r.source = env_name
        recs.append(r)
    return recs


class _Admit:
    """``async with``: one admission of ``cost`` rollouts (no-op without a controller)."""

    def __init__(self, controller, cost: int):
        self.controller, self.cost = controller, cost

    async def __aenter__(self):
        if self.controller is not None:
            await self.controller.aacquire(self.cost)
        return self

    async def __aexit__(self, *exc):
        if self.controller is not None:
            self.controller.release(self.cost)
        return False


async def run_group(vf, env, example: dict[str, Any], *, client: Any, model: str, sampling: dict[str, Any],
                    rollout_count: int, max_retries: int, failures: FailureStats | None = None,
                    admission=None) -> list[dict[str, Any]]:
    """The outputs of one prompt's group that can be trained on.
    ``admission`` (``concurrency.AdmissionController``) bounds the rollouts in
    flight and their start rate across groups; a jointly scored group is
    admitted as a whole."""

    async def one():
        async with _Admit(admission, 1):
            return await env.run_rollout(vf.RolloutInput(**example), client=client, model=model,
                                         sampling_args=sampling, max_retries=max_retries,
                                         state_columns=STATE_COLUMNS)

    if getattr(env, "requires_group_scoring", False):
        fn = getattr(env, "run_group", None)
        if not callable(fn):
            raise ValueError("the verifier environment scores groups but has no run_group()")
        async with _Admit(admission, rollout_count):
            results = list(await fn([vf.RolloutInput(**example) for _ in range(rollout_count)], client=client,
                                    model=model, sampling_args=sampling, max_retries=max_retries,
                                    state_columns=STATE_COLUMNS))
        if failures is not None:
            for _ in range(max(0, rollout_count - len(results))):
                failures.record("MissingRollout")
    else:
        results = await asyncio.gather(*(one() for _ in range(rollout_count)), return_exceptions=True)
    return successful_outputs(list(results), failures)


# ----------------------------------------------------------------------------------------------------------------
# orchestrator side
# ----------------------------------------------------------------------------------------------------------------


class VerifierEnvironment:
    """A ``verifiers`` environment as the prompt sources see an environment."""

    def __init__(self, vf, env_id: str, args: dict[str, Any] | None, extra: dict[str, Any] | None = None,
                 name: str | None = None):
        self.vf = vf
        self.env_id = env_id
        self.env, _ = load_env(vf, env_id, args, extra)
        self.name = name or env_id.split("@", 1)[0]
        self._train: list[dict[str, Any]] | None = None
        self._eval: list[dict[str, Any]] | None = None
        self.metadata = {"kind": "verifiers", "id": env_id}

    @staticmethod
    def _rows(ds) -> list[dict[str, Any]]:
        if ds is None:
            return []
        rows = ds.to_list() if hasattr(ds, "to_list") else list(ds)
        return [normalize_example(dict(r)) for r in rows]

    @property
    def examples(self) -> list[dict[str, Any]]:
        if self._train is None:
            self._train = self._rows(self.env.get_dataset())
            for i, r in enumerate(self._train):
                r.setdefault("example_id", i)
        return self._train

    @property
    def eval_examples(self) -> list[dict[str, Any]]:
        if self._eval is None:
            getter = getattr(self.env, "get_eval_dataset", None)
            self._eval = self._rows(getter()) if callable(getter) else []
            for i, r in enumerate(self._eval):
                r.setdefault("example_id", i)
        return self._eval

    def chat(self, row: dict[str, Any]) -> list[dict[str, Any]]:
        p = row.get("prompt")
        if isinstance(p, str):
            return [{"role": "user", "content": p}]
        return [dict(m) for m in (p or [])]


def verifier_train_envs(cfg, specs: list[tuple[str, dict, float]]) -> list[tuple[VerifierEnvironment, float]]:
    """(environment, ratio) for every training entry, from the package."""
    vf = load_verifiers("environments")
    by_id = {e.id: e for e in cfg.orchestrator.envs}
    out = []
    for env_id, args, ratio in specs:
        entry = by_id.get(env_id)
        out.append((VerifierEnvironment(vf, env_id, args, env_kwargs(cfg),
                                        name=getattr(entry, "resolved_name", None)), float(ratio)))
    return out


class VerifierRollouts:
    """``RLOrchestrator``'s rollout function for prompts of verifier
    environments (``custom_rollout(prompts, step) -> records``); records of
    other prompts are generated by ``fallback`` (the native path)."""

    def __init__(self, cfg, envs: dict[str, VerifierEnvironment], engine: Any | None = None, fallback=None):
        from .algorithms import algorithm_scope, build_algorithm

        self.cfg = cfg
        self.envs = envs
        self.vf = load_verifiers("environments")
        self.clients = client_configs(self.vf, cfg)
        self.model = model_name(cfg, engine)
        self.fallback = fallback
        self.entries = {getattr(e, "resolved_name", e.id): e for e in cfg.orchestrator.envs}
        self._adm = None
        self._adaptive = None
        self._algos = {}
        for name in envs:
            e = self.entries.get(name)
            a = (e.algo if e is not None and e.algo is not None else cfg.algo)
            self._algos[name] = (build_algorithm(a), algorithm_scope(a))
        self.last_stats: dict[str, float] = {}

    def _group_size(self, name: str) -> int:
        e = self.entries.get(name)
        if e is not None and e.group_size is not None:
            return int(e.group_size)
        return int(self.cfg.orchestrator.rollouts_per_example or 1)

    def _sampling(self, name: str, step: int) -> dict[str, Any]:
        e = self.entries.get(name)
        s = self.cfg.resolved_train_sampling(e) if e is not None else self.cfg.inference.sampling
        return sampling_args(s, cache_salt=str(step))

    def _advantages(self, name: str, outputs: list[dict[str, Any]], group: str) -> list[float | None]:
        from .algorithms import score_records

        algo, scope = self._algos[name]
        proto = [RLExample(prompt=[], completion=[], advantage=o.get("advantage"), reward=float(o["reward"]),
                           metadata={"group": group, "is_truncated": bool(o.get("is_truncated")),
                                     "completion_token_count": sum(
                                         len(((s or {}).get("tokens") or {}).get("completion_ids") or [])
                                         for s in (o.get("trajectory") or []))},
                           source=name) for o in outputs]
        scored = score_records(algo, proto, scope, group_key=lambda r: 0)
        return [r.advantage for r in scored]

    def _admission(self):
        """In-flight cap (``max_inflight_rollouts``, resized by the adaptive
        controller when ``orchestrator.concurrency`` is set) and start rate
        (``tasks_per_minute``) of the rollouts; None when neither is set."""
        from .concurrency import AdaptiveConcurrency, AdmissionController

        o = self.cfg.orchestrator
        if o.max_inflight_rollouts is None and o.tasks_per_minute is None and o.concurrency is None:
            return None
        if self._adm is None:
            if o.concurrency is not None:
                self._adaptive = AdaptiveConcurrency(o.concurrency, default_initial=o.max_inflight_rollouts or 64)
            limit = self._adaptive.cap if self._adaptive is not None else (o.max_inflight_rollouts or 1 << 30)
            if self._adaptive is not None and o.max_inflight_rollouts:
                limit = min(limit, o.max_inflight_rollouts)
            tpm = o.tasks_per_minute
            self._adm = AdmissionController(limit, rate=tpm / 60.0 if tpm else None, burst=tpm)
        return self._adm

    async def _poll_load(self, adm) -> None:
        """Feed server load samples to the adaptive controller every poll interval."""
        from .inference_metrics import EngineMetricsScraper

        c = self.cfg.orchestrator.concurrency
        scraper = EngineMetricsScraper()
        roots = [u[: -len("/v1")] if u.endswith("/v1") else u for u in base_urls(self.cfg)]
        while True:
            await asyncio.sleep(c.poll_interval_seconds)
            loads = []
            for root in roots:
                try:
                    loads.append(await asyncio.to_thread(scraper.scrape, root, c.request_timeout_seconds))
                except Exception as exc:  # noqa: BLE001 - a missed sample is skipped
                    log.debug("load sample from %s failed: %s", root, exc)
            if not loads:
                continue
            from .concurrency import EngineLoad

            agg = EngineLoad(kv_cache_usage=max(x.kv_cache_usage for x in loads),
                             running=sum(x.running for x in loads), waiting=sum(x.waiting for x in loads),
                             preemptions_delta=sum(x.preemptions_delta for x in loads))
            cap = self._adaptive.observe(agg, adm.inflight)
            mx = self.cfg.orchestrator.max_inflight_rollouts
            adm.set_limit(min(cap, mx) if mx else cap)

    async def _run(self, prompts, step: int, failures: FailureStats) -> list[RLExample]:
        adm = self._admission()
        poller = asyncio.create_task(self._poll_load(adm)) if adm is not None and self._adaptive is not None else None
        try:
            return await self._run_groups(prompts, step, adm, failures)
        finally:
            if poller is not None:
                poller.cancel()
                await asyncio.gather(poller, return_exceptions=True)

    async def _run_groups(self, prompts, step: int, adm, failures: FailureStats) -> list[RLExample]:
        jobs, keys = [], []
        for i, p in enumerate(prompts):
            name = p.metadata.get("env")
            env = self.envs[name]
            example = dict(p.metadata.get("env_row") or {})
            jobs.append(run_group(self.vf, env.env, example, client=self.clients[i % len(self.clients)],
                                  model=self.model, sampling=self._sampling(name, step),
                                  rollout_count=self._group_size(name),
                                  max_retries=int(self.cfg.orchestrator.verifier_max_retries),
                                  failures=failures, admission=adm))
            keys.append((i, name))
        results = await asyncio.gather(*jobs, return_exceptions=True)
        recs: list[RLExample] = []
        for (i, name), res in zip(keys, results):
            if isinstance(res, BaseException):
                raise_if_rate_limited(res)
                failures.record(res)
                log.warning("verifier rollout group failed: %r", res)
                continue
            if len(res) < self._group_size(name) and self.cfg.orchestrator.batch_selection != "rollouts":
                # batches count whole groups: a group that lost rollouts is not trained on
                # (orchestrator.batch_selection: rollouts keeps the survivors)
                if res:
                    failures.record("IncompleteGroup")
                continue
            group = f"{step}:{i}"
            for out, adv in zip(res, self._advantages(name, res, group)):
                recs += output_records(out, group=group, env_name=name, step=step, advantage=adv)
        return recs

    takes_fallback = True  # RLOrchestrator passes its own native generation for mixed batches

    def __call__(self, prompts, step: int, fallback=None) -> tuple[list[RLExample], dict[str, float]]:
        """(records, statistics) of one step; every call keeps its own
        failure counts, so steps generated concurrently do not mix them."""
        failures = FailureStats()
        mine = [p for p in prompts if p.metadata.get("env") in self.envs]
        others = [p for p in prompts if p.metadata.get("env") not in self.envs]
        recs = asyncio.run(self._run(mine, step, failures)) if mine else []
        if others:
            fb = fallback or self.fallback
            if fb is None:
                raise ValueError("prompts of native environments reached the verifier rollout function")
            recs += fb(others, step)
        stats = failures.consume()
        rewards = [float(r.reward) for r in recs if (r.metadata or {}).get("rollout_count")]
        stats["verifier/rollouts"] = float(len(rewards))
        if self._adaptive is not None:
            stats.update(self._adaptive.metrics())
        if rewards:
            stats["verifier/reward_mean"] = sum(rewards) / len(rewards)
        self.last_stats = stats
        return recs, stats


# ----------------------------------------------------------------------------------------------------------------
# evaluation
# ----------------------------------------------------------------------------------------------------------------


def _eval_output(value: Any, example: dict[str, Any], index: int) -> dict[str, Any]:
    ex_id = str(example.get("example_id", index))
    if isinstance(value, BaseException):
        raise_if_rate_limited(value)
        return {"example_id": ex_id, "error": _truncate(str(value)), "completion": []}
    try:
        out = json.loads(json.dumps(dict(value), default=_json_default))
    except (TypeError, ValueError) as exc:
        return {"example_id": ex_id, "error": f"invalid verifier result: {exc}", "completion": []}
    out.setdefault("example_id", ex_id)
    out["example_id"] = str(out["example_id"])
    if out.get("error") is not None:
        raise_if_rate_limited(out["error"])
        out["error"] = _truncate(str(out["error"]))
        out.pop("reward", None)
    elif "reward" in out:
        r = out["reward"]
        if isinstance(r, bool) or not isinstance(r, (int, float)) or not math.isfinite(r):
            return {"example_id": ex_id, "error": "invalid verifier result: the reward is not a finite number",
                    "completion": []}
    return out


def _json_default(v: Any) -> Any:
    dump = getattr(v, "model_dump", None)
    if callable(dump):
        return dump(mode="json", exclude_none=True)
    return str(v)


async def _eval_rollouts(vf, env, examples, *, clients, model, sampling, k: int, max_retries: int,
                         max_inflight: int | None, journal=None, live: dict[str, Any] | None = None,
                         cancel=None) -> list[dict[str, Any]]:
    """Every (example, sample) rollout; results already committed in
    ``journal`` are reused, new ones are committed as they finish; ``live``
    (LiveEpisode arguments) traces each rollout for the dashboard."""
    from .eval_journal import episode_keys
    from .live import LiveEpisode

    total = len(examples) * k
    keys = episode_keys(examples, k)
    results: list[dict[str, Any] | None] = [None] * total
    nxt = 0

    async def worker():
        nonlocal nxt
        while nxt < total:
            if cancel is not None and cancel.is_set():
                return  # no new rollouts once the evaluation is cancelled
            idx = nxt
            nxt += 1
            ei, ri = divmod(idx, k)
            done = journal.completed(keys[idx]) if journal is not None else None
            if done is not None:
                results[idx] = done
                continue
            s = dict(sampling)
            if s.get("seed") is not None and ri:
                s["seed"] = int(s["seed"]) + ri  # distinct samples for avg@k / pass@k
            ep = LiveEpisode(**live, example_id=keys[idx]) if live is not None else None
            try:
                if ep is not None:
                    await ep.__aenter__()
                val = await env.run_rollout(vf.RolloutInput(**examples[ei]), client=clients[ei % len(clients)],
                                            model=model, sampling_args=s, max_retries=max_retries,
                                            state_columns=STATE_COLUMNS)
            except asyncio.CancelledError:
                if ep is not None:
                    await ep.__aexit__(asyncio.CancelledError, asyncio.CancelledError(), None)
                raise
            except Exception as exc:  # noqa: BLE001 - an environment failure is a failed sample
                val = exc
            out = _eval_output(val, examples[ei], ei)
            if ep is not None:
                err = out.get("error")
                if err is not None:
                    ep.finish("error", error=err)
                await ep.__aexit__(None, None, None)
            results[idx] = journal.record(keys[idx], out) if journal is not None else out

    n_workers = max(1, min(total, max_inflight or total))
    tasks = [asyncio.create_task(worker()) for _ in range(n_workers)]
    try:
        await asyncio.gather(*tasks)
    finally:
        for t in tasks:
            if not t.done():
                t.cancel()
        await asyncio.gather(*tasks, return_exceptions=True)
    return [r for r in results if r is not None]


def evaluate(cfg, env_cfg, *, step: int, out_dir: Path, engine: Any | None = None,
             cancel=None) -> dict[str, float] | None:
    """Evaluate the served policy on one verifier environment entry of
    ``eval.env`` (resumable through its journal when ``eval.resume`` is on)."""
    from .evals import group_metrics

    vf = load_verifiers("evals")
    env, _ = load_env(vf, env_cfg.id, {k: v for k, v in (env_cfg.args or {}).items() if k != "success_threshold"},
                      env_kwargs(cfg))
    getter = getattr(env, "get_eval_dataset", None) or env.get_dataset
    n = env_cfg.num_examples if env_cfg.num_examples > 0 else -1
    ds = getter(n=n) if n > 0 else getter()
    examples = [normalize_example(dict(r)) for r in (ds.to_list() if hasattr(ds, "to_list") else list(ds))]
    if n > 0:
        examples = examples[:n]
    for i, r in enumerate(examples):
        r.setdefault("example_id", i)
    sargs = env_cfg.sampling.to_sampling_args()  # only what the entry sets; the server's defaults otherwise
    sargs["extra_body"] = {**sargs.get("extra_body", {}), "cache_salt": f"eval-{step}"}
    from .eval_journal import EvalJournal, signature

    from ..configs.config import RLEvalConfig

    ev = cfg.eval if cfg.eval is not None else RLEvalConfig()
    name = env_cfg.resolved_name
    model = model_name(cfg, engine)
    sig = signature(env_id=env_cfg.id, env_args=env_cfg.args, env_kwargs=env_kwargs(cfg), model=model,
                    sampling=sargs, samples=env_cfg.rollouts_per_example, num_examples=env_cfg.num_examples,
                    model_config=cfg.model.model_dump(mode="json"), model_revision=ev.model_revision,
                    policy_step=step, endpoints=base_urls(cfg))
    live = ({"run_dir": Path(out_dir), "env": name, "kind": "eval", "step": step, "policy_step": step}
            if ev.live_traces else None)
    with EvalJournal(Path(out_dir) / "evals" / name / f"journal-step-{step}", sig=sig,
                     resume=bool(ev.resume)) as journal:
        outs = asyncio.run(_eval_rollouts(vf, env, examples,
                                          clients=client_configs(vf, cfg, client_type="openai_chat_completions"),
                                          model=model, sampling=sargs, k=env_cfg.rollouts_per_example,
                                          max_retries=int(getattr(env_cfg, "max_retries", 0) or 0),
                                          max_inflight=ev.max_inflight_rollouts,
                                          journal=journal, live=live, cancel=cancel))
    if cancel is not None and cancel.is_set():
        return None  # stopped part-way; committed episodes stay in the journal
    elapsed = journal.elapsed_seconds
    by_ex: dict[str, list[float | None]] = {}
    for o in outs:
        by_ex.setdefault(str(o["example_id"]), []).append(float(o["reward"]) if "reward" in o else None)
    thr = float((env_cfg.args or {}).get("success_threshold", 1.0))
    m = group_metrics(f"eval/{name}", by_ex, thr)
    m[f"eval/{name}/time"] = elapsed  # summed over resumed attempts
    lens = [sum(len(((st or {}).get("tokens") or {}).get("completion_ids") or []) for st in (o.get("trajectory") or []))
            for o in outs if o.get("error") is None]
    if lens:
        m[f"eval/{name}/completion_len/mean"] = sum(lens) / len(lens)
    trunc = [bool(o.get("is_truncated")) for o in outs]
    if trunc:
        m[f"eval/{name}/is_truncated/mean"] = sum(trunc) / len(trunc)
    d = Path(out_dir) / "evals" / name
    d.mkdir(parents=True, exist_ok=True)
    with (d / f"step-{step}.jsonl").open("w", encoding="utf-8") as f:
        for o in outs:
            f.write(json.dumps(o, default=_json_default) + "\n")
    from .evals import prune_eval_sets

    prune_eval_sets(d, ev.keep_last_rollout_sets)
    return m
