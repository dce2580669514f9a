"""Asynchronous rollout scheduler of the process-mode rollout role.

The rollout role of the reference (orchestrator/scheduler.py: the batched
prefetch publisher :1999-2377, the verifier scheduler's retries and stale-request
handling :440-1860, evals :3104-3590, colocate_sleep :3592-3690, resume of
environment cursors and curriculum :3271-3365) keeps several optimizer
steps of rollouts in flight while the trainer works.  This is this project's
own formulation of the same behaviour:

* **Bounded prefetch.**  Up to ``P = max(1, min(max_async_level, steps left))``
  steps are generated concurrently on worker threads when the engine serves
  concurrent calls (``engine.concurrent_generate``: HTTP servers batch the
  requests); the in-process generator runs one step at a time, still ahead of
  the trainer.  A step may start once a policy snapshot at or after
  ``required_policy_step(step)`` is loaded, so no batch is ever more than
  ``max_async_level + max_off_policy_steps`` steps behind.
* **In-order publish.**  Finished steps are published to the durable queue in
  step order, each with the policy step that generated it.
* **Chunks.**  With ``orchestrator.rollout_chunk_examples`` an optimizer step's
  prompts are split into chunks of that many examples, each its own queue step
  (queue step q = chunk q % C of optimizer step q // C), so the trainer can
  start on the first chunk while later ones are generated.
* **Policy loads.**  The newest STABLE snapshot is loaded as soon as it
  appears: in the background while steps are in flight when the engine can
  swap weights under load (``engine.concurrent_policy_load``: the HTTP servers
  pause themselves), otherwise once the in-flight steps have drained.  A step
  that must wait for a newer policy blocks only its own submission.
* **Freshness.**  A finished step whose generating policy is older than its
  required policy (possible when the lag bound shrinks on resume) is
  discarded and regenerated (``rollout/stale_discarded``).
* **Retries.**  A step whose materialisation raises is retried up to
  ``orchestrator.verifier_max_retries`` times (``rollout/retries``) before the
  run fails.
* **Evals.**  After each policy load, every eval environment whose interval
  divides the policy step (and that has not seen this policy) is evaluated,
  inline or, with ``eval.background``, on a thread beside the rollouts (the
  next policy load cancels it, or waits for it with
  ``eval.cancel_on_new_policy: false``);
  the base model (policy 0) too when ``eval.eval_base_model``.  At the end the
  final policy is loaded if needed and the environments not yet evaluated at
  it run (``eval.final_eval``).  Results go to ``eval_metrics.jsonl``; a resumed
  run reads the last evaluated step of each environment back from it.
* **colocate_sleep.**  With ``launcher.mode: colocate_sleep`` the engine sleeps
  after each publish that leaves nothing in flight (the trainer takes the GPU
  memory) and, before the next generation or load, waits until the trainer's
  GPUs have ``gpu_memory_utilization - colocate_memory_wait_margin`` of their
  memory free (``nvidia-smi``, bounded by
  ``colocate_memory_wait_timeout_seconds``) and wakes it.
* **Resume.**  The first step to produce is one past the last consumed batch;
  batches at or beyond it are discarded.  Each manifest records the prompt
  source state right after the step's prompts were drawn (draws happen in step
  order on the scheduler thread) and the curriculum state at publish, and a
  resumed run restores both from the manifest of the step before it.  Prompts
  drawn later by zero-advantage refills of that step may be drawn again.
"""

from __future__ import annotations

import json
import logging
import math
import subprocess
import threading
import time
from concurrent.futures import FIRST_COMPLETED, Future, ThreadPoolExecutor, wait
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable

from ..data.rl import example_to_payload
from ..monitor import append_jsonl, emit_perf, utc_now
from ..transport.queue import FileSystemPolicyReceiver, FileSystemRolloutSender, prune_from, stable_steps, step_dir
from .schedule import chunks_per_step, required_policy_step, target_steps

log = logging.getLogger("wavelet")


class LockedPrompts:
    """Serialises draws from a prompt source shared by worker threads."""

    def __init__(self, source):
        self.source = source
        self.lock = threading.Lock()
        self.curriculum = getattr(source, "curriculum", None)

    def take(self, n: int):
        with self.lock:
            return self.source.take(n)

    def state_dict(self) -> dict | None:
        sd = getattr(self.source, "state_dict", None)
        with self.lock:
            return sd() if callable(sd) else None

    def load_state_dict(self, sd: dict) -> None:
        fn = getattr(self.source, "load_state_dict", None)
        if callable(fn) and sd is not None:
            with self.lock:
                fn(sd)


class _Prefilled:
    """A prompt source that first returns a pre-drawn list, then draws more
    (zero-advantage refills) from the shared source."""

    def __init__(self, first: list, shared: LockedPrompts):
        self.first = list(first)
        self.shared = shared
        self.curriculum = shared.curriculum

    def take(self, n: int):
        if self.first:
            out, self.first = self.first[:n], self.first[n:]
            if len(out) < n:
                out += self.shared.take(n - len(out))
            return out
        return self.shared.take(n)


@dataclass
class _Step:
    step: int
    policy: int | None
    prompt_state: dict | None
    attempt: int = 0
    t_submit: float = field(default_factory=time.perf_counter)


def eval_steps_done(metrics_path: Path, env_names: list[str]) -> dict[str, int]:
    """Last policy step evaluated per environment, from eval_metrics.jsonl."""
    last = {n: -1 for n in env_names}
    if not metrics_path.exists():
        return last
    for line in metrics_path.read_text().splitlines():
        try:
            m = json.loads(line)
        except json.JSONDecodeError:
            continue
        if not isinstance(m, dict):
            continue
        ps = m.get("progress/policy_step")
        if not isinstance(ps, (int, float)) or isinstance(ps, bool) or not math.isfinite(ps):
            continue
        for n in env_names:
            if any(str(k).startswith(f"eval/{n}/") for k in m):
                last[n] = max(last[n], int(ps))
    return last


def due_eval_envs(cfg, policy_step: int, last: dict[str, int], final: bool = False) -> list:
    """Eval environments to run at ``policy_step``: interval multiples (and
    the base model at 0 with eval.eval_base_model); every environment not yet
    evaluated at it when ``final``."""
    if cfg.eval is None:
        return []
    out = []
    for env in cfg.eval.env:
        name = env.resolved_name
        if last.get(name, -1) >= policy_step:
            continue
        if final:
            out.append(env)
        elif policy_step == 0:
            if cfg.eval.eval_base_model:
                out.append(env)
        elif policy_step % env.interval == 0:
            out.append(env)
    return out


def query_gpu_memory_mib(devices: set[str], runner: Callable = subprocess.run) -> dict[str, tuple[int, int]]:
    """index -> (total MiB, used MiB) of the given GPUs (nvidia-smi)."""
    try:
        r = runner(["nvidia-smi", "--query-gpu=index,memory.total,memory.used", "--format=csv,noheader,nounits"],
                   check=True, capture_output=True, text=True, timeout=10.0)
    except Exception:
        return {}
    out = {}
    for line in r.stdout.splitlines():
        p = [x.strip() for x in line.split(",")]
        if len(p) == 3 and p[0] in devices:
            try:
                out[p[0]] = (int(p[1]), int(p[2]))
            except ValueError:
                pass
    return out


def trainer_device_ids(cfg) -> set[str]:
    v = cfg.launcher.trainer_cuda_visible_devices or cfg.launcher.inference_cuda_visible_devices
    if v is None:
        return set()
    parts = v.replace(";", ",").replace("|", ",").split(",") if isinstance(v, str) else \
        [x for item in v for x in item.split(",")]
    return {x.strip() for x in parts if x.strip().isdigit()}


def wait_for_trainer_memory(cfg, query: Callable[[set[str]], dict] = query_gpu_memory_mib,
                            sleep: Callable[[float], None] = time.sleep,
                            clock: Callable[[], float] = time.monotonic) -> None:
    """colocate_sleep: block until the trainer's GPUs have the inference
    engine's share of memory free again (or raise after the timeout)."""
    timeout = cfg.launcher.colocate_memory_wait_timeout_seconds
    devices = trainer_device_ids(cfg)
    if timeout <= 0 or not devices:
        return
    need = max(cfg.inference.vllm.gpu_memory_utilization - cfg.launcher.colocate_memory_wait_margin, 0.0)
    deadline = clock() + timeout
    stats: dict = {}
    while True:
        stats = query(devices)
        if not stats or all(total - used >= int(total * need) for total, used in stats.values()):
            return
        if clock() >= deadline:
            break
        sleep(cfg.launcher.colocate_memory_wait_poll_seconds)
    detail = ", ".join(f"gpu{i}: used={u}MiB free={t - u}MiB total={t}MiB" for i, (t, u) in sorted(stats.items()))
    raise RuntimeError(f"timed out waiting for the colocated trainer to release GPU memory (need {need:.2f} of "
                       f"each GPU free); last seen: {detail}")


class AsyncRolloutScheduler:
    def __init__(self, cfg, orchestrator, engine, sender: FileSystemRolloutSender,
                 policies: FileSystemPolicyReceiver, prompts=None, *, evaluate: Callable | None = None,
                 wait_memory: Callable | None = None):
        self.cfg = cfg
        self.orch = orchestrator
        self.engine = engine
        self.sender = sender
        self.policies = policies
        self.out = Path(cfg.output_dir)
        base = prompts if prompts is not None else orchestrator.prompts
        self.prompts = base if isinstance(base, LockedPrompts) else LockedPrompts(base)
        self.evaluate = evaluate
        # live state (state_server.OrchestratorRunState) and the periodic
        # status snapshots; both optional
        self.run_state = None
        self.status_sink = None
        self.metrics_sink: Callable | None = None  # each published step's metrics (W&B)
        self.wait_memory = wait_memory or (lambda: wait_for_trainer_memory(cfg))
        self.concurrent_generate = bool(getattr(engine, "concurrent_generate", False))
        self.concurrent_load = bool(getattr(engine, "concurrent_policy_load", False))
        # background evaluation (eval.background): one at a time on its own thread
        self.eval_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="wavelet-evals")
        self.eval_future: Future | None = None
        self.eval_cancel: threading.Event | None = None
        self.loaded: int | None = None
        self.pending: dict[Future, _Step] = {}
        self.done: dict[int, tuple[_Step, list, dict]] = {}
        self.load_future: Future | None = None
        self.asleep = False
        self.C = chunks_per_step(cfg)  # queue steps (chunks) per optimizer step
        self.stats = {"rollout/retries": 0.0, "rollout/stale_discarded": 0.0}
        names = [e.resolved_name for e in cfg.eval.env] if cfg.eval is not None else []
        self.last_eval = eval_steps_done(self.out / "eval_metrics.jsonl", names)

    # ------------------------------------------------------------ resume
    def resume_step(self) -> int:
        """One past the last consumed batch; later batches are discarded and
        the prompt / curriculum state of the preceding manifest is restored."""
        qdir = self.sender.queue_dir
        done = stable_steps(qdir)
        consumed = [s for s in done if (step_dir(qdir, s) / "consumed.json").exists()]
        start = (max(consumed) + 1) if consumed else 0
        prune_from(qdir, start)
        if start > 0:
            batch = self.sender.stable_batch(start - 1)
            man = batch.manifest if batch is not None else None
            if man is not None:
                if man.prompt_source_state is not None:
                    self.prompts.load_state_dict(man.prompt_source_state)
                cur = self.prompts.curriculum
                if cur is not None and man.curriculum_state is not None:
                    cur.load_state_dict(man.curriculum_state)
        return start

    # ------------------------------------------------------------ policy
    def _newest_policy(self) -> int | None:
        latest = self.policies.latest()
        return None if latest is None else latest.step

    def _load(self, step: int) -> int:
        snap = self.policies.wait_for_step(step)
        if self.eval_future is not None:  # the old policy's background evaluation ends before its weights change
            ev = self.cfg.eval
            self._join_eval(cancel=ev is None or ev.cancel_on_new_policy)
        self._wake()
        t0 = time.perf_counter()
        self.engine.load_policy(snap.step_dir, step=snap.step)
        emit_perf("policy_load", step=snap.step, load_policy=time.perf_counter() - t0)
        return snap.step

    def _after_load(self, step: int) -> None:
        self.loaded = step
        self._run_evals(due_eval_envs(self.cfg, step, self.last_eval), step)

    def _finish_load(self, block: bool = False) -> bool:
        f = self.load_future
        if f is None or (not block and not f.done()):
            return False
        self.load_future = None
        self._after_load(f.result())
        return True

    def _broadcast_updates(self) -> bool:
        """Device policy updates over the NCCL broadcast (``flat_v1``) are
        collectives with the trainer: every exported step must be loaded, in
        order (a peer-memory update or a filesystem snapshot may be skipped)."""
        if self.cfg.policy_transfer.type != "nccl":
            return False
        latest = self.policies.latest()
        if latest is None:
            return False
        try:
            info = json.loads((latest.step_dir / "update_info.json").read_text())
        except (OSError, ValueError):
            return False
        return info.get("protocol") == "flat_v1"

    def _maybe_start_load(self, pool: ThreadPoolExecutor) -> None:
        """Load the newest snapshot when it is newer than the loaded one (the
        next one in order for broadcast updates)."""
        if self.load_future is not None:
            return
        newest = self._newest_policy()
        if newest is None or (self.loaded is not None and newest <= self.loaded):
            return
        if self._broadcast_updates():
            newer = [s for s in stable_steps(self.policies.policy_dir) if self.loaded is None or s > self.loaded]
            newest = newer[0] if newer else newest
        if self._eval_running():
            ev = self.cfg.eval
            if ev is not None and not ev.cancel_on_new_policy:
                return  # eval.cancel_on_new_policy: false -> the load waits for the evaluation
            self._join_eval(cancel=True)  # the evaluation of the old policy stops before its weights change
        elif self.eval_future is not None:
            self._join_eval()  # finished: collect it (and its errors)
        if self.pending and not self.concurrent_load:
            return  # the engine cannot swap weights under load: wait for a drain
        if self.pending:
            self.load_future = pool.submit(self._load, newest)
        else:
            self._after_load(self._load(newest))

    # ------------------------------------------------------------ sleep
    def _sleep(self) -> None:
        if self.cfg.launcher.mode == "colocate_sleep" and not self.asleep:
            self.engine.sleep()
            self.asleep = True

    def _wake(self) -> None:
        if self.cfg.launcher.mode == "colocate_sleep" and self.asleep:
            self.wait_memory()
            self.engine.wake()
            self.asleep = False

    # ------------------------------------------------------------ evals
    def _run_evals(self, envs: list, policy_step: int, *, inline: bool = False) -> None:
        """Evaluate ``envs`` on the loaded policy.  With ``eval.background``
        (and an engine that serves concurrent calls) they run on their own
        thread while rollouts continue; the next policy load then cancels
        them (``eval.cancel_on_new_policy``, the default) or waits for them."""
        if not envs:
            return
        self._wake()
        ev = self.cfg.eval
        if not inline and ev is not None and ev.background and self.concurrent_generate:
            self._join_eval()  # one background evaluation at a time
            self.eval_cancel = threading.Event()
            self.eval_future = self.eval_pool.submit(self._eval_envs, envs, policy_step, self.eval_cancel)
            return
        self._eval_envs(envs, policy_step, None)

    def _eval_envs(self, envs: list, policy_step: int, cancel: threading.Event | None) -> None:
        for env in envs:
            if cancel is not None and cancel.is_set():
                self.stats["eval/cancelled"] = self.stats.get("eval/cancelled", 0.0) + 1
                continue
            if self.evaluate is not None:
                m = self.evaluate(env, policy_step, cancel) if cancel is not None else self.evaluate(env, policy_step)
            else:
                from .evals import run_eval_env

                m = run_eval_env(self.cfg, self.orch.engine, env, policy_step, self.out, cancel=cancel)
            if m is None:  # cancelled part-way: no metrics for this policy
                self.stats["eval/cancelled"] = self.stats.get("eval/cancelled", 0.0) + 1
                continue
            append_jsonl(self.out / "eval_metrics.jsonl",
                         {"step": policy_step, "progress/policy_step": policy_step, "timestamp": utc_now(), **m})
            self.last_eval[env.resolved_name] = policy_step

    def _eval_running(self) -> bool:
        return self.eval_future is not None and not self.eval_future.done()

    def _join_eval(self, cancel: bool = False) -> None:
        """Wait for the background evaluation (asking it to stop first when
        ``cancel``); its errors surface here."""
        f = self.eval_future
        if f is None:
            return
        if cancel and self.eval_cancel is not None:
            self.eval_cancel.set()
        self.eval_future = None
        f.result()

    # ------------------------------------------------------------ steps
    def _materialize(self, st: _Step, prompts: list) -> tuple[list, dict]:
        view = self.orch.for_step(_Prefilled(prompts, self.prompts))
        recs = view.materialize(st.step)
        return recs, dict(view.last_stats)

    def _unit_examples(self, unit: int) -> int:
        o = self.cfg.orchestrator
        n = o.examples_per_step or 1
        if self.C == 1:
            return n
        ce = o.rollout_chunk_examples
        return max(1, min(ce, n - (unit % self.C) * ce))

    def _submit(self, pool: ThreadPoolExecutor, step: int, attempt: int = 0) -> None:
        prompts = self.prompts.take(self._unit_examples(step))
        st = _Step(step, self.loaded, self.prompts.state_dict(), attempt)
        self._wake()
        fut = pool.submit(self._materialize, st, prompts)
        self.pending[fut] = st
        emit_perf("inference_submit", step=step, policy=self.loaded, attempt=attempt)

    def _collect(self, futs, pool: ThreadPoolExecutor) -> None:
        max_retries = int(self.cfg.orchestrator.verifier_max_retries)
        for f in futs:
            st = self.pending.pop(f)
            try:
                recs, stats = f.result()
            except Exception as exc:
                if st.attempt < max_retries:
                    self.stats["rollout/retries"] += 1
                    log.warning("rollouts of step %d failed (%s); retry %d/%d", st.step, exc, st.attempt + 1,
                                max_retries)
                    self._submit(pool, st.step, st.attempt + 1)
                    continue
                raise
            if st.policy is not None and st.policy < required_policy_step(st.step // self.C, self.cfg):
                self.stats["rollout/stale_discarded"] += 1
                self._submit(pool, st.step, st.attempt)
                continue
            self.done[st.step] = (st, recs, stats)

    def _publish_ready(self, next_pub: int) -> int:
        while next_pub in self.done:
            st, recs, stats = self.done.pop(next_pub)
            rows = [example_to_payload(r, self.cfg.data) for r in recs]
            cur = self.prompts.curriculum
            write = getattr(self.orch, "write_materialized", None)  # orchestrator.materialize_path, when set
            if write is not None:
                write(rows, st.step)
            self.sender.publish(rows, step=st.step, training_records=rows, optimizer_step=st.step // self.C,
                                chunk_index=(st.step % self.C) if self.C > 1 else None,
                                policy_step=st.policy, tokens=sum(len(r.input_ids or []) for r in recs),
                                reward_mean=stats.get("reward/mean"), prompt_source_state=st.prompt_state,
                                curriculum_state=cur.state_dict() if cur is not None else None)
            from .rollout_metrics import rollout_metrics

            m = rollout_metrics(rows, step=st.step, group_size=int(self.cfg.orchestrator.rollouts_per_example or 1),
                                policy_step=st.policy, queue_step=st.step, optimizer_step=st.step // self.C,
                                stats=stats)
            m.update(stats)
            m.update(self.stats)
            m.update({"step": st.step, "optimizer_step": st.step // self.C, "policy_step": st.policy,
                      "policy_lag": None if st.policy is None else st.step // self.C - st.policy,
                      "time/step_seconds": time.perf_counter() - st.t_submit, "timestamp": utc_now()})
            append_jsonl(self.out / "orchestrator_metrics.jsonl", m)
            if self.metrics_sink is not None:
                self.metrics_sink(m)
            log.info("published rollouts for step %d (policy %s, reward %.4f)", st.step, st.policy,
                     m.get("reward/mean", 0.0))
            if self.run_state is not None:
                self.run_state.update(status="running", step=st.step, policy_step=st.policy,
                                      metrics={k: v for k, v in m.items() if isinstance(v, (int, float))})
                self.run_state.event("batch_published", step=st.step, policy_step=st.policy,
                                     samples=len(recs), reward_mean=m.get("reward/mean"))
            next_pub += 1
            if not self.pending:
                self._sleep()
        return next_pub

    # ------------------------------------------------------------ run
    def run(self, target: int | None = None, start: int | None = None) -> int:
        """Publish queue steps up to ``target`` optimizer steps (x chunks)."""
        total = (target_steps(self.cfg) if target is None else target) * self.C
        step = self.resume_step() if start is None else start
        next_pub = step
        prefetch = max(1, min(max(1, int(self.cfg.orchestrator.max_async_level)) * self.C, max(total - step, 1)))
        if not self.concurrent_generate:
            prefetch = 1  # one generator on one GPU: steps run back to back (still ahead of the trainer)
        poll = self.cfg.policy_transfer.poll_interval_seconds
        self._progress = {"target": total, "submitted": step, "published": next_pub}
        from .status import StatusReporter

        status = StatusReporter(self.pipeline_status, self.cfg.orchestrator.pipeline_status_interval_seconds,
                                sink=self.status_sink)
        with status, ThreadPoolExecutor(max_workers=prefetch + 1, thread_name_prefix="wavelet-rollouts") as pool:
            while next_pub < total:
                self._progress.update(submitted=step, published=next_pub)
                self._finish_load()
                self._maybe_start_load(pool)
                need = required_policy_step(step // self.C, self.cfg) if step < total else None
                ready = need is not None and self.loaded is not None and self.loaded >= need
                if need is not None and not ready and not self.pending and self.load_future is None:
                    self._after_load(self._load(need))  # nothing in flight: block for the required snapshot
                    continue
                if ready and len(self.pending) < prefetch:
                    self._submit(pool, step)
                    step += 1
                    continue
                if self.pending:
                    waits = list(self.pending) + ([self.load_future] if self.load_future else [])
                    finished, _ = wait(waits, timeout=poll, return_when=FIRST_COMPLETED)
                    self._collect([f for f in finished if f in self.pending], pool)
                    next_pub = self._publish_ready(next_pub)
                elif self.load_future is not None:
                    self._finish_load(block=True)
                else:
                    time.sleep(poll)
            self._finish_load(block=True)
        if self._broadcast_updates():
            self._drain_broadcasts(total // self.C)
        self._join_eval()  # a background evaluation of the last loaded policy finishes
        self._final_evals(total // self.C)
        self.eval_pool.shutdown(wait=True)
        return 0

    def _drain_broadcasts(self, total: int) -> None:
        """Take part in the trainer's remaining broadcast updates (it exports
        every ``export_every_steps`` up to the last step and waits for us)."""
        every = max(1, int(getattr(self.cfg.policy_transfer, "export_every_steps", 1) or 1))
        final = total - total % every
        while self.loaded is None or self.loaded < final:
            nxt = 0 if self.loaded is None else self.loaded + every - self.loaded % every
            self._after_load(self._load(min(nxt, final)))

    def pipeline_status(self) -> dict:
        """Snapshot for the periodic status line (read from another thread)."""
        p = getattr(self, "_progress", {"target": 0, "submitted": 0, "published": 0})
        return {"policy_step": self.loaded, "published": p["published"], "target": p["target"],
                "submitted": p["submitted"], "inflight": len(self.pending), "ready": len(self.done),
                "loading": self.load_future is not None}

    def _final_evals(self, total: int) -> None:
        """Evaluate the last policy the trainer exports at or before the final
        step (it exports every ``policy_transfer.export_every_steps``)."""
        cfg = self.cfg
        if cfg.eval is None or not cfg.eval.final_eval:
            return
        every = max(1, int(getattr(cfg.policy_transfer, "export_every_steps", 1) or 1))
        final = total - total % every
        envs = due_eval_envs(cfg, final, self.last_eval, final=True)
        if not envs:
            return
        if self.loaded is None or self.loaded < final:
            self.loaded = self._load(final)
        self._run_evals(envs, self.loaded, inline=True)
        self._sleep()
