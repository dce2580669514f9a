"""Asynchronous rollout scheduler (process-mode rollout role) on CPU with a
fake orchestrator and engine: bounded prefetch and in-order publish, policy
waits and lag bound, background vs drained policy loads, retries, interval /
base / final evals, colocate_sleep choreography and resume of the prompt and
curriculum state from the preceding manifest."""

import json
import threading
import time

import pytest

from wavelet_b200.configs.config import RLConfig
from wavelet_b200.data.rl import RLExample
from wavelet_b200.orchestrator.async_scheduler import (AsyncRolloutScheduler, due_eval_envs, eval_steps_done,
                                                       wait_for_trainer_memory)
from wavelet_b200.transport.queue import (STABLE, FileSystemPolicyReceiver, FileSystemRolloutSender,
                                          read_training_records, stable_steps, step_dir)


def _cfg(tmp_path, **extra):
    d = {
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 128},
        "orchestrator": {"examples_per_step": 2, "rollouts_per_example": 2},
        "algo": {"type": "grpo"},
        "lora": None,
        "output_dir": str(tmp_path / "out"),
        "max_steps": 4,
        "policy_transfer": {"poll_interval_seconds": 0.01},
    }
    for k, v in extra.items():
        if isinstance(v, dict) and isinstance(d.get(k), dict):
            d[k] = {**d[k], **v}
        else:
            d[k] = v
    return RLConfig.model_validate(d)


def _policy(out, step):
    pd = step_dir(out / "policies", step)
    pd.mkdir(parents=True, exist_ok=True)
    (pd / "policy.json").write_text(json.dumps({"step": step}))
    (pd / STABLE).touch()


class Counter:
    """Prompt source: consecutive integers; state = the cursor."""

    def __init__(self):
        self.cursor = 0
        self.curriculum = None

    def take(self, n):
        out = list(range(self.cursor, self.cursor + n))
        self.cursor += n
        return out

    def state_dict(self):
        return {"cursor": self.cursor}

    def load_state_dict(self, sd):
        self.cursor = int(sd["cursor"])


class Curr:
    def __init__(self):
        self.updates = 0

    def state_dict(self):
        return {"updates": self.updates}

    def load_state_dict(self, sd):
        self.updates = int(sd["updates"])


class FakeOrch:
    def __init__(self, prompts, delay=0.02, fail=None):
        self.prompts = prompts
        self.engine = None
        self.delay = delay
        self.fail = dict(fail or {})  # step -> failures left
        self.active = 0
        self.max_active = 0
        self.lock = threading.Lock()
        self.seen = {}

    def write_materialized(self, rows, step):
        return None

    def for_step(self, src):
        orch = self

        class View:
            last_stats = {}

            def materialize(self, step):
                with orch.lock:
                    orch.active += 1
                    orch.max_active = max(orch.max_active, orch.active)
                    left = orch.fail.get(step, 0)
                    if left:
                        orch.fail[step] = left - 1
                try:
                    time.sleep(orch.delay)
                    if left:
                        raise RuntimeError(f"environment failure at step {step}")
                    ids = src.take(2)
                    orch.seen[step] = ids
                    cur = getattr(src, "curriculum", None)
                    if cur is not None:
                        cur.updates += 1
                    self.last_stats = {"reward/mean": float(step)}
                    return [RLExample(prompt=[], completion=[], advantage=0.5, reward=1.0, input_ids=[i, i + 1],
                                      loss_mask=[False, True]) for i in ids]
                finally:
                    with orch.lock:
                        orch.active -= 1

        return View()


class FakeEngine:
    def __init__(self, concurrent=False):
        self.concurrent_generate = concurrent
        self.concurrent_policy_load = concurrent
        self.loads = []
        self.calls = []

    def load_policy(self, d, *, step):
        self.loads.append(step)
        self.calls.append(("load", step))

    def sleep(self):
        self.calls.append(("sleep",))

    def wake(self, tags=None):
        self.calls.append(("wake",))


def _sched(cfg, orch, eng, **kw):
    out = cfg.output_dir
    return AsyncRolloutScheduler(cfg, orch, eng, FileSystemRolloutSender(out, cfg.transport),
                                 FileSystemPolicyReceiver(out, cfg.policy_transfer), **kw)


def _metrics(out):
    return [json.loads(l) for l in (out / "orchestrator_metrics.jsonl").read_text().splitlines()]


def test_prefetch_runs_ahead_and_publishes_in_order(tmp_path):
    cfg = _cfg(tmp_path, orchestrator={"max_async_level": 2}, max_steps=6)
    out = cfg.output_dir
    _policy(out, 0)
    orch = FakeOrch(Counter(), delay=0.05)
    eng = FakeEngine(concurrent=True)

    def trainer():  # publishes policy s+1 once batch s is out
        for s in range(1, 6):
            while s - 1 not in stable_steps(out / "rollouts"):
                time.sleep(0.005)
            time.sleep(0.02)
            _policy(out, s)

    t = threading.Thread(target=trainer, daemon=True)
    t.start()
    assert _sched(cfg, orch, eng).run() == 0
    t.join(timeout=10)
    assert stable_steps(out / "rollouts") == list(range(6))
    m = _metrics(out)
    assert [r["step"] for r in m] == list(range(6))  # in order
    assert all(r["policy_lag"] <= 2 for r in m)  # never beyond max_async_level
    assert orch.max_active == 2  # two steps generated concurrently
    assert eng.loads == sorted(eng.loads) and eng.loads[0] == 0


def test_lag_bound_blocks_until_policy_and_in_process_engine_is_sequential(tmp_path):
    cfg = _cfg(tmp_path, orchestrator={"max_async_level": 1}, max_steps=3)
    out = cfg.output_dir
    _policy(out, 0)
    orch = FakeOrch(Counter())
    eng = FakeEngine(concurrent=False)

    def trainer():
        while 1 not in stable_steps(out / "rollouts"):
            time.sleep(0.005)
        time.sleep(0.05)
        assert 2 not in stable_steps(out / "rollouts")  # step 2 needs policy >= 1
        _policy(out, 1)

    t = threading.Thread(target=trainer, daemon=True)
    t.start()
    _sched(cfg, orch, eng).run()
    t.join(timeout=10)
    m = _metrics(out)
    assert [r["policy_step"] for r in m] == [0, 0, 1]
    assert orch.max_active == 1


def test_failed_step_is_retried_then_gives_up(tmp_path):
    cfg = _cfg(tmp_path, orchestrator={"verifier_max_retries": 2, "max_async_level": 2}, max_steps=2)
    _policy(cfg.output_dir, 0)
    orch = FakeOrch(Counter(), fail={1: 2})
    _sched(cfg, orch, FakeEngine()).run()
    m = _metrics(cfg.output_dir)
    assert m[-1]["rollout/retries"] == 2
    cfg2 = _cfg(tmp_path / "b", orchestrator={"verifier_max_retries": 1, "max_async_level": 2}, max_steps=2)
    _policy(cfg2.output_dir, 0)
    with pytest.raises(RuntimeError, match="environment failure"):
        _sched(cfg2, FakeOrch(Counter(), fail={0: 5}), FakeEngine()).run()


def test_interval_base_and_final_evals(tmp_path):
    cfg = _cfg(tmp_path, max_steps=5, orchestrator={"max_async_level": 0},
               eval={"env": [{"id": "reverse", "interval": 2}], "final_eval": True})
    out = cfg.output_dir
    orch = FakeOrch(Counter(), delay=0.0)
    evals = []

    def evaluate(env, policy_step):
        evals.append(policy_step)
        return {f"eval/{env.resolved_name}/avg@1": 1.0}

    def trainer():
        for s in range(0, 6):
            while s > 0 and s - 1 not in stable_steps(out / "rollouts"):
                time.sleep(0.002)
            _policy(out, s)

    t = threading.Thread(target=trainer, daemon=True)
    t.start()
    _sched(cfg, orch, FakeEngine(), evaluate=evaluate).run()
    t.join(timeout=10)
    assert evals[0] == 0 and 2 in evals and 4 in evals
    assert evals[-1] == 5 and len(evals) == len(set(evals))  # the final policy once
    last = eval_steps_done(out / "eval_metrics.jsonl", ["reverse"])
    assert last["reverse"] == 5
    assert due_eval_envs(cfg, 5, last, final=True) == []


def test_colocate_sleep_choreography(tmp_path):
    cfg = _cfg(tmp_path, max_steps=2, launcher={"mode": "colocate_sleep"})
    out = cfg.output_dir
    _policy(out, 0)
    eng = FakeEngine()
    waits = []
    sch = _sched(cfg, FakeOrch(Counter(), delay=0.0), eng, wait_memory=lambda: waits.append(1))

    def trainer():
        while 0 not in stable_steps(out / "rollouts"):
            time.sleep(0.002)
        _policy(out, 1)

    t = threading.Thread(target=trainer, daemon=True)
    t.start()
    sch.run()
    t.join(timeout=10)
    names = [c[0] for c in eng.calls]
    # every publish that empties the pipeline puts the engine to sleep; each
    # later load / generation first waits for the trainer's memory, then wakes it
    assert names[0] == "load" and names.count("sleep") == names.count("wake") + 1
    for i, c in enumerate(names):
        if c == "wake":
            assert names[i - 1] == "sleep"
    assert len(waits) == names.count("wake") >= 1


def test_wait_for_trainer_memory_times_out_with_details(tmp_path):
    cfg = _cfg(tmp_path, launcher={"mode": "colocate_sleep", "trainer_cuda_visible_devices": "0,1",
                                   "colocate_memory_wait_timeout_seconds": 0.05,
                                   "colocate_memory_wait_poll_seconds": 0.01})
    busy = {"0": (1000, 900), "1": (1000, 100)}
    with pytest.raises(RuntimeError, match="gpu0: used=900MiB"):
        wait_for_trainer_memory(cfg, query=lambda d: busy)
    wait_for_trainer_memory(cfg, query=lambda d: {"0": (1000, 100), "1": (1000, 100)})


def test_resume_restores_prompt_and_curriculum_state(tmp_path):
    cfg = _cfg(tmp_path, max_steps=3, orchestrator={"max_async_level": 4})
    out = cfg.output_dir
    _policy(out, 0)
    src = Counter()
    src.curriculum = Curr()
    _sched(cfg, FakeOrch(src, delay=0.0), FakeEngine()).run()
    q = out / "rollouts"
    assert stable_steps(q) == [0, 1, 2]
    for s in (0, 1):  # the trainer consumed steps 0 and 1
        (step_dir(q, s) / "consumed.json").write_text("{}")
    src2 = Counter()
    src2.curriculum = Curr()
    cfg2 = _cfg(tmp_path, max_steps=4, orchestrator={"max_async_level": 4})
    orch2 = FakeOrch(src2, delay=0.0)
    sch = _sched(cfg2, orch2, FakeEngine())
    assert sch.resume_step() == 2
    assert src2.cursor == 4 and src2.curriculum.updates == 2  # state after step 1's draw / publish
    sch.run(start=2)
    assert stable_steps(q) == [0, 1, 2, 3]
    rows = read_training_records(step_dir(q, 2) / "rollouts.jsonl.train.msgpack")
    assert [r["input_ids"][0] for r in rows] == [4, 5]  # step 2 redrawn from the restored cursor


def test_pipeline_status_and_live_state(tmp_path, caplog):
    """The periodic status line (pipeline_status_interval_seconds) and the
    live run state: every published batch becomes an event, the status
    snapshot reaches the state's sink."""
    import logging

    from wavelet_b200.orchestrator.state_server import OrchestratorRunState
    from wavelet_b200.orchestrator.status import StatusReporter, pipeline_line

    cfg = _cfg(tmp_path, orchestrator={"max_async_level": 1, "pipeline_status_interval_seconds": 0.02},
               max_steps=3)
    out = cfg.output_dir
    for s in range(4):
        _policy(out, s)
    sch = _sched(cfg, FakeOrch(Counter(), delay=0.05), FakeEngine())
    state = OrchestratorRunState(out)
    snaps = []
    sch.run_state = state
    sch.status_sink = snaps.append
    with caplog.at_level(logging.INFO, logger="wavelet"):
        assert sch.run() == 0
    ev = [e for e in state.events() if e["event"] == "batch_published"]
    assert [e["step"] for e in ev] == [0, 1, 2] and state.snapshot()["step"] == 2
    assert snaps and {"published", "target", "inflight", "ready", "loading", "policy_step"} <= set(snaps[-1])
    assert snaps[-1]["target"] == 3
    assert any("pipeline: policy" in r.getMessage() for r in caplog.records)
    line = pipeline_line({"policy_step": None, "published": 1, "target": 4, "submitted": 2, "inflight": 1,
                          "ready": 0, "loading": True})
    assert "policy none" in line and "published 1/4" in line and "policy load running" in line
    r = StatusReporter(lambda: {"policy_step": 3, "published": 0, "target": 1, "submitted": 0, "inflight": 0,
                                "ready": 0, "loading": False}, 10.0, sink=lambda s: 1 / 0)
    assert r.emit()["policy_step"] == 3  # a failing sink does not raise


def _background_run(tmp_path, cancel_on_new_policy):
    cfg = _cfg(tmp_path, max_steps=4, orchestrator={"max_async_level": 1},
               eval={"env": [{"id": "reverse", "interval": 1}], "background": True,
                     "cancel_on_new_policy": cancel_on_new_policy, "final_eval": False,
                     "eval_base_model": True})
    out = cfg.output_dir
    orch = FakeOrch(Counter(), delay=0.01)
    started, finished, cancelled, loads_during = [], [], [], []
    eng = FakeEngine(concurrent=True)
    running = threading.Event()

    def evaluate(env, step, cancel=None):
        started.append(step)
        running.set()
        for _ in range(40):  # a long evaluation: 0.4 s
            if cancel is not None and cancel.is_set():
                cancelled.append(step)
                running.clear()
                return None
            time.sleep(0.01)
        finished.append(step)
        running.clear()
        return {"eval/reverse/reward_mean": 0.0}

    orig_load = eng.load_policy

    def load_policy(d, *, step):
        loads_during.append(running.is_set())
        orig_load(d, step=step)

    eng.load_policy = load_policy

    def trainer():
        for s in range(0, 4):
            while s > 0 and s - 1 not in stable_steps(out / "rollouts"):
                time.sleep(0.002)
            _policy(out, s)

    t = threading.Thread(target=trainer, daemon=True)
    t.start()
    t0 = time.perf_counter()
    _sched(cfg, orch, eng, evaluate=evaluate).run()
    t.join(timeout=10)
    return started, finished, cancelled, loads_during, time.perf_counter() - t0


def test_background_evals_are_cancelled_by_a_new_policy(tmp_path):
    started, finished, cancelled, loads_during, _ = _background_run(tmp_path, True)
    assert started and cancelled  # evaluations of superseded policies stopped part-way
    assert not any(loads_during)  # never a weight swap under a running evaluation
    m = [json.loads(l) for l in (tmp_path / "out" / "eval_metrics.jsonl").read_text().splitlines()] \
        if (tmp_path / "out" / "eval_metrics.jsonl").exists() else []
    assert sorted(r["step"] for r in m) == sorted(finished)  # only finished evaluations report metrics


def test_background_evals_can_delay_the_policy_load(tmp_path):
    started, finished, cancelled, loads_during, _ = _background_run(tmp_path, False)
    assert not cancelled and sorted(finished) == sorted(started)
    assert not any(loads_during)
