"""verifiers-package environments through the orchestrator bridge.

The ``verifiers`` package is not in this image, so a stand-in module with the
calls the bridge makes (``load_environment``, ``ClientConfig``,
``RolloutInput``, ``env.run_rollout`` / ``run_group``, ``get_dataset`` /
``get_eval_dataset``, ``set_kwargs``) is installed in ``sys.modules``.  Its
environment plays a two-turn tool episode per rollout (the second model call
sees the first call's prompt, its completion and a tool response), so the
checks cover the token merging, the reward / advantage plumbing, dropped
rollouts, rate limits, group scoring and evaluation (ref orchestrator/envs.py:
600-1640).
"""

from __future__ import annotations

import json
import sys
import types

import pytest

from wavelet_b200.configs.config import RLConfig


class _Rows:
    def __init__(self, rows):
        self.rows = rows

    def to_list(self):
        return [dict(r) for r in self.rows]


class FakeEnv:
    requires_group_scoring = False

    def __init__(self, n=4, fail_ids=(), rate_limit=False, flat_ids=(), **args):
        self.args = args
        self.flat_ids = set(flat_ids)
        self.kwargs = {}
        self.fail_ids = set(fail_ids)
        self.rate_limit = rate_limit
        self.calls = []
        self.rows = [{"prompt": [{"role": "user", "content": f"q{i}"}], "answer": str(i), "task": "fake",
                      "example_id": i} for i in range(n)]

    def set_kwargs(self, **kw):
        self.kwargs.update(kw)

    def get_dataset(self, n=-1, seed=None):
        return _Rows(self.rows)

    def get_eval_dataset(self, n=-1):
        return _Rows(self.rows[: n if n > 0 else len(self.rows)])

    async def run_rollout(self, inp, client, model, sampling_args, max_retries=0, state_columns=None):
        self.calls.append({"input": dict(inp), "client": client, "model": model, "sampling": dict(sampling_args)})
        ex = int(inp["example_id"])
        k = sum(1 for c in self.calls if int(c["input"]["example_id"]) == ex) - 1  # sample index of this example
        if self.rate_limit:
            return {"error": "Error code: 429 - rate limit exceeded for judge", "example_id": ex}
        if ex in self.fail_ids:
            raise ConnectionError("server went away")
        p1 = [100 + ex, 101, 102]
        c1 = [7, 8]
        tool = [150, 151]
        p2 = p1 + c1 + tool
        c2 = [9, 10, 11]
        reward = 1.0 if ex in self.flat_ids else float((ex + k) % 2)  # alternating within a group
        return {
            "example_id": ex, "reward": reward, "is_truncated": False, "stop_condition": "done",
            "sampling_args": dict(sampling_args),
            "trajectory": [
                {"prompt": [{"role": "user", "content": f"q{ex}"}], "completion": [{"role": "assistant", "content": "t"}],
                 "tokens": {"prompt_ids": p1, "completion_ids": c1, "completion_mask": [1, 1],
                            "completion_logprobs": [-0.1, -0.2]}},
                {"prompt": [{"role": "user", "content": f"q{ex}"}], "completion": [{"role": "assistant", "content": "a"}],
                 "tokens": {"prompt_ids": p2, "completion_ids": c2, "completion_mask": [1, 1, 1],
                            "completion_logprobs": [-0.3, -0.4, -0.5]}},
            ],
        }


class GroupEnv(FakeEnv):
    requires_group_scoring = True

    async def run_group(self, inputs, client, model, sampling_args, max_retries=0, state_columns=None):
        outs = [await self.run_rollout(i, client, model, sampling_args) for i in inputs]
        return outs[:-1]  # one rollout lost: counted as MissingRollout


@pytest.fixture
def fake_vf(monkeypatch):
    from wavelet_b200.orchestrator import verifier_envs

    mod = types.ModuleType("verifiers")
    mod.made = {}

    class ClientConfig:
        def __init__(self, **kw):
            self.__dict__.update(kw)

    def load_environment(env_id, **args):
        cls = GroupEnv if env_id.startswith("group") else FakeEnv
        env = cls(**args)
        mod.made[env_id] = env
        return env

    mod.ClientConfig = ClientConfig
    mod.RolloutInput = lambda **kw: dict(kw)
    mod.load_environment = load_environment
    monkeypatch.setitem(sys.modules, "verifiers", mod)
    monkeypatch.setattr(verifier_envs, "_ENV_CACHE", {})
    return mod


def _cfg(tmp_path, envs, **orch):
    return RLConfig.model_validate({
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64, "fake_prompt_len": 6},
        "inference": {"sampling": {"max_completion_tokens": 8, "seed": 5},
                      "vllm": {"server_backend": "openai"}, "http": {"host": "127.0.0.1", "ports": [8101, 8102]}},
        "launcher": {"mode": "process"},
        "orchestrator": {"custom_rollout_function": "verifiers", "envs": envs, "examples_per_step": 2,
                         "rollouts_per_example": 4, "max_async_level": 1, "verifier_timeout_seconds": 30.0, **orch},
        "algo": {"type": "grpo"},
        "lora": None, "output_dir": str(tmp_path / "out")})


def _orchestrator(cfg):
    from wavelet_b200.orchestrator.rollouts import RLOrchestrator
    from wavelet_b200.orchestrator.runtime import build_prompt_source

    return RLOrchestrator(cfg, None, None, build_prompt_source(cfg, 64))


def test_training_rollouts_merge_turns_and_carry_rewards(tmp_path, fake_vf):
    cfg = _cfg(tmp_path, [{"id": "fake-env", "args": {"n": 2, "fail_ids": [1]}}])
    orch = _orchestrator(cfg)
    env = fake_vf.made["fake-env"]
    assert env.kwargs == {"max_seq_len": 128, "max_total_completion_tokens": -1, "timeout_seconds": 30.0}
    recs = orch.materialize(0)
    # both examples are drawn; example 0: four rollouts of two model calls each, merged
    # into one row per rollout; example 1's rollouts fail and are dropped
    assert len(recs) == 4 and len({r.metadata["group"] for r in recs}) == 1
    assert {r.metadata["example_id"] for r in recs} == {"0"}
    r = recs[0]
    assert r.input_ids == [100, 101, 102, 7, 8, 150, 151, 9, 10, 11]
    assert r.loss_mask == [False, False, False, True, True, False, False, True, True, True]
    assert r.inference_logprobs == [-0.1, -0.2, -0.3, -0.4, -0.5]
    assert r.metadata["reward_source"] == "verifier" and r.metadata["turn_count"] == 2
    assert r.source == "fake-env"
    # rewards alternate 0/1 within the group: GRPO advantages are centred
    rewards = sorted(x.reward for x in recs)
    assert rewards == [0.0, 0.0, 1.0, 1.0]
    assert abs(sum(x.advantage for x in recs)) < 1e-6 and all(abs(x.advantage) > 0 for x in recs)
    assert orch.last_stats["verifier/failures/ConnectionError"] == 4.0
    assert orch.last_stats["verifier/rollouts"] == 4.0
    # the rollout inputs, clients and sampling the environment got
    c = env.calls[0]
    assert c["input"]["info"] == {"env_id": "fake"} and "task" not in c["input"]
    assert c["model"] == "tiny" and c["client"].api_base_url in ("http://127.0.0.1:8101/v1", "http://127.0.0.1:8102/v1")
    assert c["sampling"]["extra_body"]["return_token_ids"] is True and c["sampling"]["max_completion_tokens"] == 8
    assert c["sampling"]["extra_body"]["cache_salt"] == "0" and c["sampling"]["logprobs"] is True


def test_group_size_and_group_scoring(tmp_path, fake_vf):
    # batch_selection: rollouts keeps the survivors of a group that lost a rollout
    cfg = _cfg(tmp_path, [{"id": "group-env", "args": {"n": 2}, "group_size": 3}], batch_selection="rollouts",
               refill_zero_advantage=False, filter_zero_advantage=False)
    orch = _orchestrator(cfg)
    recs = orch.materialize(3)
    groups = {r.metadata["group"] for r in recs}
    assert groups == {"3:0", "3:1"}
    per_group = {g: sum(1 for r in recs if r.metadata["group"] == g) for g in groups}
    assert all(n == 2 for n in per_group.values())  # 3 asked, one lost by run_group
    assert orch.last_stats["verifier/failures/MissingRollout"] == 2.0
    # batch_selection: groups (the default) does not train on an incomplete group
    fake_vf.made.clear()
    from wavelet_b200.orchestrator import verifier_envs

    verifier_envs._ENV_CACHE.clear()
    orch = _orchestrator(_cfg(tmp_path, [{"id": "group-env", "args": {"n": 2}, "group_size": 3}]))
    recs, stats = orch.custom_rollout([p for p in orch.prompts.take(2)], 0)
    assert stats["verifier/failures/IncompleteGroup"] == 2.0 and recs == []


def test_rollout_selection_trims_and_drops_single_rollouts(tmp_path, fake_vf):
    # 2 prompts x 4 rollouts asked, rewards alternate 0/1 within each group: with
    # batch_selection: rollouts zero-advantage rollouts are dropped one by one and
    # the batch is cut at examples_per_step x rollouts_per_example rollouts
    cfg = _cfg(tmp_path, [{"id": "fake-env", "args": {"n": 2, "flat_ids": [0]}}], batch_selection="rollouts",
               refill_zero_advantage=False)
    orch = _orchestrator(cfg)
    recs = orch.materialize(0)
    # example 0 scores 1.0 on every rollout: its four zero-advantage rollouts are dropped one by one
    assert len(recs) == 4 and {r.metadata["example_id"] for r in recs} == {"1"}
    assert orch.last_stats["rollout/zero_advantage_dropped"] == 4.0

    from wavelet_b200.data.rl import RLExample
    from wavelet_b200.orchestrator.rollouts import _trim_rollouts

    rows = [RLExample([], [], 1.0, 1.0, metadata={"rollout_count": c, "i": i}) for i, c in enumerate([1, 0, 1, 1, 0])]
    assert [r.metadata["i"] for r in _trim_rollouts(rows, 2)] == [0, 1, 2]  # a rollout's later rows stay with it


def test_rate_limit_stops_the_run(tmp_path, fake_vf):
    cfg = _cfg(tmp_path, [{"id": "fake-env", "args": {"rate_limit": True}}])
    orch = _orchestrator(cfg)
    with pytest.raises(RuntimeError, match="rate limited"):
        orch.materialize(0)


def test_mixed_native_and_verifier_environments(tmp_path, fake_vf):
    cfg = _cfg(tmp_path, [{"id": "fake-env", "args": {"n": 3}, "ratio": 1.0},
                          {"id": "equation_builder", "args": {"num_examples": 8, "eval_examples": 2}, "ratio": 1.0}])
    from wavelet_b200.orchestrator.runtime import build_prompt_source

    src = build_prompt_source(cfg, 64)
    prompts = src.take(4)
    assert sorted(p.metadata["env"] for p in prompts) == ["equation_builder", "equation_builder", "fake-env", "fake-env"]
    state = src.state_dict()
    src2 = build_prompt_source(cfg, 64)
    src2.load_state_dict(state)
    assert [p.example_id for p in src2.take(2)] == [p.example_id for p in src.take(2)]


def test_missing_package_is_named(tmp_path, monkeypatch):
    monkeypatch.setitem(sys.modules, "verifiers", None)  # import fails
    cfg = _cfg(tmp_path, [{"id": "some-hub-env"}])
    from wavelet_b200.orchestrator.runtime import build_prompt_source

    with pytest.raises(ValueError, match="needs the verifiers package"):
        build_prompt_source(cfg, 64)


def test_legacy_verifier_env_id(tmp_path, fake_vf):
    from wavelet_b200.orchestrator import runtime

    cfg = RLConfig.model_validate({
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64, "fake_prompt_len": 6},
        "orchestrator": {"verifier_env_id": "fake-env"}, "lora": None, "output_dir": str(tmp_path / "o")})
    src = runtime.build_prompt_source(cfg, 64)
    assert src.envs[0][0].metadata["kind"] == "verifiers" and src.envs[0][0].name == "fake-env"


def test_evaluation_metrics_and_files(tmp_path, fake_vf):
    from wavelet_b200.orchestrator.evals import run_evals

    from wavelet_b200.configs.config import RLEvalEnvConfig

    cfg = _cfg(tmp_path, [{"id": "fake-env"}])

    ev = RLEvalEnvConfig(id="fake-env", name="fe", args={"n": 3, "fail_ids": [2]}, rollouts_per_example=2,
                         num_examples=3, sampling={"seed": 11, "temperature": 0.7})
    m = run_evals(cfg, None, step=5, envs=[ev])
    assert m["eval/fe/num_examples"] == 3.0
    assert m["eval/fe/failed_rollouts"] == 2.0
    # example k's sample j has reward (k + j) % 2: examples 0 and 1 each have one success of two
    assert m["eval/fe/pass@2"] == pytest.approx(2 / 3)
    assert m["eval/fe/pass@1"] == pytest.approx(1 / 3)
    env = fake_vf.made["fake-env"]
    seeds = sorted(c["sampling"]["seed"] for c in env.calls)
    assert seeds == [11, 11, 11, 12, 12, 12] and env.calls[0]["sampling"]["temperature"] == 0.7
    rows = [json.loads(line) for line in (tmp_path / "out" / "evals" / "fe" / "step-5.jsonl").read_text().splitlines()]
    assert len(rows) == 6 and sum("error" in r for r in rows) == 2
    assert json.loads((tmp_path / "out" / "eval_metrics.jsonl").read_text().splitlines()[-1])["step"] == 5


def test_inflight_rollouts_are_capped(tmp_path, fake_vf):
    import asyncio

    from wavelet_b200.orchestrator import verifier_envs

    state = {"now": 0, "peak": 0}
    orig = FakeEnv.run_rollout

    async def slow(self, *a, **k):
        state["now"] += 1
        state["peak"] = max(state["peak"], state["now"])
        await asyncio.sleep(0.01)
        state["now"] -= 1
        return await orig(self, *a, **k)

    FakeEnv.run_rollout = slow
    try:
        cfg = _cfg(tmp_path, [{"id": "fake-env", "args": {"n": 2}}], max_inflight_rollouts=5)
        recs = _orchestrator(cfg).materialize(0)
    finally:
        FakeEnv.run_rollout = orig
    assert len(recs) == 8 and state["peak"] == 5
    assert verifier_envs is not None


def test_adaptive_concurrency_sheds_under_load(tmp_path, fake_vf, monkeypatch):
    import asyncio

    from wavelet_b200.orchestrator.concurrency import EngineLoad
    from wavelet_b200.orchestrator.inference_metrics import EngineMetricsScraper

    seen = []
    monkeypatch.setattr(EngineMetricsScraper, "scrape",
                        lambda self, root, timeout=5.0: seen.append(root) or EngineLoad(kv_cache_usage=0.95))
    orig = FakeEnv.run_rollout

    async def slow(self, *a, **k):
        await asyncio.sleep(0.03)
        return await orig(self, *a, **k)

    monkeypatch.setattr(FakeEnv, "run_rollout", slow)
    cfg = _cfg(tmp_path, [{"id": "fake-env", "args": {"n": 2}}], tasks_per_minute=6000,
               concurrency={"initial_inflight": 8, "poll_interval_seconds": 0.005})
    orch = _orchestrator(cfg)
    recs = orch.materialize(0)
    assert len(recs) == 8
    assert orch.last_stats["concurrency/shed"] >= 1 and orch.last_stats["concurrency/limit"] < 8
    assert set(seen) <= {"http://127.0.0.1:8101", "http://127.0.0.1:8102"} and seen
    adm = orch.custom_rollout._adm
    assert adm.rate == 100.0 and adm.burst == 6000.0 and adm.inflight == 0


def test_native_server_metrics_are_scraped():
    from wavelet_b200.orchestrator.inference_metrics import EngineMetricsScraper

    load = EngineMetricsScraper().from_prometheus(
        "wavelet:kv_cache_usage_perc 0.5\nwavelet:num_requests_running 1\nwavelet:num_requests_waiting 3\n")
    assert load.kv_cache_usage == 0.5 and load.running == 1 and load.waiting == 3


def test_concurrency_rules(tmp_path):
    with pytest.raises(ValueError, match="at least rollouts_per_example=4"):
        _cfg(tmp_path, [{"id": "fake-env"}], concurrency={"initial_inflight": 2})
    with pytest.raises(ValueError, match="cannot exceed the explicit"):
        _cfg(tmp_path, [{"id": "fake-env"}], max_inflight_rollouts=8, concurrency={"max_inflight": 16})
    with pytest.raises(ValueError, match="requires the Verifiers rollout source"):
        RLConfig.model_validate({"orchestrator": {"concurrency": {}}})
    from wavelet_b200.orchestrator.concurrency import AdmissionController

    adm = AdmissionController(2)
    assert adm.acquire(3, timeout=0)  # larger than the cap: admitted alone
    assert not adm.acquire(1, timeout=0)
    adm.release(3)
    assert adm.acquire(1, timeout=0)


def test_evaluation_resumes_from_its_journal(tmp_path, fake_vf):
    from wavelet_b200.configs.config import RLEvalEnvConfig
    from wavelet_b200.orchestrator.verifier_envs import evaluate

    from wavelet_b200.configs.config import RLEvalConfig

    cfg = _cfg(tmp_path, [{"id": "fake-env"}])
    cfg = cfg.model_copy(update={"eval": RLEvalConfig(resume=True)})
    ev = RLEvalEnvConfig(id="fake-env", name="fe", args={"n": 3, "fail_ids": [2]}, rollouts_per_example=2,
                         num_examples=3, sampling={"seed": 11})
    out = tmp_path / "out"
    m1 = evaluate(cfg, ev, step=4, out_dir=out)
    env = fake_vf.made["fake-env"]
    assert len(env.calls) == 6 and m1["eval/fe/failed_rollouts"] == 2.0
    # the rerun reuses the four committed results and retries only the two failed episodes
    env.calls.clear()
    m2 = evaluate(cfg, ev, step=4, out_dir=out)
    assert len(env.calls) == 2 and {int(c["input"]["example_id"]) for c in env.calls} == {2}
    assert m2["eval/fe/pass@1"] == m1["eval/fe/pass@1"] and m2["eval/fe/time"] >= m1["eval/fe/time"]
    journal = out / "evals" / "fe" / "journal-step-4"
    assert len(list(journal.glob("episode-*.json"))) == 6 and (journal / "manifest.json").exists()
    # live traces: one document per evaluated episode
    assert len(list((out / "traces" / "live").glob("*.json"))) >= 6
    # different settings against the same journal, or a journal without eval.resume: refused
    ev2 = ev.model_copy(update={"sampling": ev.sampling.model_copy(update={"seed": 12})})
    with pytest.raises(ValueError, match="settings differ"):
        evaluate(cfg, ev2, step=4, out_dir=out)
    cfg_nr = cfg.model_copy(update={"eval": cfg.eval.model_copy(update={"resume": False})})
    with pytest.raises(FileExistsError, match="eval.resume"):
        evaluate(cfg_nr, ev, step=4, out_dir=out)


def test_native_eval_resume_skips_a_finished_evaluation(tmp_path, monkeypatch):
    from wavelet_b200.configs.config import RLEvalEnvConfig
    from wavelet_b200.orchestrator import evals

    cfg = RLConfig.model_validate(
        {"eval": {"resume": True}, "output_dir": str(tmp_path / "o")})
    calls = []
    monkeypatch.setattr(evals, "_run_native_eval",
                        lambda c, e, env, step, out: calls.append(step) or {"eval/reverse/reward_mean": 0.25})
    env = RLEvalEnvConfig(id="reverse")
    assert evals.run_eval_env(cfg, None, env, 3, tmp_path / "o") == {"eval/reverse/reward_mean": 0.25}
    assert evals.run_eval_env(cfg, None, env, 3, tmp_path / "o") == {"eval/reverse/reward_mean": 0.25}
    assert calls == [3]
