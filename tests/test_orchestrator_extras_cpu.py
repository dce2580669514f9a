"""Curriculum samplers and gates, adaptive concurrency and admission, engine
metrics parsing, agent-trajectory merging, live episodes and the state server."""

import json
from pathlib import Path
import threading
import time

import pytest

from wavelet_b200.configs.config import RLConfig


def test_standard_and_difficulty_samplers_resume():
    from wavelet_b200.orchestrator.curriculum import DifficultyPoolSampler, StandardSampler, build_curriculum

    s = StandardSampler(5, seed=3)
    first = [s.next_index() for _ in range(5)]
    assert sorted(first) == list(range(5))
    sd = s.state_dict()
    nxt = [s.next_index() for _ in range(3)]
    s2 = StandardSampler(5, seed=3)
    s2.load_state_dict(sd)
    assert [s2.next_index() for _ in range(3)] == nxt
    cfg = RLConfig.model_validate({"orchestrator": {"curriculum": {"sampler": {"type": "difficulty_pool"},
                                                                  "gates": {"adv": {"type": "advantage_range"}}}}})
    sampler, gates = build_curriculum(cfg.orchestrator.curriculum, 4)
    assert isinstance(sampler, DifficultyPoolSampler)
    # task 0 always solved (easy, weight 0.2), task 1 never (hard, weight 0.2), 2/3 unseen (weight 1)
    for _ in range(5):
        sampler.observe("record:0", [1.0, 1.0])
        sampler.observe("record:1", [0.0, 0.0])
    assert sampler.pool_of(0) == "easy" and sampler.pool_of(1) == "hard"
    counts = [0] * 4
    for _ in range(2000):
        counts[sampler.next_index()] += 1
    assert counts[2] > 3 * counts[0] and counts[3] > 3 * counts[1]
    sd = json.loads(json.dumps(sampler.state_dict()))
    again = DifficultyPoolSampler(cfg.orchestrator.curriculum.sampler, 4)
    again.load_state_dict(sd)
    assert [again.next_index() for _ in range(10)] == [sampler.next_index() for _ in range(10)]
    g = gates["adv"]
    assert not g.admit([0.0, 0.0]) and g.admit([0.5, -0.5]) and g.metrics()["admission_rate"] == 0.5


def test_adaptive_concurrency_and_admission():
    from wavelet_b200.orchestrator.concurrency import AdaptiveConcurrency, AdmissionController, EngineLoad

    from wavelet_b200.configs.config import RLAdaptiveConcurrencyConfig

    c = AdaptiveConcurrency(RLAdaptiveConcurrencyConfig(max_inflight=256), default_initial=64)
    start = c.cap
    for _ in range(c.cfg.growth_gate_polls):
        c.observe(EngineLoad(kv_cache_usage=0.2, running=64), inflight=start)
    assert c.cap > start  # binding and low KV usage: grow
    grown = c.cap
    c.observe(EngineLoad(kv_cache_usage=0.95, running=64), inflight=grown)
    assert c.cap < grown and c.signal == "hard"
    a = AdmissionController(limit=2)
    assert a.acquire() and a.acquire() and not a.acquire(timeout=0.05)
    threading.Timer(0.05, a.release).start()
    assert a.acquire(timeout=2.0)


def test_prometheus_parsing():
    from wavelet_b200.orchestrator.inference_metrics import EngineMetricsScraper, parse_prometheus

    text = """# HELP vllm:kv_cache_usage_perc KV usage
vllm:kv_cache_usage_perc{engine="0"} 0.5
vllm:num_requests_running{engine="0"} 12
vllm:num_requests_waiting{engine="0"} 3
vllm:num_preemptions_total{engine="0"} 7
"""
    assert parse_prometheus(text)["vllm:num_requests_running"] == 12
    s = EngineMetricsScraper()
    first = s.from_prometheus(text)
    assert first.kv_cache_usage == 0.5 and first.running == 12 and first.waiting == 3 and first.preemptions_delta == 0
    second = s.from_prometheus(text.replace(" 7", " 9"))
    assert second.preemptions_delta == 2


def test_agent_trajectory_merge_and_branch():
    from wavelet_b200.orchestrator.agent_trajectory import TokenSegment, merge_token_segments, to_rl_example

    s1 = TokenSegment([1, 2, 3], [10, 11], [-0.1, -0.2])
    s2 = TokenSegment([1, 2, 3, 10, 11, 50, 51], [12], [-0.3])  # tool response 50, 51 then another call
    s3 = TokenSegment([1, 9], [13], [-0.4])  # rewritten context: a new row
    rows = merge_token_segments([s1, s2, s3])
    assert len(rows) == 2
    r = rows[0]
    assert r.input_ids == [1, 2, 3, 10, 11, 50, 51, 12]
    assert r.loss_mask == [False, False, False, True, True, False, False, True]
    assert r.inference_logprobs[3:5] == [-0.1, -0.2] and r.inference_logprobs[-1] == -0.3
    assert rows[1].input_ids == [1, 9, 13] and rows[1].segments == [2]
    ex = to_rl_example(r, reward=1.0)
    assert ex.loss_mask == r.loss_mask
    with pytest.raises(ValueError):
        TokenSegment([1], [2, 3], [-0.1])


def test_live_episode_and_state_server(tmp_path):
    import asyncio
    import subprocess
    import sys as _sys

    from fastapi.testclient import TestClient

    from wavelet_b200.orchestrator import live
    from wavelet_b200.orchestrator.live import (LiveEpisode, current_episode, episode_abandoned,
                                                install_environment_hooks, list_episodes, read_episode)
    from wavelet_b200.orchestrator.state_server import OrchestratorRunState, build_state_app

    with LiveEpisode(tmp_path, "reverse", step=3, example_id="e1") as ep:
        assert current_episode() is ep
        ep.event("generation", prompt_tokens=10, output_tokens=5, text="x" * (live.MAX_TEXT + 10))
    doc = read_episode(tmp_path, ep.id)
    assert doc["status"] == "completed" and [e["phase"] for e in doc["events"]] == ["episode_started", "generation"]
    assert doc["events"][1]["text"].endswith("10 more]")
    assert current_episode() is None
    with pytest.raises(ValueError):
        with LiveEpisode(tmp_path, "reverse") as bad:
            raise ValueError("boom")
    assert read_episode(tmp_path, bad.id)["status"] == "error" and "boom" in read_episode(tmp_path, bad.id)["error"]

    async def arun():
        async with LiveEpisode(tmp_path, "async-env") as a:
            await a.aevent("turn", n=1)
        return a.id

    aid = asyncio.run(arun())
    assert read_episode(tmp_path, aid)["status"] == "completed"
    # an episode whose writer died reads as abandoned (a child process that exits)
    code = ("import sys; sys.path.insert(0, %r); from wavelet_b200.orchestrator.live import LiveEpisode; "
            "e = LiveEpisode(%r, 'dead'); e.event('episode_started'); print(e.id)") % (str(Path(__file__).resolve().parents[1]), str(tmp_path))
    dead_id = subprocess.run([_sys.executable, "-c", code], capture_output=True, text=True).stdout.strip()
    metas = {m["id"]: m for m in list_episodes(tmp_path)}
    assert metas[dead_id]["abandoned"] and episode_abandoned(metas[dead_id])
    assert not metas[ep.id]["abandoned"]
    # bounded documents and pruning of finished episodes
    with LiveEpisode(tmp_path, "big") as big:
        for i in range(live.MAX_EVENTS + 20):
            big.event("e", i=i)
    assert len(read_episode(tmp_path, big.id)["events"]) <= live.MAX_EVENTS
    assert live.prune_finished(tmp_path / "traces" / "live", keep=1) >= 3
    assert len([m for m in list_episodes(tmp_path) if m["status"] != "running" or m["abandoned"]]) == 1

    class Env:
        def score(self, x):
            return 2.0 * x

    env = install_environment_hooks(Env())
    with LiveEpisode(tmp_path, "hooked") as hk:
        assert env.score(1.5) == 3.0
    assert [e["phase"] for e in read_episode(tmp_path, hk.id)["events"]][-2:] == ["score_started", "score_finished"]
    assert env.score(1.0) == 2.0  # outside an episode: untouched
    st = OrchestratorRunState(tmp_path)
    st.update(status="running", step=4)
    st.event("batch_published", step=4)
    c = TestClient(build_state_app(st))
    assert c.get("/api/state").json()["step"] == 4
    assert c.get("/api/events", params={"after": 0}).json()["events"][0]["event"] == "batch_published"
    assert c.get("/api/events", params={"after": 1}).json()["events"] == []


def test_ray_role_backend_with_a_stand_in_ray(tmp_path, monkeypatch):
    """launcher.backend=ray: roles run as Ray tasks behind the same poll /
    terminate surface (a minimal stand-in for the ray module runs the tasks
    on threads)."""
    import sys
    import threading
    import types

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.orchestrator.launcher import RoleRunner, RoleSpec, wait_for_roles

    calls = {"init": None, "cancel": [], "shutdown": 0}

    class Ref:
        def __init__(self, fn, args):
            self.result = None
            self.t = threading.Thread(target=lambda: setattr(self, "result", fn(*args)), daemon=True)
            self.t.start()

    fake = types.ModuleType("ray")
    fake.remote = lambda fn: types.SimpleNamespace(remote=lambda *a: Ref(fn, a))
    fake.init = lambda **kw: calls.__setitem__("init", kw)

    def wait(refs, timeout=None):
        for r in refs:
            r.t.join(timeout)
        return [r for r in refs if not r.t.is_alive()], [r for r in refs if r.t.is_alive()]

    fake.wait = wait
    fake.get = lambda r: r.result
    fake.cancel = lambda r, force=False: calls["cancel"].append(force)
    fake.shutdown = lambda: calls.__setitem__("shutdown", calls["shutdown"] + 1)
    monkeypatch.setitem(sys.modules, "ray", fake)
    cfg = RLConfig.model_validate({"launcher": {"mode": "process", "backend": "ray", "ray_address": "auto"},
                                   "output_dir": str(tmp_path / "o")})
    runner = RoleRunner(cfg, tmp_path / "logs")
    assert calls["init"]["address"] == "auto"
    py = sys.executable
    ok = runner.start(RoleSpec("rl-trainer", [py, "-c", "print('hi')"]))
    bad = runner.start(RoleSpec("rl-inference", [py, "-c", "import sys; sys.exit(4)"]))
    svc = runner.start(RoleSpec("inference-server-0", [py, "-c", "import time; time.sleep(1.5)"], service=True))
    assert wait_for_roles([ok, bad], [svc], poll=0.05) == 1
    assert ok.poll() == 0 and bad.poll() == 4
    assert False in calls["cancel"]  # the server task was asked to stop
    assert "hi" in (tmp_path / "logs" / "rl-trainer.log").read_text()
    runner.close()
    assert calls["shutdown"] == 1
