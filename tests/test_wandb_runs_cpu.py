"""W&B run lifecycle through a stand-in ``wandb`` module (ref monitor.py:555-640,
orchestrator/runtime.py:559-585): the persisted run id, resume of the same
run, the shared run of process-mode roles, and the offline fallback."""

from __future__ import annotations

import sys
import types

import pytest

from wavelet_b200.configs.config import RLConfig, WandbConfig
from wavelet_b200.monitor import RunMonitor, finish_shared_wandb_run, shared_wandb_environment


class _Run:
    def __init__(self, kw):
        self.kw = kw
        self.id = kw.get("id") or "run123"
        self.logged = []
        self.defined = []
        self.finished = None

    def define_metric(self, name, step_metric=None):
        self.defined.append((name, step_metric))

    def log(self, row):
        self.logged.append(row)

    def finish(self, exit_code=0):
        self.finished = exit_code


@pytest.fixture
def fake_wandb(monkeypatch):
    mod = types.ModuleType("wandb")
    mod.inits = []
    mod.fail_online = False

    class Settings:
        def __init__(self, **kw):
            self.kw = kw

    def init(**kw):
        mod.inits.append(kw)
        if mod.fail_online and kw.get("mode") == "online":
            raise ConnectionError("no network")
        run = _Run(kw)
        mod.runs.append(run)
        return run

    mod.runs = []
    mod.Settings = Settings
    mod.init = init
    monkeypatch.setitem(sys.modules, "wandb", mod)
    for k in ("WANDB_SHARED_MODE", "WANDB_RUN_ID", "WANDB_SHARED_LABEL", "WANDB_MODE"):
        monkeypatch.delenv(k, raising=False)
    return mod


def _mon(tmp_path, **w):
    return RunMonitor(tmp_path, log_cuda_memory=False, log_disk_usage=False,
                      wandb=WandbConfig(enabled=True, create_overview=False, **w))


def test_run_id_is_persisted_and_a_resumed_run_continues_it(tmp_path, fake_wandb):
    m = _mon(tmp_path, mode="offline", project="p")
    m.start_run(run_config={"a": 1})
    first = fake_wandb.inits[-1]
    assert first["id"] is None and first["resume"] is None and first["mode"] == "offline"
    assert (tmp_path / "wandb_run_id.txt").read_text() == "run123"
    assert ("*", "step") in fake_wandb.runs[-1].defined  # metrics plotted against the step
    m.log({"loss": 1.0}, 3)
    assert fake_wandb.runs[-1].logged[-1]["loss"] == 1.0 and fake_wandb.runs[-1].logged[-1]["step"] == 3
    m.finish(status="completed", step=3)
    (tmp_path / "wandb_run_id.txt").write_text("abc999")
    m2 = _mon(tmp_path, mode="offline", project="p")
    m2.start_run(run_config={"a": 1}, resumed_from=str(tmp_path / "checkpoint-3"))
    assert fake_wandb.inits[-1]["id"] == "abc999" and fake_wandb.inits[-1]["resume"] == "allow"


def test_online_failure_falls_back_to_an_offline_run(tmp_path, fake_wandb):
    fake_wandb.fail_online = True
    m = _mon(tmp_path, mode="online")
    m.start_run(run_config={})
    assert [k.get("mode") for k in fake_wandb.inits] == ["online", "offline"]
    assert m._wandb is not None and fake_wandb.inits[-1]["id"] is None
    events = (tmp_path / "events.jsonl").read_text()
    assert "wandb_init_failed" in events and "offline" in events
    m3 = _mon(tmp_path / "b", mode="online", offline_fallback=False)
    with pytest.raises(ConnectionError):
        m3.start_run(run_config={})


def test_shared_run_of_process_roles(tmp_path, fake_wandb, monkeypatch):
    cfg = RLConfig.model_validate({"monitor": {"wandb": {"enabled": True, "mode": "online", "project": "p"}},
                                   "output_dir": str(tmp_path / "run")})
    env = shared_wandb_environment(cfg)
    assert env["WANDB_SHARED_MODE"] == "1" and len(env["WANDB_RUN_ID"]) == 8
    assert (tmp_path / "run" / "wandb_run_id.txt").read_text() == env["WANDB_RUN_ID"]
    # a role joins the shared run with its label; the orchestrator is the primary
    for k, v in {**env, "WANDB_SHARED_LABEL": "orchestrator"}.items():
        monkeypatch.setenv(k, v)
    m = _mon(tmp_path / "run", mode="online")
    m.start_run(run_config={})
    kw = fake_wandb.inits[-1]
    assert kw["id"] == env["WANDB_RUN_ID"] and kw["resume"] == "allow" and "mode" not in kw
    st = kw["settings"].kw
    assert st["mode"] == "shared" and st["x_label"] == "orchestrator" and st["x_primary"] is True
    monkeypatch.setenv("WANDB_SHARED_LABEL", "trainer")
    _mon(tmp_path / "run", mode="online").start_run(run_config={})
    assert fake_wandb.inits[-1]["settings"].kw["x_primary"] is False
    # the launcher finishes the shared run with the roles' exit code
    finish_shared_wandb_run(cfg, env, exit_code=3)
    assert fake_wandb.runs[-1].finished == 3 and fake_wandb.inits[-1]["settings"].kw["x_label"] == "launcher"
    # offline runs and runs without W&B get no shared environment
    off = cfg.model_copy(update={"monitor": cfg.monitor.model_copy(update={
        "wandb": cfg.monitor.wandb.model_copy(update={"mode": "offline"})})})
    assert shared_wandb_environment(off) == {}


def test_launcher_roles_carry_the_shared_run(tmp_path, fake_wandb):
    from wavelet_b200.orchestrator.launcher import build_roles
    from wavelet_b200.utils.pathing import create_launch_attempt

    cfg = RLConfig.model_validate({"launcher": {"mode": "process"}, "output_dir": str(tmp_path / "run"),
                                   "monitor": {"wandb": {"enabled": True, "mode": "online"}}})
    env = shared_wandb_environment(cfg)
    services, jobs = build_roles(cfg, create_launch_attempt(tmp_path / "run"), shared_wandb=env)
    labels = {j.name: j.env.get("WANDB_SHARED_LABEL") for j in jobs}
    assert labels == {"rl-trainer": "trainer", "rl-inference": "orchestrator"}
    assert all(j.env["WANDB_RUN_ID"] == env["WANDB_RUN_ID"] for j in jobs)
