"""Process-mode placement, the run-directory contract and step-boundary GC
(ref orchestrator/placement.py, utils/pathing.py, trainer/garbage_collection.py;
behaviours from the reference's launcher and pathing tests)."""

from __future__ import annotations

import gc
import os

import pytest

from wavelet_b200.configs.config import RLConfig


def _cfg(**launcher):
    http = launcher.pop("http", {})
    return RLConfig.model_validate({"launcher": {"mode": "process", **launcher},
                                    "inference": {"http": {"host": "127.0.0.1", "port": 8200, **http}}})


# ------------------------------------------------------------------ placement
def test_default_split_gives_trainer_the_first_gpus():
    from wavelet_b200.orchestrator.placement import plan

    p = plan(_cfg(trainer_num_processes=4, inference_num_replicas=2), [str(i) for i in range(8)])
    assert p.trainer_devices == ["0", "1", "2", "3"]
    assert p.inference_devices == [["4", "5"], ["6", "7"]]
    assert p.ports == [8200, 8201] and p.host == "127.0.0.1"


def test_explicit_devices_and_overlap():
    from wavelet_b200.orchestrator.placement import plan

    avail = [str(i) for i in range(8)]
    p = plan(_cfg(trainer_num_processes=2, inference_cuda_visible_devices="6,7", inference_num_replicas=2), avail)
    assert p.trainer_devices == ["0", "1"] and p.inference_devices == [["6"], ["7"]]
    p = plan(_cfg(trainer_num_processes=2, trainer_cuda_visible_devices=["4", "5"]), avail)
    assert p.trainer_devices == ["4", "5"] and p.inference_devices == [["0", "1", "2", "3", "6", "7"]]
    with pytest.raises(ValueError, match="overlap"):
        plan(_cfg(trainer_num_processes=2, trainer_cuda_visible_devices="0,1",
                  inference_cuda_visible_devices="1,2"), avail)
    with pytest.raises(ValueError, match="trainer_num_processes=2 but 3"):
        plan(_cfg(trainer_num_processes=2, trainer_cuda_visible_devices="0,1,2"), avail)


def test_too_few_gpus_and_ports():
    from wavelet_b200.orchestrator.placement import plan

    with pytest.raises(ValueError, match="only 2 are visible"):
        plan(_cfg(trainer_num_processes=2, inference_num_replicas=1), ["0", "1"])
    with pytest.raises(ValueError, match="one port per replica"):
        plan(_cfg(inference_num_replicas=2, http={"ports": [9000]}), [str(i) for i in range(4)])
    p = plan(_cfg(inference_num_replicas=2, http={"ports": [9000, 9005]}), [str(i) for i in range(4)])
    assert p.ports == [9000, 9005]


def test_colocate_shares_the_trainer_gpus():
    from wavelet_b200.orchestrator.placement import plan

    for mode in ("colocate", "colocate_sleep"):
        p = plan(_cfg(mode=mode, trainer_num_processes=2, inference_num_replicas=2), [str(i) for i in range(8)])
        assert p.trainer_devices == ["0", "1"] and p.inference_devices == [["0"], ["1"]]
    # one trainer GPU cannot hold two replicas
    with pytest.raises(ValueError, match="not enough inference devices"):
        plan(_cfg(mode="colocate", trainer_num_processes=1, inference_num_replicas=2), ["0", "1"])


def test_cpu_host_runs_roles_unpinned(monkeypatch):
    from wavelet_b200.orchestrator.placement import plan, visible_devices

    p = plan(_cfg(inference_num_replicas=2), [])
    assert p.trainer_devices == [] and p.inference_devices == [[], []] and p.ports == [8200, 8201]
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert visible_devices() == ["3", "5"]


# ------------------------------------------------------------------ run directory
def test_launch_attempts_count_up_and_repoint_latest(tmp_path):
    from wavelet_b200.utils.pathing import create_launch_attempt, get_config_dir, write_launch_artifacts

    a1 = create_launch_attempt(tmp_path)
    a2 = create_launch_attempt(tmp_path)
    assert a1.config_attempt_dir.name == "attempt_1" and a2.config_attempt_dir.name == "attempt_2"
    assert os.readlink(tmp_path / "configs" / "latest") == "attempt_2"
    assert os.readlink(tmp_path / "logs" / "latest") == "attempt_2"
    assert get_config_dir(tmp_path) == tmp_path / "configs" / "latest" / "resolved"
    cfg = tmp_path / "rl.yaml"
    cfg.write_text("max_steps: 3\n")
    write_launch_artifacts(a2, command="rl", argv=["@", str(cfg), "--max-steps", "4"])
    assert (a2.config_attempt_dir / "rl.yaml").read_text() == "max_steps: 3\n"
    assert "wavelet rl @" in (a2.config_attempt_dir / "command.txt").read_text()


def test_output_dir_guard_clean_and_resume(tmp_path, monkeypatch):
    from wavelet_b200.utils.pathing import validate_output_dir

    run = tmp_path / "run"
    (run / "rollouts").mkdir(parents=True)
    (run / "checkpoint-3").mkdir()
    (run / "notes.txt").write_text("keep me")
    with pytest.raises(FileExistsError, match="rollouts, checkpoint-3"):
        validate_output_dir(run, clean=False, resuming=False)
    validate_output_dir(run, clean=False, resuming=True)  # resuming keeps everything
    with pytest.raises(ValueError, match="cannot be used with checkpoint resume"):
        validate_output_dir(run, clean=True, resuming=True)
    model = run / "model"
    model.mkdir()
    with pytest.raises(ValueError, match="required input"):
        validate_output_dir(run, clean=True, resuming=False, protected_paths=[model])
    model.rmdir()
    validate_output_dir(run, clean=True, resuming=False)
    assert sorted(p.name for p in run.iterdir()) == ["notes.txt"]  # unrelated files stay
    monkeypatch.chdir(run)
    with pytest.raises(ValueError, match="current working directory"):
        validate_output_dir(run, clean=True, resuming=False)


def test_checkpoint_listing_and_resume_resolution(tmp_path):
    from wavelet_b200.utils.pathing import latest_checkpoint_step, list_checkpoint_steps, resolve_resume_dir

    for s, stable in ((2, True), (5, True), (7, False)):
        d = tmp_path / f"checkpoint-{s}"
        d.mkdir()
        if stable:
            (d / "STABLE").touch()
    assert list_checkpoint_steps(tmp_path) == [2, 5]
    assert list_checkpoint_steps(tmp_path, stable_only=False) == [2, 5, 7]
    assert latest_checkpoint_step(tmp_path) == 5
    assert resolve_resume_dir(tmp_path, -1, None) == tmp_path / "checkpoint-5"
    assert resolve_resume_dir(tmp_path, 2, None) == tmp_path / "checkpoint-2"
    assert resolve_resume_dir(tmp_path, None, None) is None
    with pytest.raises(FileNotFoundError, match="not STABLE"):
        resolve_resume_dir(tmp_path, 7, None)
    with pytest.raises(FileNotFoundError, match="no stable checkpoint"):
        resolve_resume_dir(tmp_path / "empty", -1, None)


# ------------------------------------------------------------------ garbage collection
def test_step_gc_collects_on_the_interval_and_restores_gc(monkeypatch):
    from wavelet_b200.trainer.gc_control import StepGarbageCollector

    was = gc.isenabled()
    calls = []
    monkeypatch.setattr(gc, "collect", lambda gen=2: calls.append(gen) or 0)
    try:
        gc.enable()
        g = StepGarbageCollector(3)
        assert not gc.isenabled() and calls == [1]  # one collection at start
        for step in range(0, 10):
            g.run(step)
        assert calls == [1, 1, 1, 1]  # steps 3, 6, 9
        g.close()
        assert gc.isenabled()
        g.close()  # idempotent
        with pytest.raises(ValueError, match="positive"):
            StepGarbageCollector(0)
    finally:
        (gc.enable if was else gc.disable)()


def test_phase_timer_is_off_without_cuda(monkeypatch):
    import torch

    from wavelet_b200.trainer.profiling import PhaseTimer

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    t = PhaseTimer(True)  # CUDA-event timing: nothing to record on a CPU host
    t.start("x")
    t.stop("x")
    assert not t.enabled and t.read() == {}
