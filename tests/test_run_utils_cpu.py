"""Run-directory pathing, per-node telemetry, step-boundary garbage
collection and step-range profiling, against the behaviour the reference's
tests pin (tests/test_pathing.py, test_telemetry.py, test_trainer_gc.py,
test_trainer_profiling.py of the reference)."""

import gc
import json
import os
import tempfile
from pathlib import Path
from unittest.mock import Mock

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wavelet_b200.trainer.gc_control import StepGarbageCollector
from wavelet_b200.trainer.profiling import PhaseTimer, StepProfiler
from wavelet_b200.trainer.telemetry import RankSample, Telemetry, node_metrics, rank_rows
from wavelet_b200.utils import pathing


# ------------------------------------------------------------------ pathing
def test_launch_attempts_keep_configs_commands_and_logs(tmp_path):
    src = tmp_path / "source config.yaml"
    src.write_text("max_steps: 3\n")
    out = tmp_path / "run"
    first = pathing.create_launch_attempt(out)
    pathing.write_launch_artifacts(first, command="rl", argv=["@", str(src)])
    (first.log_dir / "rl_inference.log").write_text("first\n")
    second = pathing.create_launch_attempt(out)
    assert first.config_attempt_dir.name == "attempt_1" and second.config_attempt_dir.name == "attempt_2"
    assert (first.config_attempt_dir / "rl.yaml").read_text() == "max_steps: 3\n"
    assert "source config.yaml" in (first.config_attempt_dir / "command.txt").read_text()
    assert (first.log_dir / "rl_inference.log").read_text() == "first\n"
    assert (out / "configs" / "latest").resolve() == second.config_attempt_dir.resolve()
    assert (out / "logs" / "latest").resolve() == second.log_dir.resolve()
    assert pathing.get_config_dir(out).resolve() == second.config_dir.resolve()


def test_launch_artifacts_copy_each_composed_config(tmp_path):
    a, b = tmp_path / "base.yaml", tmp_path / "overlay.yaml"
    a.write_text("max_steps: 3\n")
    b.write_text("launcher:\n  mode: process\n")
    att = pathing.create_launch_attempt(tmp_path / "run")
    pathing.write_launch_artifacts(att, command="rl", argv=["@", str(a), f"@{b}"])
    assert (att.config_attempt_dir / "rl_1.yaml").read_text() == "max_steps: 3\n"
    assert (att.config_attempt_dir / "rl_2.yaml").read_text() == "launcher:\n  mode: process\n"


def test_output_dir_rules(tmp_path):
    out = tmp_path / "run"
    out.mkdir()
    pathing.validate_output_dir(out, resuming=False, clean=False)  # empty is fine
    (out / "rollouts" / "step-000000").mkdir(parents=True)
    (out / "rollouts" / "step-000000" / "STABLE").touch()
    with pytest.raises(FileExistsError, match="rollouts"):
        pathing.validate_output_dir(out, resuming=False, clean=False)
    pathing.validate_output_dir(out, resuming=True, clean=False)
    assert "rollouts" in pathing.existing_run_state_entries(out)
    with pytest.raises(ValueError, match="cannot be used with checkpoint resume"):
        pathing.validate_output_dir(out, resuming=True, clean=True)
    pathing.validate_output_dir(out, resuming=False, clean=True)
    assert not out.exists()  # nothing but run state was in it


def test_clean_keeps_unrelated_files_and_protected_inputs(tmp_path):
    out = tmp_path / "run"
    (out / "policies" / "step-1" / "adapter").mkdir(parents=True)
    marker = out / "policies" / "step-1" / "adapter" / "adapter_model.safetensors"
    marker.write_text("weights")
    with pytest.raises(ValueError, match="would remove required input"):
        pathing.validate_output_dir(out, resuming=False, clean=True, protected_paths=(marker.parent, None))
    assert marker.read_text() == "weights"
    (out / "notes.txt").write_text("keep")
    (out / "checkpoint-3").mkdir()
    pathing.validate_output_dir(out, resuming=False, clean=True, protected_paths=("Qwen/Qwen3-0.6B",))
    assert sorted(p.name for p in out.iterdir()) == ["notes.txt"]


def test_clean_refuses_working_directory(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    with pytest.raises(ValueError, match="current working directory"):
        pathing.validate_output_dir(tmp_path, resuming=False, clean=True)


def test_resume_resolution(tmp_path):
    for s, stable in ((1, True), (2, True), (3, False)):
        d = pathing.checkpoint_dir(tmp_path, s)
        d.mkdir()
        if stable:
            (d / pathing.STABLE).write_text(str(s))
    assert pathing.list_checkpoint_steps(tmp_path) == [1, 2]
    assert pathing.resolve_resume_dir(tmp_path, -1, None) == pathing.checkpoint_dir(tmp_path, 2)
    assert pathing.resolve_resume_dir(tmp_path, None, None) is None
    with pytest.raises(FileNotFoundError):
        pathing.resolve_resume_dir(tmp_path, 3, None)


# ---------------------------------------------------------------- telemetry
def _rank(r, node, tokens, seconds, peak):
    return RankSample(r, r % 2, node, f"cuda:{r % 2}", tokens, seconds, peak - 3.0, peak)


def test_node_metrics_aggregate_per_node():
    m = node_metrics([_rank(0, "host-a", 600.0, 2.0, 20.0), _rank(1, "host-a", 400.0, 2.5, 21.0),
                      _rank(2, "host-b", 900.0, 2.0, 18.0), _rank(3, "host-b", 1100.0, 2.0, 19.0)])
    assert m["perf/nodes"] == 2.0
    assert m["node/host-a/ranks"] == 2.0 and m["node/host-a/tokens"] == 1000.0
    assert m["node/host-a/tokens_per_second"] == 1000.0 / 2.5  # the slowest rank's time
    assert m["node/host-a/peak_memory_gib"] == 21.0 and m["node/host-a/memory_allocated_gib"] == 18.0
    assert m["node/host-b/tokens_per_second"] == 1000.0
    assert m["perf/rank_tokens_per_second_min"] == 160.0 and m["perf/rank_tokens_per_second_max"] == 550.0
    assert m["perf/rank_peak_memory_gib_max"] == 21.0
    assert node_metrics([]) == {}
    row = rank_rows([_rank(0, "host-a", 600.0, 2.0, 20.0)])[0]
    assert row["rank"] == 0 and row["node"] == "host-a" and row["tokens_per_second"] == 300.0


def test_sample_divides_tokens_by_model_parallel_replication(monkeypatch):
    monkeypatch.setenv("WAVELET_NODE_NAME", "unit/test")
    (s,) = Telemetry(None, replication=2).sample(1000, 4.0)
    assert s.rank == 0 and s.node == "unit_test" and s.tokens == 500.0 and s.tokens_per_second == 125.0


class _World:
    def __init__(self, rank, world):
        self.rank, self.world_size, self.local_rank, self.device = rank, world, rank, torch.device("cpu")


def _telemetry_worker(rank, world, init_file, out):
    os.environ["WAVELET_NODE_NAME"] = "host-a" if rank == 0 else "host-b"
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    samples = Telemetry(_World(rank, world)).sample(100.0 * (rank + 1), 1.0 + rank)
    Path(f"{out}.{rank}").write_text(json.dumps(rank_rows(samples)))
    dist.destroy_process_group()


def test_two_ranks_exchange_samples():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_telemetry_worker, args=(2, os.path.join(d, "init"), os.path.join(d, "res")), nprocs=2, join=True)
        rows = [json.loads(Path(d, f"res.{r}").read_text()) for r in range(2)]
    assert rows[0] == rows[1]
    assert [(r["node"], r["tokens"], r["seconds"]) for r in rows[0]] == [("host-a", 100.0, 1.0), ("host-b", 200.0, 2.0)]


# ----------------------------------------------------------------------- gc
def test_gc_collects_on_interval_and_restores_automatic_gc(monkeypatch):
    was = gc.isenabled()
    gc.enable()
    collect = Mock(return_value=0)
    monkeypatch.setattr(gc, "collect", collect)
    c = StepGarbageCollector(interval=3)
    try:
        assert not gc.isenabled()
        collect.assert_called_once_with(1)
        c.run(1)
        c.run(2)
        collect.assert_called_once_with(1)
        c.run(3)
        assert collect.call_count == 2
    finally:
        c.close()
    assert gc.isenabled()
    if not was:
        gc.disable()


def test_gc_keeps_a_disabled_collector_disabled(monkeypatch):
    was = gc.isenabled()
    gc.disable()
    monkeypatch.setattr(gc, "collect", Mock(return_value=0))
    try:
        StepGarbageCollector(interval=1).close()
        assert not gc.isenabled()
    finally:
        if was:
            gc.enable()
    with pytest.raises(ValueError):
        StepGarbageCollector(interval=0)


# ---------------------------------------------------------------- profiling
def test_step_profiler_traces_the_inclusive_range(tmp_path):
    trace = tmp_path / "trace" / "steps.json"
    p = StepProfiler(trace, start_step=2, end_step=3)
    for step in range(1, 6):
        p.before_step(step)
        assert (p._prof is not None) == (2 <= step <= 3)
        torch.ones(8).add_(1)
        p.after_step(step)
    p.close()
    assert trace.exists() and "traceEvents" in json.loads(trace.read_text())


def test_phase_timer_is_inert_without_cuda():
    t = PhaseTimer(enabled=True)
    t.start("forward")
    t.stop("forward")
    assert t.read() == {} or torch.cuda.is_available()


def test_emit_perf_line_shape(monkeypatch, capsys):
    from wavelet_b200.monitor import emit_perf

    monkeypatch.delenv("WAVELET_PERF_LOG", raising=False)
    emit_perf("example", step=2)
    assert capsys.readouterr().out == ""
    monkeypatch.setenv("WAVELET_PERF_LOG", "1")
    emit_perf("example", step=2, seconds=0.125, mode="async")
    assert capsys.readouterr().out == "WAVELET_PERF example step=2 seconds=0.125 mode=async\n"
