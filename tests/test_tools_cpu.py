"""CLI tools, dashboard API, SLURM rendering and trace conversion on CPU."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_dashboard_api_over_synthetic_run(tmp_path):
    from fastapi.testclient import TestClient

    from wavelet_b200.dashboard.server import RunRegistry, build_app, default_static_dir
    from wavelet_b200.dashboard.synth import write_synthetic_run

    write_synthetic_run(tmp_path / "runA", steps=30, ranks=4)
    app = build_app(RunRegistry([tmp_path]), default_static_dir())
    c = TestClient(app)
    assert c.get("/api/health").json()["ok"]
    runs = c.get("/api/runs").json()["runs"]
    assert runs[0]["run_id"] == "runA" and runs[0]["status"] == "completed"
    keys = c.get("/api/runs/runA/metrics/keys").json()
    assert "loss" in keys["trainer"] and "reward/mean" in keys["orchestrator"]
    s = c.get("/api/runs/runA/series", params={"keys": "loss", "points": 10}).json()
    assert 0 < len(s["steps"]) <= 12 and len(s["series"]["loss"]) == len(s["steps"])
    assert max(s["series"]["loss"]) == max(json.loads(l)["loss"] for l in (tmp_path / "runA/metrics.jsonl").read_text().splitlines())
    assert c.get("/api/runs/runA/series", params={"keys": "nope"}).status_code == 400
    assert len(c.get("/api/runs/runA/nodes").json()["ranks"]) == 4
    q = c.get("/api/runs/runA/queue").json()
    assert q["published"] == 30 and q["consumed"] == 30
    rows = c.get("/api/runs/runA/rollouts/rows", params={"step": 3}).json()
    assert rows["total"] == 4
    assert c.get("/api/runs/runA/evals").json()["metrics"]
    assert "trainer.log" in c.get("/api/runs/runA/logs").json()["logs"]
    assert "step 30" in c.get("/api/runs/runA/logs/trainer.log").text
    assert c.get("/api/runs/runA/logs/..%2F..%2Fetc%2Fpasswd").status_code == 404
    assert c.get("/").status_code == 200
    # incremental tail: a new row appears without reopening
    with open(tmp_path / "runA/metrics.jsonl", "a") as f:
        f.write(json.dumps({"step": 31, "loss": 0.1}) + "\n")
    s2 = c.get("/api/runs/runA/series", params={"keys": "loss", "after": 30}).json()
    assert s2["steps"] == [31.0]


def test_trace_conversion(tmp_path):
    from wavelet_b200.orchestrator.trace import TraceWriter
    from wavelet_b200.tools.convert_traces import main

    tw = TraceWriter(tmp_path / "run", "orchestrator")
    tw.event("batch_published", step=3, policy_step=2, path="x")
    tw.event("rollout", step=3, rollout_id="3:0", reward=1.0)
    assert main([str(tmp_path / "run"), "--output-dir", str(tmp_path / "ds")]) == 0
    import pyarrow.parquet as pq

    t = pq.read_table(tmp_path / "ds" / "default" / "train-00000-of-00001.parquet").to_pylist()
    assert [r["event"] for r in t] == ["batch_published", "rollout"]
    assert json.loads(t[1]["payload"])["reward"] == 1.0 and t[0]["policy_step"] == 2


def test_slurm_render_and_nodelist(tmp_path):
    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.deployment.slurm import expand_nodelist, plan_roles, render_sbatch
    from wavelet_b200.utils.config import load_yaml

    assert expand_nodelist("gpu[01-03,07],login1") == ["gpu01", "gpu02", "gpu03", "gpu07", "login1"]
    cfg = RLConfig.model_validate({"output_dir": str(tmp_path), "slurm": {"partition": "p", "time_limit": "1:00:00"},
                                   "deployment": {"type": "multi_node", "num_train_nodes": 2,
                                                  "num_inference_nodes": 1, "gpus_per_node": 8,
                                                  "inference_replicas_per_node": 2},
                                   "launcher": {"mode": "process"}, "max_steps": 3})
    script = render_sbatch(cfg, "rl", ["@", "x.yaml"])
    assert "#SBATCH --nodes=3" in script and "#SBATCH --partition=p" in script and "slurm-worker rl" in script
    roles = plan_roles(cfg, "rl", ["n0", "n1", "n2"], tmp_path)
    names = [r.name for r in roles]
    assert names == ["inference_server_0", "inference_server_1", "trainer", "rl_inference"]
    s0, s1, tr, ri = roles
    assert s0.service and s0.endpoint == "http://n2:8000" and s1.endpoint == "http://n2:8001"
    assert "--nodelist=n2" in s0.argv and "--gpus-per-task=4" in s0.argv
    assert "--nodelist=n0,n1" in tr.argv and "--nnodes=2" in tr.argv and "--nproc-per-node=8" in tr.argv
    assert "--rdzv-endpoint=n0:29500" in tr.argv and "rl-trainer" in tr.argv
    assert ri.env["CUDA_VISIBLE_DEVICES"] == "" and "srun" not in ri.argv
    ic = load_yaml(tmp_path / "rl_inference.yaml")
    assert ic["inference"]["http"]["hosts"] == ["n2", "n2"] and ic["inference"]["http"]["ports"] == [8000, 8001]
    assert "slurm" not in ic and ic["deployment"]["type"] == "single_node"
    sc = load_yaml(tmp_path / "inference_server_1.yaml")
    assert sc["inference"]["http"]["host"] == "0.0.0.0" and sc["inference"]["http"]["port"] == 8001
    with pytest.raises(RuntimeError, match="needs 3"):
        plan_roles(cfg, "rl", ["n0", "n1"], tmp_path)


def test_slurm_controller_lifecycle(tmp_path):
    """Servers first, health wait, then jobs; a failing job tears everything
    down; a server dying before health fails fast; success terminates the
    servers."""
    import sys as _sys
    import time as _time

    from wavelet_b200.deployment.slurm import RoleLaunch, run_roles

    py = _sys.executable
    server = RoleLaunch("server", [py, "-c", "import time; time.sleep(60)"], service=True, endpoint="http://x:1")
    ok_job = RoleLaunch("trainer", [py, "-c", "import time; time.sleep(0.3)"])
    ok_job2 = RoleLaunch("rl_inference", [py, "-c", "pass"])
    bad_job = RoleLaunch("trainer", [py, "-c", "import sys; sys.exit(3)"])
    calls = []

    def healthy(urls, t):
        calls.append(list(urls))

    t0 = _time.monotonic()
    assert run_roles([server, ok_job, ok_job2], tmp_path / "a", health=healthy, poll=0.05) == 0
    assert calls == [["http://x:1"]] and _time.monotonic() - t0 < 20
    assert run_roles([server, bad_job, ok_job2], tmp_path / "b", health=healthy, poll=0.05) == 1
    dying = RoleLaunch("server", [py, "-c", "import sys; sys.exit(2)"], service=True, endpoint="http://x:1")

    def never(urls, t):
        _time.sleep(0.1)
        raise TimeoutError

    assert run_roles([dying, ok_job], tmp_path / "c", health=never, startup_timeout=30, poll=0.05) == 1
    assert (tmp_path / "a" / "trainer.log").exists()


@pytest.mark.integration
def test_convert_checkpoint_and_benchmark_compare(tmp_path):
    import os

    out = tmp_path / "out"
    cfg = tmp_path / "sft.yaml"
    cfg.write_text((ROOT / "examples" / "tiny_cpu" / "sft.yaml").read_text().replace("outputs/tiny_cpu_sft", str(out))
                   .replace("max_steps: 10", "max_steps: 3") + "ckpt:\n  mode: async\n  interval: 3\n")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "convert-checkpoint", str(out / "checkpoint-3"),
                        str(tmp_path / "hf"), "--dtype", "float32"], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert (tmp_path / "hf" / "config.json").exists() and list((tmp_path / "hf").glob("*.safetensors"))
    from wavelet_b200.tools.benchmark import aggregate, compare

    res = aggregate(out, warmup_steps=1)
    assert res["steps"] == 2 and res["tokens_per_second"]["median"] > 0
    worse = json.loads(json.dumps(res))
    worse["tokens_per_second"]["median"] *= 0.5
    lines, bad = compare(worse, res, 0.05)
    assert bad and "REGRESSION" in "\n".join(lines)


def test_debug_preflight_and_trainer_inspect(tmp_path, capsys):
    from wavelet_b200.debug import build_preflight_report, inspect_rollout_batch, main
    from wavelet_b200.configs.config import RLConfig

    ok = build_preflight_report(RLConfig.model_validate({"output_dir": str(tmp_path / "o"), "model": {"name": "tiny"},
                                                         "data": {"source": "fake"}}))
    assert ok["ok"], ok["checks"]
    bad = build_preflight_report(RLConfig.model_validate({
        "output_dir": str(tmp_path / "o"), "model": {"name": "tiny"}, "algo": {"type": "grpo"}, "data": {"source": "fake"},
        "orchestrator": {"rollouts_per_example": 1}}))
    assert not bad["ok"] and any(c["name"] == "grpo_group" for c in bad["checks"])
    assert main(["preflight", "--json", "--output-dir", str(tmp_path / "o"), "--model.name", "tiny",
                 "--data.source", "fake"]) == 0
    nf = build_preflight_report(RLConfig.model_validate({"output_dir": str(tmp_path / "o"), "data": {"source": "local"},
                                                         "model": {"name": "tiny"}}))
    assert any(c["name"] == "data_paths" and c["status"] == "error" for c in nf["checks"])
    # a rollout batch with a misaligned mask is flagged
    d = tmp_path / "step-000000"
    d.mkdir()
    rows = [{"prompt": [], "completion": [], "advantage": 0.5, "reward": 1.0, "input_ids": [1, 2, 3],
             "loss_mask": [False, True, True], "inference_logprobs": [-0.1, -0.2]},
            {"prompt": [], "completion": [], "advantage": 0.5, "reward": 1.0, "input_ids": [1, 2, 3],
             "loss_mask": [False, True]}]
    (d / "rollouts.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    rep = inspect_rollout_batch(d)
    assert rep["rows"] == 2 and not rep["ok"] and rep["issues"][0]["row"] == 1


def test_dashboard_page_routes_all_answer(tmp_path):
    """Every API route the single-page dashboard calls answers for a run, and
    series carry timestamps for the elapsed-time axis."""
    import re as _re

    from fastapi.testclient import TestClient

    from wavelet_b200.dashboard.server import RunRegistry, build_app, default_static_dir
    from wavelet_b200.dashboard.synth import write_synthetic_run

    write_synthetic_run(tmp_path / "runB", steps=12, ranks=2)
    c = TestClient(build_app(RunRegistry([tmp_path]), default_static_dir()))
    page = c.get("/").text
    used = set(_re.findall(r"\$\{API\}/runs/\$\{encodeURIComponent\(S\.run\)\}/([a-z/]+)", page))
    assert {"summary", "metrics/keys", "rollouts", "rollouts/rows", "evals", "episodes", "nodes", "logs", "config",
            "timeline"} <= used | {"rollouts/rows"}
    for route in sorted(used):
        params = {"step": 3} if route == "rollouts/rows" else {}
        if route.endswith("/"):
            continue
        assert c.get(f"/api/runs/runB/{route}", params=params).status_code == 200, route
    s = c.get("/api/runs/runB/series", params={"keys": "loss", "points": 50}).json()
    assert len(s["times"]) == len(s["steps"]) and s["times"][0]
    assert c.get("/api/current").json()["run"] == "runB"


def test_orchestrator_live_episodes_reach_the_dashboard(tmp_path):
    """With orchestrator.live_traces on, each prompt group being generated has
    a live episode document; the dashboard lists and serves them."""
    from fastapi.testclient import TestClient

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.dashboard.server import RunRegistry, build_app, default_static_dir
    from wavelet_b200.dashboard.synth import write_synthetic_run
    from wavelet_b200.orchestrator.rollouts import PromptRecord, RLOrchestrator

    run = tmp_path / "runL"
    write_synthetic_run(run, steps=3, ranks=1)
    cfg = RLConfig.model_validate({"output_dir": str(run),
                                   "orchestrator": {"examples_per_step": 2, "rollouts_per_example": 2}})

    orch = RLOrchestrator(cfg, engine=None, sender=None, prompts=None)
    prompts = [PromptRecord([1, 2, 3], example_id="p0"), PromptRecord([4, 5], example_id="p1")]
    eps = orch._live_episodes(prompts, 7)
    assert len(eps) == 2
    for ep in eps:
        ep.finish("completed")
    c = TestClient(build_app(RunRegistry([tmp_path]), default_static_dir()))
    listed = c.get("/api/runs/runL/live").json()["episodes"]
    assert {e["example_id"] for e in listed} == {"p0", "p1"} and all(e["step"] == 7 for e in listed)
    doc = c.get(f"/api/runs/runL/live/{listed[0]['id']}").json()
    assert doc["events"][0]["phase"] == "episode_started"
    assert c.get("/api/runs/runL/live/nothere").status_code == 404
    off = RLOrchestrator(RLConfig.model_validate({"output_dir": str(run), "orchestrator": {"live_traces": False}}),
                         engine=None, sender=None, prompts=None)
    assert off._live_episodes(prompts, 8) == []
