"""Device policy transfer on the CPU: the push segments re-form the full
generator weights from tensor-parallel, expert-parallel and data-parallel
trainer ranks; the exporter -> receiver protocol over in-process buffers
(slots, epochs, the sequence-lock re-copy, a step that never arrives); the
NCCL-fallback broadcast between a trainer process and a generator process
over gloo."""

import dataclasses
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.qwen import build_model
from wavelet_b200.transport.peer_policy import apply_segments, push_segments, used_numel


def _layout(m):
    return dict(m.flat.offsets)


def _same_params(dst, full):
    """Every parameter of ``full`` equals its place in ``dst`` (the flat store
    aligns parameters, so the gaps between them are not compared)."""
    for name, (off, n) in full.flat.offsets.items():
        torch.testing.assert_close(dst[off:off + n], full.flat.compute[off:off + n], rtol=0, atol=0, msg=name)


def _gen(cfg, seed=0):
    return build_model(cfg, "cpu", torch.float32, seed=seed, with_grad=False, with_optimizer=False)


@pytest.mark.parametrize("bias", [False, True])
def test_tp2_segments_rebuild_the_full_weights(bias):
    cfg = PRESETS["tiny"]
    if bias:
        cfg = dataclasses.replace(cfg, arch="qwen2", qkv_bias=True, qk_norm=False)
    full = _gen(cfg, seed=4)
    dst = torch.full_like(full.flat.compute, float("nan"))
    for r in range(2):
        part = build_model(cfg, "cpu", torch.float32, seed=4, tp=(2, r), with_grad=False, with_optimizer=False)
        for src, segs in push_segments(part, _layout(full), rank=r, world=2).items():
            assert src == "flat"
            apply_segments(part.flat.compute, segs, dst)
    _same_params(dst, full)


def test_dp_replicas_split_the_work_without_overlap():
    cfg = PRESETS["tiny"]
    full = _gen(cfg, seed=2)
    seen = torch.zeros(full.flat.compute.numel(), dtype=torch.int32)
    for r in range(3):
        for segs in push_segments(full, _layout(full), rank=r, world=3).values():
            for so, do, rows, n, ss, ds in segs:
                assert so == do and rows == 1
                seen[do:do + n] += 1
    assert int(seen.max()) == 1
    for off, n in full.flat.offsets.values():
        assert int(seen[off:off + n].min()) == 1


def test_ep2_with_expert_dp_rebuilds_the_experts():
    cfg = PRESETS["tiny-moe"]
    full = _gen(cfg, seed=6)
    dst = torch.full_like(full.flat.compute, float("nan"))
    world, ep = 4, 2  # ranks (ep_rank, ep_dp_rank): 0 -> (0, 0), 1 -> (1, 0), 2 -> (0, 1), 3 -> (1, 1)
    for rank in range(world):
        er, edr = rank % ep, rank // ep
        part = build_model(cfg, "cpu", torch.float32, seed=6, ep=(ep, er, edr, world // ep), with_grad=False,
                           with_optimizer=False)
        segs = push_segments(part, _layout(full), rank=rank, world=world)
        src = {"flat": part.flat.compute, "expert": part.expert_flat.compute}
        for k, v in segs.items():
            apply_segments(src[k], v, dst)
    _same_params(dst, full)


def test_lora_trainers_are_refused():
    cfg = PRESETS["tiny"]
    lora = type("L", (), {"rank": 4, "alpha": 8.0, "target_modules": ["q_proj"], "dropout": 0.0})()
    m = build_model(cfg, "cpu", torch.float32, seed=0, lora=lora)
    with pytest.raises(NotImplementedError, match="filesystem"):
        push_segments(m, _layout(_gen(cfg)))


def _pt_cfg(**kw):
    from wavelet_b200.configs.config import RLPolicyTransferConfig

    return RLPolicyTransferConfig(**{"type": "nccl", "nccl_timeout_seconds": 5, **kw})


def test_exporter_to_receiver_over_in_process_slots(tmp_path):
    from wavelet_b200.transport.policy import DevicePolicyReceiver, PolicyExporter, load_policy_into
    from wavelet_b200.transport.queue import STABLE, step_dir

    cfg = PRESETS["tiny"]
    gen = _gen(cfg, seed=1)
    pt = _pt_cfg(peer_slots=2)
    rec = DevicePolicyReceiver(gen, tmp_path, pt, index=0)
    assert (tmp_path / "policies" / "peer" / "receiver-0.json").exists() or rec.peer.path.exists()
    trainer = build_model(cfg, "cpu", torch.float32, seed=7)
    exp = PolicyExporter(tmp_path, pt, rank=0)
    for step in (1, 2, 3):
        with torch.no_grad():
            trainer.flat.compute.add_(0.01 * step)
        d = exp.export(trainer, step)
        assert exp.device_mode == "peer" and (d / STABLE).exists()
        info = json.loads((d / "update_info.json").read_text())
        assert info["protocol"] == "peer_v1" and info["slot"] == step % 2 and info["epoch"] == step + 1
        meta = load_policy_into(gen, d, rec, step)
        assert meta["loaded_step"] == step
        _same_params(gen.flat.compute, trainer)
    assert sorted(rec.peer.epochs()) == [3, 4]
    # a generator asking for an older step gets the newest complete one
    assert rec.peer.load(1, timeout_s=1) == 3
    # sequence lock: the slot's epoch changes during the copy -> copy again
    calls = {"n": 0}
    real = rec.peer.epochs

    def flaky():
        calls["n"] += 1
        e = real()
        return [x + 10 for x in e] if calls["n"] == 2 else e

    rec.peer.epochs = flaky
    assert rec.peer.load(3, timeout_s=1) >= 3 and calls["n"] >= 4
    rec.peer.epochs = real
    with pytest.raises(TimeoutError, match="did not arrive"):
        rec.peer.load(9, timeout_s=0.05)
    exp.close()
    rec.close()
    assert not rec_path_exists(tmp_path)
    # a device snapshot without a receiver is an error, not a silent no-op
    with pytest.raises(RuntimeError, match="device receiver"):
        load_policy_into(gen, step_dir(tmp_path / "policies", 3))


def rec_path_exists(tmp_path):
    return any((tmp_path / "policies" / "peer").glob("receiver-*.json"))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_fallback_worker(role, out_dir, port, res):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    from pathlib import Path

    from wavelet_b200.transport.policy import DevicePolicyReceiver, PolicyExporter, load_policy_into
    from wavelet_b200.transport.queue import STABLE, step_dir

    cfg = PRESETS["tiny"]
    pt = _pt_cfg(peer=False, nccl_port=port, nccl_inference_world_size=1, nccl_timeout_seconds=60)
    out = Path(out_dir)
    if role == 0:
        trainer = build_model(cfg, "cpu", torch.float32, seed=11)
        exp = PolicyExporter(out, pt, rank=0)
        exp.export(trainer, 5)
        torch.save({"w": trainer.flat.compute[:used_numel(trainer.flat)].clone(), "mode": exp.device_mode}, f"{res}.0")
        exp.close()
    else:
        gen = _gen(cfg, seed=0)
        rec = DevicePolicyReceiver(gen, out, pt, index=0)
        d = step_dir(out / "policies", 5)
        import time

        t0 = time.monotonic()
        while not (d / STABLE).exists() and time.monotonic() - t0 < 60:
            time.sleep(0.02)
        meta = load_policy_into(gen, d, rec, 5)
        torch.save({"w": gen.flat.compute[:used_numel(gen.flat)].clone(), "step": meta["loaded_step"]}, f"{res}.1")
        rec.close()


def test_nccl_fallback_broadcast_between_processes(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    res = str(tmp_path / "res")
    ps = [ctx.Process(target=_nccl_fallback_worker, args=(r, str(tmp_path / "run"), port, res)) for r in (0, 1)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    a, b = torch.load(f"{res}.0"), torch.load(f"{res}.1")
    assert a["mode"] == "nccl" and b["step"] == 5
    torch.testing.assert_close(b["w"], a["w"], rtol=0, atol=0)


def test_launcher_keeps_every_gpu_visible_for_device_transfer(tmp_path):
    """Device transfer between processes: each role sees its own GPUs first
    and every other GPU of the placement (an IPC handle opens only where the
    owning GPU is visible); every generator knows its replica index and the
    trainer expects one receiver per replica."""
    import yaml

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.orchestrator.launcher import build_roles
    from wavelet_b200.utils.pathing import LaunchAttempt

    def roles(transfer):
        cfg = RLConfig.model_validate({
            "output_dir": str(tmp_path / "o"), "policy_transfer": {"type": transfer},
            "inference": {"mode": "vllm_http"},
            "launcher": {"mode": "process", "trainer_num_processes": 2, "inference_num_replicas": 2,
                         "trainer_cuda_visible_devices": "0,1", "inference_cuda_visible_devices": "2,3"}})
        att = LaunchAttempt(tmp_path / "a", tmp_path / "a" / "cfg", tmp_path / "a" / "logs")
        att.config_dir.mkdir(parents=True, exist_ok=True)
        return build_roles(cfg, att)

    services, main = roles("nccl")
    envs = {r.name: r.env for r in services + main}
    assert envs["inference-server-0"]["CUDA_VISIBLE_DEVICES"] == "2,0,1,3"
    assert envs["inference-server-1"]["CUDA_VISIBLE_DEVICES"] == "3,0,1,2"
    assert envs["inference-server-1"]["WAVELET_INFERENCE_REPLICA"] == "1"
    tr = [r for r in main if r.name == "rl-trainer"][0]
    assert tr.env["CUDA_VISIBLE_DEVICES"] == "0,1,2,3"
    conf = yaml.safe_load((tmp_path / "a" / "cfg" / "rl_trainer.yaml").read_text())
    assert conf["policy_transfer"]["nccl_inference_world_size"] == 2
    services, main = roles("filesystem")
    assert {r.name: r.env for r in services}["inference-server-1"]["CUDA_VISIBLE_DEVICES"] == "3"
