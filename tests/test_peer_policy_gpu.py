"""Device policy push on the GPU: the policy_push kernel against the torch
view copy for every dtype pair (vector and scalar paths, several
destinations), its bounds check, the exporter -> receiver flow inside one
process, and a trainer process pushing into a generator process's receive
slots through CUDA IPC (one GPU, host-side waits only)."""

import json
import os
import random
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

from wavelet_b200 import ops  # noqa: E402
from wavelet_b200.transport.peer_policy import apply_segments  # noqa: E402


def _segments(rng, n_src, aligned, count=40):
    a = 8 if aligned else 1
    segs, dst_off = [], 0
    for _ in range(count):
        rows = rng.randint(1, 6)
        row_len = a * rng.randint(1, 40)
        ss = row_len + a * rng.randint(0, 5)
        ds = row_len + a * rng.randint(0, 5)
        so = a * rng.randint(0, (n_src - (rows - 1) * ss - row_len) // a)
        segs.append((so, dst_off, rows, row_len, ss, ds))
        dst_off += (rows - 1) * ds + row_len + a * rng.randint(0, 3)
    return segs, dst_off


@pytest.mark.parametrize("src_dtype,dst_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                                 (torch.bfloat16, torch.float32), (torch.float32, torch.bfloat16)])
@pytest.mark.parametrize("aligned", [True, False])
def test_policy_push_matches_view_copy(src_dtype, dst_dtype, aligned):
    m = ops.ext()
    rng = random.Random(hash((str(src_dtype), str(dst_dtype), aligned)) & 0xFFFF)
    src = torch.randn(1 << 16, device="cuda").to(src_dtype)
    segs, n_dst = _segments(rng, src.numel(), aligned)
    dsts = [torch.full((n_dst,), -7.0, device="cuda", dtype=dst_dtype) for _ in range(3)]
    want = torch.full((n_dst,), -7.0, device="cuda", dtype=dst_dtype)
    apply_segments(src, segs, want)
    vec = m.policy_push(src, [d.data_ptr() for d in dsts], n_dst, dst_dtype == torch.bfloat16,
                        torch.tensor(segs, dtype=torch.int64))
    torch.cuda.synchronize()
    assert vec == (1 if not aligned else (4 if src_dtype == dst_dtype == torch.float32 else 8))
    for d in dsts:
        assert torch.equal(d, want)


def test_policy_push_rejects_out_of_bounds_segments():
    m = ops.ext()
    src = torch.zeros(1024, device="cuda", dtype=torch.bfloat16)
    dst = torch.zeros(1024, device="cuda", dtype=torch.bfloat16)
    bad_src = torch.tensor([[1000, 0, 1, 64, 64, 64]], dtype=torch.int64)
    bad_dst = torch.tensor([[0, 0, 4, 256, 256, 300]], dtype=torch.int64)
    with pytest.raises(RuntimeError, match="reads past src"):
        m.policy_push(src, [dst.data_ptr()], dst.numel(), True, bad_src)
    with pytest.raises(RuntimeError, match="writes past dst"):
        m.policy_push(src, [dst.data_ptr()], dst.numel(), True, bad_dst)


def _params_equal(a, b):
    for name, (off, n) in a.flat.offsets.items():
        assert torch.equal(a.flat.compute[off:off + n], b.flat.compute[off:off + n]), name


def _pt(**kw):
    from wavelet_b200.configs.config import RLPolicyTransferConfig

    return RLPolicyTransferConfig(**{"type": "nccl", "nccl_timeout_seconds": 60, **kw})


def test_exporter_to_receiver_in_one_process(tmp_path):
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.transport.policy import DevicePolicyReceiver, PolicyExporter, load_policy_into

    cfg = PRESETS["tiny-moe-gpu"]
    gen = build_model(cfg, "cuda", torch.bfloat16, seed=0, with_grad=False, with_optimizer=False)
    rec = DevicePolicyReceiver(gen, tmp_path, _pt(), index=0)
    trainer = build_model(cfg, "cuda", torch.bfloat16, seed=3)
    exp = PolicyExporter(tmp_path, _pt(), rank=0)
    for step in (0, 1, 2):
        with torch.no_grad():
            trainer.flat.compute.mul_(1.5)
        d = exp.export(trainer, step)
        assert json.loads((d / "update_info.json").read_text())["protocol"] == "peer_v1"
        assert load_policy_into(gen, d, rec, step)["loaded_step"] == step
        _params_equal(gen, trainer)
    assert sorted(rec.peer.epochs()) == [2, 3]
    exp.close()
    rec.close()


def _generator_proc(out_dir, res):
    from pathlib import Path

    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.transport.policy import DevicePolicyReceiver, load_policy_into
    from wavelet_b200.transport.queue import STABLE, step_dir

    out = Path(out_dir)
    gen = build_model(PRESETS["tiny-gpu"], "cuda", torch.bfloat16, seed=0, with_grad=False, with_optimizer=False)
    rec = DevicePolicyReceiver(gen, out, _pt(), index=0)
    d = step_dir(out / "policies", 2)
    t0 = time.monotonic()
    while not (d / STABLE).exists() and time.monotonic() - t0 < 120:
        time.sleep(0.02)
    meta = load_policy_into(gen, d, rec, 2)
    torch.save({"w": {n: gen.flat.view(n).cpu() for n in gen.flat.names()}, "step": meta["loaded_step"]}, res)
    done = out / "trainer-closed"
    t0 = time.monotonic()
    while not done.exists() and time.monotonic() - t0 < 120:  # the trainer unmaps before the slots are freed
        time.sleep(0.02)
    rec.close()


def test_push_into_another_process_through_ipc(tmp_path):
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.transport.policy import PolicyExporter

    out = tmp_path / "run"
    res = str(tmp_path / "gen.pt")
    ctx = mp.get_context("spawn")
    child = ctx.Process(target=_generator_proc, args=(str(out), res))
    child.start()
    try:
        trainer = build_model(PRESETS["tiny-gpu"], "cuda", torch.bfloat16, seed=5)
        exp = PolicyExporter(out, _pt(), rank=0)
        exp.export(trainer, 2)  # waits (bounded) for the generator's receiver to be announced
        assert exp.device_mode == "peer" and exp.last_update["receivers"] == 1
        exp.close()
    finally:
        (out / "trainer-closed").parent.mkdir(parents=True, exist_ok=True)
        (out / "trainer-closed").touch()
        child.join(180)
    assert child.exitcode == 0
    got = torch.load(res)
    assert got["step"] == 2
    for n in trainer.flat.names():
        assert torch.equal(got["w"][n], trainer.flat.view(n).cpu()), n
