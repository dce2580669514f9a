"""Loading a Hugging Face checkpoint into parallel layouts: a tensor-parallel
rank gets its Megatron part of every split parameter, an expert-parallel rank
its block of experts, a ZeRO-3 rank its shard — each equal to the same part
of the full model."""

import torch

from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.hf_io import load_hf_weights, save_hf
from wavelet_b200.models.qwen import build_model, tp_slicers


def _full(preset, tmp_path):
    m = build_model(PRESETS[preset], "cpu", torch.float32, seed=21)
    save_hf(m, tmp_path / "ck", dtype=torch.float32)
    return m


def test_tp2_ranks_load_their_parts(tmp_path):
    cfg = PRESETS["tiny"]
    full = _full("tiny", tmp_path)
    for r in range(2):
        part = build_model(cfg, "cpu", torch.float32, seed=99, tp=(2, r))
        load_hf_weights(part, tmp_path / "ck")
        sl = tp_slicers(cfg, 2, r)
        for n in part.flat.names():
            suffix = n.split(".", 1)[-1]
            want = sl[suffix][1](full.flat.view(n)) if suffix in sl else full.flat.view(n)
            torch.testing.assert_close(part.flat.view(n), want, rtol=0, atol=0, msg=n)


def test_ep2_ranks_load_their_experts(tmp_path):
    cfg = PRESETS["tiny-moe"]
    full = _full("tiny-moe", tmp_path)
    el = cfg.num_experts // 2
    for r in range(2):
        part = build_model(cfg, "cpu", torch.float32, seed=99, ep=(2, r, 0, 1))
        load_hf_weights(part, tmp_path / "ck")
        for n in part.expert_flat.names():
            torch.testing.assert_close(part.expert_flat.view(n), full.flat.view(n)[r * el:(r + 1) * el],
                                       rtol=0, atol=0, msg=n)
        for n in part.flat.names():
            torch.testing.assert_close(part.flat.view(n), full.flat.view(n), rtol=0, atol=0, msg=n)


def test_zero3_shards_load_their_elements(tmp_path):
    cfg = PRESETS["tiny"]
    full = _full("tiny", tmp_path)
    for r in range(3):
        part = build_model(cfg, "cpu", torch.float32, seed=99, dp_rank=r, dp_world=3, shard_params=True)
        load_hf_weights(part, tmp_path / "ck")
        f = part.flat
        for n, (off, k) in f.offsets.items():
            rr = f.local_range(off, k)
            if rr is None:
                continue
            ll, lh, tl, th = rr
            torch.testing.assert_close(f.compute[ll:lh], full.flat.view(n).reshape(-1)[tl:th], rtol=0, atol=0, msg=n)
