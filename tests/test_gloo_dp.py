"""Plumbing configuration: tiny decoder SFT on CPU/gloo, world_size=2, sharded
data parallel (2 layers, hidden 128, 4/2 heads x 32, SwiGLU 512, vocab 1024,
RMSNorm, RoPE 1e4, fp32, N(0, 0.02) init, batch 8 x 128 seed-generated tokens
in [3, 1024), loss on the second half of each sequence, AdamW lr 1e-3, 10
steps).  The 2-rank run must match a single-process run on the same global
batch step for step."""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batch(B=8, S=128, vocab=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(3, vocab, (B, S), generator=g)
    return ids


def _packed(ids):
    from wavelet_b200.data.sft import pack

    S = ids.shape[1]
    masks = []
    for _ in range(ids.shape[0]):
        m = torch.zeros(S)
        m[S // 2 :] = 1
        masks.append(m)
    return pack(list(ids), masks)


def _train(rank, world, steps, init_file, out):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    if world > 1:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    torch.manual_seed(0)
    cfg = PRESETS["tiny"]
    m = build_model(cfg, "cpu", torch.float32, dp_rank=rank, dp_world=world, seed=0)
    eng = Engine(m, AdamWHyper(lr=1e-3, max_grad_norm=1.0), dp_group=None, dp_world=world)
    ids = _batch()
    per = ids.shape[0] // world
    mine = _packed(ids[rank * per : (rank + 1) * per])
    losses = []
    for _ in range(steps):
        local = float(mine.loss_mask.sum())
        total = eng.global_token_count(local, torch.device("cpu"))
        loss = eng.sft_micro_step(mine, 1.0 / total)
        if world > 1:
            dist.all_reduce(loss)
        eng.optimizer_step(1e-3)
        losses.append(loss.item())
    if rank == 0:
        torch.save({"losses": losses, "w": m.flat.compute.detach().clone()}, out)
    if world > 1:
        dist.destroy_process_group()


def test_tiny_sft_gloo_world2_matches_single_process():
    with tempfile.TemporaryDirectory() as d:
        f1 = os.path.join(d, "w1.pt")
        f2 = os.path.join(d, "w2.pt")
        _train(0, 1, 10, None, f1)
        mp.spawn(_train, args=(2, 10, os.path.join(d, "init"), f2), nprocs=2, join=True)
        a = torch.load(f1)
        b = torch.load(f2)
        assert a["losses"][-1] < a["losses"][0] - 0.5, a["losses"]
        for x, y in zip(a["losses"], b["losses"]):
            assert abs(x - y) < 1e-4 * max(1.0, abs(x)), (a["losses"], b["losses"])
        assert (a["w"] - b["w"]).abs().max().item() < 1e-3, (a["w"] - b["w"]).abs().max().item()
