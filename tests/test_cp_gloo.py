"""Context parallelism on 2 gloo CPU ranks: every packed sequence is padded,
cut into 2*cp chunks and load-balanced over the ranks; attention runs over
the all-gathered keys with bottom-right causal alignment and dK/dV are
reduce-scattered back.  Loss and (summed) gradients match the unsplit batch."""

import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batch(cfg):
    from wavelet_b200.data.fake import synthetic_sft_microbatches

    (b,) = synthetic_sft_microbatches(1, 96, cfg.vocab_size, seed=4, seqs_per_micro=3)
    return b


def _worker(rank, world, init_file, out):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.context_parallel import shard_batch
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    cfg = PRESETS["tiny"]
    m = build_model(cfg, "cpu", torch.float32, seed=9)
    b = _batch(cfg)
    local = shard_batch(b, world, rank, dist.group.WORLD, align=8)
    assert local.num_tokens % 16 == 0 and float(local.loss_mask.sum()) > 0
    loss = Engine(m, AdamWHyper()).sft_micro_step(local, 1.0 / float(b.loss_mask.sum()))
    loss = loss.detach().clone()
    dist.all_reduce(loss)
    g = m.flat.grad.clone()
    dist.all_reduce(g)
    torch.save({"loss": float(loss), "grad": g}, f"{out}.{rank}")
    dist.destroy_process_group()


def test_cp2_matches_unsplit():
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, os.path.join(d, "init"), os.path.join(d, "res")), nprocs=world, join=True)
        got = [torch.load(os.path.join(d, f"res.{r}")) for r in range(world)]
    cfg = PRESETS["tiny"]
    ref = build_model(cfg, "cpu", torch.float32, seed=9)
    ref.fused_cpu = True
    b = _batch(cfg)
    loss = Engine(ref, AdamWHyper()).sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    for r in range(world):
        assert abs(got[r]["loss"] - float(loss)) < 1e-4 * abs(float(loss)) + 1e-6, (got[r]["loss"], float(loss))
        torch.testing.assert_close(got[r]["grad"], ref.flat.grad, rtol=1e-3, atol=1e-6)


def test_shard_layout():
    """Chunk pairing and key prefixes of the plan (host-only)."""
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.parallel.context_parallel import shard_batch

    cfg = PRESETS["tiny"]
    b = _batch(cfg)
    cp = 2
    lens = (b.cu_seqlens[1:] - b.cu_seqlens[:-1]).tolist()
    for r in range(cp):
        loc = shard_batch(b, cp, r, None, align=8)
        p = loc.cp
        C = [(-(-L // (2 * cp * 8))) * 8 for L in lens]
        assert p.TA == sum(C) and p.T == 2 * sum(C)
        assert p.cu_k[0][1:].sub(p.cu_k[0][:-1]).tolist() == [(r + 1) * c for c in C]
        assert p.cu_k[1][1:].sub(p.cu_k[1][:-1]).tolist() == [(2 * cp - r) * c for c in C]
        # positions: chunk r then chunk 2cp-1-r of the first sequence
        first = int(b.position_ids[0])
        assert int(loc.position_ids[0]) == first + r * C[0]
        assert int(loc.position_ids[p.TA]) == first + (2 * cp - 1 - r) * C[0]
