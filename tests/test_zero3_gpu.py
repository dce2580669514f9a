"""ZeRO-3 on B200s: sharded bf16 weights gathered layer by layer give the
losses of the replicated-weights store, on one GPU (local gathers) and over
2 GPUs (NCCL broadcasts / reductions with prefetch on the side)."""

import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _train(model, steps=3, micro=2, seed=1, rank=0, world=1, group=None):
    from wavelet_b200.data.fake import synthetic_sft_microbatches
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    eng = Engine(model, AdamWHyper(lr=1e-3), dp_group=group, dp_world=world)
    bs = [b.to("cuda") for b in synthetic_sft_microbatches(micro, 512, model.cfg.vocab_size, seed=seed + 17 * rank,
                                                           seqs_per_micro=2)]
    n = torch.tensor([float(sum(b.loss_mask.sum() for b in bs))], device="cuda")
    if world > 1:
        dist.all_reduce(n, group=group)
    losses = []
    for _ in range(steps):
        tot = torch.zeros((), device="cuda")
        for b in bs:
            tot += eng.sft_micro_step(b, 1.0 / float(n))
        eng.optimizer_step(1e-3)
        losses.append(float(tot))
    return losses


def test_zero3_one_gpu_matches_replicated(cuda_ext):
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero3 import ParamGatherer

    cfg = PRESETS["tiny-moe-gpu"]
    a = _train(build_model(cfg, "cuda", torch.bfloat16, seed=3))
    m = build_model(cfg, "cuda", torch.bfloat16, seed=3, shard_params=True)
    ParamGatherer(m)
    b = _train(m)
    for x, y in zip(a, b):
        assert abs(x - y) <= 2e-3 * abs(x), (a, b)
    assert cuda_ext.read_error(0) == 0


def _worker(rank, world, init_file, res, shard):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero3 import ParamGatherer

    cfg = PRESETS["tiny-gpu"]
    m = build_model(cfg, "cuda", torch.bfloat16, dp_rank=rank, dp_world=world, seed=3, shard_params=shard)
    if shard:
        ParamGatherer(m, group=dist.group.WORLD)
        assert m.flat.compute.numel() == m.flat.shard_numel
    losses = _train(m, rank=rank, world=world, group=dist.group.WORLD)
    if rank == 0:
        torch.save(losses, res)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero3_two_gpus_matches_replicated():
    out = []
    for shard in (False, True):
        with tempfile.TemporaryDirectory() as d:
            res = os.path.join(d, "res.pt")
            mp.spawn(_worker, args=(2, os.path.join(d, "init"), res, shard), nprocs=2, join=True)
            out.append(torch.load(res))
    a, b = out
    for x, y in zip(a, b):
        assert abs(x - y) <= 2e-3 * abs(x), (a, b)
