"""Context parallelism on 2 GPUs (NCCL all-gather of K/V, tcgen05 attention
over separate key sequences, reduce-scatter of dK/dV) against the same packed
micro-batch on one GPU: loss and summed gradients."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    from wavelet_b200.data.fake import synthetic_sft_microbatches
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.context_parallel import shard_batch
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        cfg = PRESETS["tiny-gpu"]
        (b,) = synthetic_sft_microbatches(1, 2048, cfg.vocab_size, seed=7, seqs_per_micro=3)
        scale = 1.0 / float(b.loss_mask.sum())
        cpm = build_model(cfg, dev, torch.bfloat16, seed=13)
        local = shard_batch(b, world, rank, dist.group.WORLD, align=128).to(dev)
        lc = Engine(cpm, AdamWHyper()).sft_micro_step(local, scale).detach().clone()
        dist.all_reduce(lc)
        g = cpm.flat.grad.clone()
        dist.all_reduce(g)
        full = build_model(cfg, dev, torch.bfloat16, seed=13)
        lf = Engine(full, AdamWHyper()).sft_micro_step(b.to(dev), scale)
        torch.cuda.synchronize()
        assert abs(lc.item() - lf.item()) < 1e-2 * abs(lf.item()) + 1e-4, (lc.item(), lf.item())
        for n in full.flat.names():
            a, r = g[full.flat.offsets[n][0]:][: full.flat.offsets[n][1]], full.flat.grad_view(n).reshape(-1)
            cos = torch.nn.functional.cosine_similarity(a.float(), r.float(), dim=0).item()
            rel = ((a.float() - r.float()).norm() / (r.float().norm() + 1e-12)).item()
            assert cos > 0.99 and rel < 0.1, (n, cos, rel)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()[-1500:]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_cp2_model_matches_single_gpu():
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
