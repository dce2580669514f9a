"""Expert-parallel policy refresh over peer memory: a full-weight generator
replica re-formed from every rank's expert shard equals the unsharded model,
before and after an optimizer update (2 GPUs)."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.fabric import Fabric
    from wavelet_b200.parallel.policy_sync import ExpertPolicySync

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        cfg = PRESETS["tiny-moe-gpu"]
        fab = Fabric(rank, world, dev)
        ep = build_model(cfg, dev, torch.bfloat16, seed=21, ep=(world, rank, 0, 1), ep_fabric=fab)
        full = build_model(cfg, dev, torch.bfloat16, seed=21)
        gen = build_model(cfg, dev, torch.bfloat16, init=False, with_grad=False, with_optimizer=False)
        sync = ExpertPolicySync(ep, gen, fab)
        sync.refresh()
        torch.cuda.synchronize()
        assert torch.equal(gen.flat.compute, full.flat.compute)
        # a rank-specific update of the expert shards shows up in every replica
        with torch.no_grad():
            ep.expert_flat.compute.add_(float(rank + 1))
        torch.cuda.synchronize()
        dist.barrier()
        sync.refresh()
        torch.cuda.synchronize()
        El = cfg.num_experts // world
        for n in ep.expert_flat.names():
            g = gen.flat.view(n)
            for r in range(world):
                want = (full.flat.view(n)[r * El:(r + 1) * El].float() + (r + 1)).to(torch.bfloat16)
                assert torch.equal(g[r * El:(r + 1) * El], want), n
        fab.check()
        fab.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()[-1500:]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_policy_refresh():
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
