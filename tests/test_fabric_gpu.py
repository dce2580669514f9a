"""Peer-memory fabric and the fused reduce-scatter / AdamW / all-gather step.

On one GPU the collective kernels are checked by handing them several local
buffers as the "ranks" (no kernel waits on another launch); with two or more
GPUs a two-process run compares the fused step against the NCCL path.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _bufs(fab, n, dtype, k):
    return [fab.alloc(n, dtype) for _ in range(k)]


def test_rs_and_adamw_allgather_emulated_ranks(cuda_ext):
    from wavelet_b200.parallel.fabric import Fabric

    fab = Fabric(0, 1, torch.device("cuda", 0))
    W, n = 3, 1 << 16
    torch.manual_seed(0)
    grads = _bufs(fab, W * n, torch.float32, W)
    for b in grads:
        b.tensor.copy_(torch.randn(W * n, device="cuda"))
    lo = n  # shard 1
    out = torch.empty(n, device="cuda")
    stats = torch.zeros(2, device="cuda")
    cuda_ext.rs_sum_sumsq([b.ptrs[0] for b in grads], W, lo, n, 0.5, out, stats)
    ref = 0.5 * sum(b.tensor[lo : lo + n] for b in grads)
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(stats[0], ref.pow(2).sum(), rtol=1e-4, atol=0)
    assert stats[1].item() == 0
    # AdamW + all-gather into three "ranks'" compute buffers
    comp = _bufs(fab, W * n, torch.bfloat16, W)
    master = torch.randn(n, device="cuda")
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    tot = torch.tensor([1.0, 0.0, 0.25], device="cuda")
    mref, gref = master.clone(), out * 0.25
    cuda_ext.adamw_allgather([b.ptrs[0] for b in comp], W, lo, master, out, m, v, 1e-2, 0.9, 0.999, 1e-8, 0.1, 1, tot)
    p = mref * (1 - 1e-2 * 0.1)
    mm = 0.1 * gref
    vv = 0.001 * gref * gref
    p = p - (1e-2 / 0.1) * mm / ((vv / 0.001).sqrt() + 1e-8)
    torch.testing.assert_close(master, p, rtol=1e-5, atol=1e-6)
    for b in comp:
        torch.testing.assert_close(b.tensor[lo : lo + n].float(), p.to(torch.bfloat16).float())
        assert torch.all(b.tensor[:lo] == 0)
    # non-finite totals: no update, parameters re-broadcast unchanged
    before = master.clone()
    cuda_ext.adamw_allgather([b.ptrs[0] for b in comp], W, lo, master, out, m, v, 1e-2, 0.9, 0.999, 1e-8, 0.1, 2,
                             torch.tensor([1.0, 3.0, 1.0], device="cuda"))
    torch.testing.assert_close(master, before)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    fab.close()


def test_barrier_times_out_without_peer(cuda_ext):
    """A peer that never signals: the bounded wait gives up and reports."""
    from wavelet_b200.parallel.fabric import ERR_TIMEOUT_PEER, Fabric

    fab = Fabric(0, 1, torch.device("cuda", 0))
    ghost = fab.alloc(256, torch.int32)  # stands in for rank 1's pad; nothing ever writes slot 1 of ours
    cuda_ext.clear_error(0)
    cuda_ext.peer_barrier([fab.pads.ptrs[0], ghost.ptrs[0]], 0, 2, 1, 0, 0.2)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) & ERR_TIMEOUT_PEER
    cuda_ext.clear_error(0)
    # the context is still usable
    x = torch.ones(4, device="cuda")
    assert x.sum().item() == 4
    fab.close()


def test_fused_step_world1_matches_nccl_path(cuda_ext):
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.fabric import Fabric
    from wavelet_b200.parallel.zero import AdamWHyper, FusedShardedAdamW, ShardedAdamW

    cfg = PRESETS["tiny-gpu"]
    fab = Fabric(0, 1, torch.device("cuda", 0))
    a = build_model(cfg, "cuda", torch.bfloat16, seed=3, fabric=fab)
    b = build_model(cfg, "cuda", torch.bfloat16, seed=3)
    h = AdamWHyper(lr=1e-3, weight_decay=0.01, max_grad_norm=0.5)
    oa, ob = FusedShardedAdamW(a.flat, h, fab), ShardedAdamW(b.flat, h)
    for it in range(3):
        g = torch.randn(a.flat.numel, device="cuda") * (it + 1)
        a.flat.grad.copy_(g)
        b.flat.grad.copy_(g)
        ra, rb = oa.step(), ob.step()
        assert abs(ra["grad_norm"] - rb["grad_norm"]) / rb["grad_norm"] < 1e-4
        torch.testing.assert_close(a.flat.master, b.flat.master, rtol=1e-6, atol=1e-7)
        # masters agree to ~1 fp32 ulp, so a few bf16 roundings may flip by one bf16 ulp
        torch.testing.assert_close(a.flat.compute.float(), b.flat.compute.float(), rtol=8e-3, atol=1e-6)
        assert torch.equal(a.flat.compute, a.flat.master.to(torch.bfloat16))
    fab.close()


def test_fused_step_skips_an_overflowing_norm(cuda_ext):
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.fabric import Fabric
    from wavelet_b200.parallel.zero import AdamWHyper, FusedShardedAdamW, NonFiniteGradientError

    fab = Fabric(0, 1, torch.device("cuda", 0))
    a = build_model(PRESETS["tiny-gpu"], "cuda", torch.bfloat16, seed=3, fabric=fab)
    opt = FusedShardedAdamW(a.flat, AdamWHyper(lr=1e-3, max_grad_norm=1.0), fab)
    master, compute = a.flat.master.clone(), a.flat.compute.clone()
    a.flat.grad.fill_(1e30)  # finite elements, fp32 sum of squares overflows
    with pytest.raises(NonFiniteGradientError):
        opt.step()
    assert torch.equal(a.flat.master, master) and torch.equal(a.flat.compute, compute)
    assert opt.step_count == 0
    fab.close()


def _two_rank_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.fabric import Fabric
    from wavelet_b200.parallel.zero import AdamWHyper, FusedShardedAdamW, ShardedAdamW

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        cfg = PRESETS["tiny-gpu"]
        fab = Fabric(rank, world, dev)
        a = build_model(cfg, dev, torch.bfloat16, dp_rank=rank, dp_world=world, seed=5, fabric=fab)
        b = build_model(cfg, dev, torch.bfloat16, dp_rank=rank, dp_world=world, seed=5)
        h = AdamWHyper(lr=1e-3, weight_decay=0.01, max_grad_norm=1.0)
        oa, ob = FusedShardedAdamW(a.flat, h, fab), ShardedAdamW(b.flat, h, None, world)
        gen = torch.Generator(device=dev)
        for it in range(3):
            gen.manual_seed(100 * it + rank)
            g = torch.randn(a.flat.numel, device=dev, generator=gen)
            a.flat.grad.copy_(g)
            b.flat.grad.copy_(g)
            ra, rb = oa.step(), ob.step()
            assert abs(ra["grad_norm"] - rb["grad_norm"]) / rb["grad_norm"] < 1e-4, (ra, rb)
            torch.testing.assert_close(a.flat.master, b.flat.master, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(a.flat.compute.float(), b.flat.compute.float(), rtol=8e-3, atol=1e-6)
        torch.cuda.synchronize()
        fab.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_step_two_ranks_matches_nccl():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
