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



def test_weighted_norm_boundary(cuda_ext):
    """Elements below the boundary enter the squared norm with weight w_lo
    (tensor-parallel replicated parameters); the reduced values are unchanged."""
    from wavelet_b200.parallel.fabric import Fabric

    fab = Fabric(0, 1, torch.device("cuda", 0))
    W, n = 2, 1 << 15
    grads = _bufs(fab, W * n, torch.float32, W)
    torch.manual_seed(1)
    for b in grads:
        b.tensor.copy_(torch.randn(W * n, device="cuda"))
    lo, w_end = n, n + 4096
    out = torch.empty(n, device="cuda")
    stats = torch.zeros(2, device="cuda")
    cuda_ext.rs_sum_sumsq([b.ptrs[0] for b in grads], W, lo, n, 1.0, out, stats, w_end, 0.5)
    ref = sum(b.tensor[lo : lo + n] for b in grads)
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
    want = 0.5 * ref[:4096].pow(2).sum() + ref[4096:].pow(2).sum()
    torch.testing.assert_close(stats[0], want, rtol=1e-4, atol=0)
    fab.close()


def test_fabric_waits_run_out_and_report(cuda_ext):
    """A bounded device-side wait that no peer ever satisfies ends after its
    budget: the barrier and the norm exchange set the timeout bit of the error
    word (the norm exchange also marks the step non-finite, so no rank would
    update), ``Fabric.check`` raises ``PeerTimeoutError``, and the context stays
    usable.  The "peer" is a second local pad that nothing writes, so no other
    process or launch is involved."""
    import time

    from wavelet_b200.parallel.fabric import ERR_TIMEOUT_PEER, SLOT_BARRIER, SLOT_NORM, Fabric, PeerTimeoutError

    dev = torch.device("cuda", 0)
    fab = Fabric(0, 1, dev, budget_s=0.05)
    ghost = fab.alloc(256, torch.int32)  # pad of a "rank 1" that never signals
    pads = [fab.pads.ptrs[0], ghost.ptrs[0]]
    cuda_ext.clear_error(0)
    t0 = time.time()
    cuda_ext.peer_barrier(pads, 0, 2, 7, SLOT_BARRIER, 0.05)
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    assert cuda_ext.read_error(0) & ERR_TIMEOUT_PEER
    with pytest.raises(PeerTimeoutError):
        fab.check()
    assert cuda_ext.read_error(0) == 0  # check() cleared it
    stats = torch.tensor([4.0, 0.0], device=dev)
    tot = torch.zeros(3, device=dev)
    cuda_ext.norm_exchange(pads, 0, 2, 9, stats, 1.0, tot, 0.05)
    torch.cuda.synchronize()
    assert tot[1].item() > 0  # a missing peer reads as a non-finite step: nobody updates
    assert cuda_ext.read_error(0) & ERR_TIMEOUT_PEER
    with pytest.raises(PeerTimeoutError):
        fab.check()
    # the context is still usable after the timeouts
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2
    fab.close()


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
    with pytest.raises(NonFiniteGradientError, match="overflows"):
        opt.step()
    assert torch.equal(a.flat.master, master) and torch.equal(a.flat.compute, compute)
    assert opt.step_count == 0
    # clipping off: the norm is not used and the finite gradients update
    opt_nc = FusedShardedAdamW(a.flat, AdamWHyper(lr=1e-3, max_grad_norm=0.0), fab)
    a.flat.grad.fill_(1e18)  # each square is finite in fp32, their sum is not
    out = opt_nc.step()
    assert out["clip_factor"] == 1.0 and opt_nc.step_count == 1
    assert torch.isfinite(a.flat.master).all() and not torch.equal(a.flat.master, master)
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
