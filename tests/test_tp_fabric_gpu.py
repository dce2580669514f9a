"""Fused GEMM -> all-reduce (tcgen05 GEMM whose epilogue stores into the
peers' receive buffers, then a rank-ordered local sum) against an fp32
PyTorch reference: one GPU (a one-rank fabric) and two GPUs."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, w, b_mn, res=None):
    y = a.float() @ (w.float() if b_mn else w.float().t())
    return y if res is None else y + res.float()


@pytest.mark.parametrize("M,N,K,b_mn", [(256, 512, 320, False), (200, 136, 192, True), (4096, 3584, 1792, False)])
def test_gemm_allreduce_one_rank(cuda_ext, M, N, K, b_mn):
    from wavelet_b200.parallel.fabric import Fabric
    from wavelet_b200.parallel.tp_fabric import TPFabric

    fab = Fabric(0, 1, torch.device("cuda", 0))
    tpf = TPFabric(fab, capacity=1024)
    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(K, N, device="cuda", generator=g) if b_mn else torch.randn(N, K, device="cuda", generator=g))
    w = (w * 0.05).bfloat16()
    res = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    for r in (None, res):
        out = tpf.gemm_allreduce(a, w, b_mn=b_mn, res=r)
        torch.cuda.synchronize()
        ref = _ref(a, w, b_mn, r)
        err = (out.float() - ref).abs().max().item()
        assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err
    fab.check()
    fab.close()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    from wavelet_b200.parallel.fabric import Fabric
    from wavelet_b200.parallel.tp_fabric import TPFabric

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        fab = Fabric(rank, world, dev)
        tpf = TPFabric(fab, capacity=4096)
        M, N, K = 1024, 768, 512
        g = torch.Generator(device=dev).manual_seed(5)
        A = [torch.randn(M, K, device=dev, generator=g).bfloat16() for _ in range(world)]
        W = [(torch.randn(N, K, device=dev, generator=g) * 0.05).bfloat16() for _ in range(world)]
        res = torch.randn(M, N, device=dev, generator=g).bfloat16()
        outs = []
        for it in range(3):  # alternate receive buffers, one growth on the first call
            out = tpf.gemm_allreduce(A[rank], W[rank], res=res)
            outs.append(out)
        torch.cuda.synchronize()
        fab.check()
        ref = sum(_ref(A[r], W[r], False) for r in range(world)) + res.float()
        for out in outs:
            err = (out.float() - ref).abs().max().item()
            assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err
        # every rank holds the identical result
        other = [torch.empty_like(outs[0]) for _ in range(world)]
        dist.all_gather(other, outs[0])
        assert all(torch.equal(o, other[0]) for o in other)
        fab.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()[-1500:]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemm_allreduce_two_ranks():
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
