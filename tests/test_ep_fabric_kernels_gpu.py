"""Expert-parallel row kernels on one GPU with several local buffers standing
in for the ranks (no kernel waits on another launch)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_rows_scatter_and_gather_sum(cuda_ext):
    from wavelet_b200.parallel.fabric import Fabric

    fab = Fabric(0, 1, torch.device("cuda", 0))
    W, H, T, k, R = 3, 256, 50, 2, 400
    bufs = [fab.alloc(R * H, torch.bfloat16) for _ in range(W)]
    for b in bufs:
        b.tensor.zero_()
    ptrs = [b.ptrs[0] for b in bufs]
    torch.manual_seed(0)
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    n = T * k
    src = torch.arange(T, device="cuda").repeat_interleave(k)
    rank = torch.randint(0, W, (n,), device="cuda", dtype=torch.int32)
    row = torch.randperm(R, device="cuda")[:n].to(torch.int64)  # distinct rows
    scale = torch.rand(n, device="cuda")
    cuda_ext.rows_scatter(x, src, rank, row, scale, ptrs, W, H)
    views = [b.tensor.view(R, H) for b in bufs]
    for i in range(0, n, 7):
        want = (x[src[i]].float() * scale[i]).to(torch.bfloat16)
        torch.testing.assert_close(views[int(rank[i])][int(row[i])], want)
    # gather-sum back with weights and a residual, bf16 and fp32 outputs
    w = torch.rand(n, device="cuda")
    res = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    cuda_ext.rows_gather_sum(ptrs, W, H, rank, row, w, k, res, out)
    out32 = torch.empty(T, H, device="cuda", dtype=torch.float32)
    cuda_ext.rows_gather_sum(ptrs, W, H, rank, row, None, k, None, out32)
    ref = res.float().clone()
    ref32 = torch.zeros(T, H, device="cuda")
    for i in range(n):
        v = views[int(rank[i])][int(row[i])].float()
        ref[i // k] += w[i] * v
        ref32[i // k] += v
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(out32, ref32, rtol=1e-5, atol=1e-5)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    fab.close()
